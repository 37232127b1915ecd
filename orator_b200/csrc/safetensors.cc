// Minimal mmap safetensors reader (single file or sharded directory with
// model.safetensors.index.json), the role io::SafeTensorReader /
// io::ShardedSafeTensors play for the reference loader
// (src/io/safetensor.cc, src/io/sharded_safetensor.cc).
#include "safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <fstream>
#include <set>
#include <sstream>
#include <stdexcept>

namespace orx {
namespace {

std::string read_file(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  if (!f) throw std::runtime_error("cannot open " + path);
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

struct Cursor {
  const std::string& s;
  size_t i = 0;
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  char peek() { ws(); return i < s.size() ? s[i] : '\0'; }
  void expect(char c) {
    if (peek() != c) throw std::runtime_error(std::string("json: expected ") + c);
    ++i;
  }
  std::string str() {
    expect('"');
    std::string out;
    while (i < s.size() && s[i] != '"') {
      if (s[i] == '\\' && i + 1 < s.size()) ++i;
      out.push_back(s[i++]);
    }
    ++i;
    return out;
  }
  int64_t num() {
    ws();
    size_t j = i;
    while (j < s.size() && (isdigit(static_cast<unsigned char>(s[j])) || s[j] == '-')) ++j;
    const int64_t v = std::stoll(s.substr(i, j - i));
    i = j;
    return v;
  }
  void skip() {  // skip any JSON value
    const char c = peek();
    if (c == '"') { str(); return; }
    if (c == '{' || c == '[') {
      const char open = c, close = c == '{' ? '}' : ']';
      int depth = 0;
      bool in_str = false;
      for (; i < s.size(); ++i) {
        if (in_str) { if (s[i] == '\\') ++i; else if (s[i] == '"') in_str = false; continue; }
        if (s[i] == '"') in_str = true;
        else if (s[i] == open) ++depth;
        else if (s[i] == close && --depth == 0) { ++i; return; }
      }
      return;
    }
    while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']') ++i;
  }
};

}  // namespace

SafeTensorsFile::SafeTensorsFile(const std::string& path) : path_(path) {
  fd_ = open(path.c_str(), O_RDONLY);
  if (fd_ < 0) throw std::runtime_error("cannot open " + path);
  struct stat st;
  fstat(fd_, &st);
  size_ = static_cast<size_t>(st.st_size);
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
  if (map_ == MAP_FAILED) throw std::runtime_error("mmap failed: " + path);
  uint64_t hlen = 0;
  std::memcpy(&hlen, map_, 8);
  if (hlen + 8 > size_) throw std::runtime_error("bad safetensors header: " + path);
  const std::string header(static_cast<const char*>(map_) + 8, hlen);
  const uint8_t* data = static_cast<const uint8_t*>(map_) + 8 + hlen;
  Cursor c{header};
  c.expect('{');
  while (c.peek() != '}') {
    const std::string name = c.str();
    c.expect(':');
    if (name == "__metadata__") {
      c.skip();
    } else {
      TensorView tv;
      c.expect('{');
      int64_t b = 0, e = 0;
      while (c.peek() != '}') {
        const std::string key = c.str();
        c.expect(':');
        if (key == "dtype") {
          tv.dtype = c.str();
        } else if (key == "shape") {
          c.expect('[');
          while (c.peek() != ']') {
            tv.shape.push_back(c.num());
            if (c.peek() == ',') c.expect(',');
          }
          c.expect(']');
        } else if (key == "data_offsets") {
          c.expect('[');
          b = c.num();
          c.expect(',');
          e = c.num();
          c.expect(']');
        } else {
          c.skip();
        }
        if (c.peek() == ',') c.expect(',');
      }
      c.expect('}');
      if (b < 0 || e < b || 8 + hlen + static_cast<uint64_t>(e) > size_)
        throw std::runtime_error("tensor out of file bounds: " + name);
      tv.data = data + b;
      tv.nbytes = static_cast<size_t>(e - b);
      tensors_[name] = tv;
    }
    if (c.peek() == ',') c.expect(',');
  }
}

SafeTensorsFile::~SafeTensorsFile() {
  if (map_ && map_ != MAP_FAILED) munmap(map_, size_);
  if (fd_ >= 0) close(fd_);
}

ShardedCheckpoint::ShardedCheckpoint(const std::string& dir) {
  const std::string idx = dir + "/model.safetensors.index.json";
  std::ifstream probe(idx);
  std::set<std::string> files;
  if (probe.good()) {
    const std::string j = read_file(idx);
    Cursor c{j};
    c.expect('{');
    while (c.peek() != '}') {
      const std::string key = c.str();
      c.expect(':');
      if (key == "weight_map") {
        c.expect('{');
        while (c.peek() != '}') {
          c.str();
          c.expect(':');
          files.insert(c.str());
          if (c.peek() == ',') c.expect(',');
        }
        c.expect('}');
      } else {
        c.skip();
      }
      if (c.peek() == ',') c.expect(',');
    }
  } else {
    files.insert("model.safetensors");
  }
  for (const auto& f : files) shards_.emplace_back(new SafeTensorsFile(dir + "/" + f));
}

std::vector<std::pair<std::string, TensorView>> ShardedCheckpoint::tensors() const {
  std::vector<std::pair<std::string, TensorView>> out;
  for (const auto& s : shards_)
    for (const auto& kv : s->tensors()) out.push_back(kv);
  return out;
}

}  // namespace orx
