// Minimal mmap safetensors reader used by the checkpoint loader.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace orx {

struct TensorView {
  std::string dtype;  // "BF16", "F32", ...
  std::vector<int64_t> shape;
  const void* data = nullptr;
  size_t nbytes = 0;
};

class SafeTensorsFile {
 public:
  explicit SafeTensorsFile(const std::string& path);
  ~SafeTensorsFile();
  const std::map<std::string, TensorView>& tensors() const { return tensors_; }

 private:
  std::string path_;
  int fd_ = -1;
  void* map_ = nullptr;
  size_t size_ = 0;
  std::map<std::string, TensorView> tensors_;
};

class ShardedCheckpoint {
 public:
  explicit ShardedCheckpoint(const std::string& dir);
  std::vector<std::pair<std::string, TensorView>> tensors() const;

 private:
  std::vector<std::unique_ptr<SafeTensorsFile>> shards_;
};

}  // namespace orx
