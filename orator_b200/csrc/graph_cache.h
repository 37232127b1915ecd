// Book-keeping for captured CUDA graphs keyed by batch size.
//
// A captured graph bakes in the device addresses of every buffer its kernels
// touch. When an owner reallocates any such buffer (a grown split-K workspace,
// grown row buffers), every graph captured before that point refers to freed
// memory and must never be replayed again. The owner counts those
// reallocations in one monotonically increasing "memory epoch"; each graph
// remembers the epoch it was captured under, and `find` hands out a graph only
// when its epoch is the current one. A graph of any other epoch is destroyed on
// sight, and `sync` drops all of them at once when the epoch moved, so no entry
// can outlive the buffers it was captured against (not even a graph for a
// batch size that is not looked up again for a long time).
//
// Header-only and independent of the CUDA runtime (the graph handle type and
// its destroy function are template parameters), so the rules are tested on
// the CPU with a fake handle.
#pragma once

#include <cstdint>
#include <map>
#include <set>

namespace orx {

template <class Exec, class Destroy>
class GraphCache {
 public:
  explicit GraphCache(Destroy destroy) : destroy_(destroy) {}
  ~GraphCache() { clear(); }
  GraphCache(const GraphCache&) = delete;
  GraphCache& operator=(const GraphCache&) = delete;

  // Drops every graph (and every "warmed" mark) when `epoch` differs from the
  // epoch the cache last saw. Call before any lookup in a step.
  void sync(uint64_t epoch) {
    if (epoch == epoch_) return;
    clear();
    epoch_ = epoch;
  }
  // The graph for `key` captured under `epoch`, or a null handle.
  Exec find(int key, uint64_t epoch) {
    sync(epoch);
    auto it = graphs_.find(key);
    if (it == graphs_.end()) return Exec{};
    if (it->second.epoch != epoch) {  // unreachable after sync; kept as a guard
      destroy_(it->second.exec);
      graphs_.erase(it);
      return Exec{};
    }
    return it->second.exec;
  }
  void insert(int key, uint64_t epoch, Exec e) {
    sync(epoch);
    auto it = graphs_.find(key);
    if (it != graphs_.end()) destroy_(it->second.exec);
    graphs_[key] = Entry{e, epoch};
  }
  // Whether `key` already ran once eagerly under the current epoch.
  bool warmed(int key) const { return warmed_.count(key) != 0; }
  void mark_warmed(int key) { warmed_.insert(key); }
  void clear() {
    for (auto& kv : graphs_) destroy_(kv.second.exec);
    graphs_.clear();
    warmed_.clear();
  }
  size_t size() const { return graphs_.size(); }
  uint64_t epoch() const { return epoch_; }

 private:
  struct Entry {
    Exec exec;
    uint64_t epoch;
  };
  Destroy destroy_;
  std::map<int, Entry> graphs_;
  std::set<int> warmed_;
  uint64_t epoch_ = 0;
};

}  // namespace orx
