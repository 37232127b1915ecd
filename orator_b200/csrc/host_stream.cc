// Streaming front door over AsrSessionPool (include/orator_b200/asr_stream.h).
#include "orator_b200/asr_stream.h"

#include <algorithm>
#include <stdexcept>

namespace orator {
namespace model {

using K = AsrStreamTokens;

AsrStreamPool::AsrStreamPool(const AsrTextDecoder& weights, AsrSessionPool& pool, int max_new,
                             int ban_steps, int eos0, int eos1)
    : w_(weights), pool_(pool), max_new_(max_new), ban_steps_(ban_steps), eos0_(eos0), eos1_(eos1) {}

std::vector<int> AsrStreamPool::PrefixIds(const std::vector<int>& system_ids) {
  std::vector<int> ids = {K::kImStart, K::kSystem, K::kNewline};
  ids.insert(ids.end(), system_ids.begin(), system_ids.end());
  ids.insert(ids.end(), {K::kImEnd, K::kNewline, K::kImStart, K::kUser, K::kNewline,
                         K::kAudioStart});
  return ids;
}

std::vector<int> AsrStreamPool::SuffixIds(const Request& r) {
  std::vector<int> ids = {K::kAudioEnd, K::kImEnd, K::kNewline, K::kImStart, K::kAssistant,
                          K::kNewline};
  ids.insert(ids.end(), r.language.begin(), r.language.end());
  ids.push_back(K::kAsrText);
  ids.insert(ids.end(), r.committed.begin(), r.committed.end());
  return ids;
}

std::vector<float> AsrStreamPool::EmbedRows(const std::vector<int>& ids) const {
  const int H = w_.hidden_size();
  std::vector<float> rows(ids.size() * static_cast<size_t>(H));
  for (size_t i = 0; i < ids.size(); ++i) w_.Embed(ids[i], rows.data() + i * H);
  return rows;
}

int AsrStreamPool::Open(const std::vector<int>& system_ids, cudaStream_t stream) {
  const int sid = pool_.CreateSession();
  const std::vector<int> ids = PrefixIds(system_ids);
  const std::vector<float> rows = EmbedRows(ids);
  pool_.PrefillAt(sid, rows.data(), static_cast<int>(ids.size()), stream);
  ckpt_[sid] = static_cast<int>(ids.size());
  return sid;
}

void AsrStreamPool::Close(int session) {
  pool_.FreeSession(session);
  ckpt_.erase(session);
}

void AsrStreamPool::AppendAudio(const std::vector<int>& sessions,
                                const std::vector<const float*>& rows,
                                const std::vector<int>& lens, cudaStream_t stream) {
  if (sessions.size() != rows.size() || sessions.size() != lens.size())
    throw std::runtime_error("AppendAudio: sessions, rows and lens differ in size");
  const size_t H = w_.hidden_size();
  size_t total = 0;
  for (int n : lens) total += static_cast<size_t>(n);
  std::vector<float> cat(total * H);
  size_t off = 0;
  for (size_t i = 0; i < sessions.size(); ++i) {
    pool_.TruncateCache(sessions[i], ckpt_.at(sessions[i]));
    std::copy(rows[i], rows[i] + static_cast<size_t>(lens[i]) * H, cat.begin() + off);
    off += static_cast<size_t>(lens[i]) * H;
  }
  pool_.PrefillAt(sessions, lens, cat.data(), stream);
  for (size_t i = 0; i < sessions.size(); ++i) ckpt_[sessions[i]] += lens[i];
}

std::map<int, std::vector<int>> AsrStreamPool::Decode(const std::map<int, Request>& requests,
                                                      cudaStream_t stream) {
  std::map<int, std::vector<int>> out;
  if (requests.empty()) return out;
  std::vector<int> sids, lens;
  std::vector<float> cat;
  for (const auto& kv : requests) {
    const int sid = kv.first;
    pool_.TruncateCache(sid, ckpt_.at(sid));
    pool_.SetBan(sid, eos0_, eos1_, ban_steps_, stream);
    const std::vector<int> ids = SuffixIds(kv.second);
    const std::vector<float> rows = EmbedRows(ids);
    cat.insert(cat.end(), rows.begin(), rows.end());
    sids.push_back(sid);
    lens.push_back(static_cast<int>(ids.size()));
    out[sid] = {};
  }
  pool_.PrefillAt(sids, lens, cat.data(), stream);
  std::vector<int> pending = pool_.PendingTokens(sids, stream);
  std::map<int, int> pend, emitted;
  for (size_t i = 0; i < sids.size(); ++i) {
    pend[sids[i]] = pending[i];
    emitted[sids[i]] = 0;
  }
  // DecodeGreedy's output rule per token: an EOS id ends the output (not
  // included), six equal tokens in a row end it (included).
  auto push = [&](int sid, int t) {
    if (t == eos0_ || t == eos1_) return true;
    std::vector<int>& o = out[sid];
    o.push_back(t);
    if (o.size() >= 6) {
      for (size_t k = o.size() - 6; k < o.size(); ++k)
        if (o[k] != o.back()) return false;
      return true;
    }
    return false;
  };
  std::vector<int> active = max_new_ > 0 ? sids : std::vector<int>{};
  while (!active.empty()) {
    const std::vector<int> nxt = pool_.StepAll(active, stream);
    std::vector<int> still;
    for (size_t i = 0; i < active.size(); ++i) {
      const int s = active[i];
      ++emitted[s];
      const bool stop = push(s, pend[s]);
      pend[s] = nxt[i];
      if (!stop && emitted[s] < max_new_) still.push_back(s);
    }
    active.swap(still);
  }
  for (int sid : sids) {
    pool_.TruncateCache(sid, ckpt_.at(sid));
    pool_.SetBan(sid, -1, -1, 0, stream);
  }
  return out;
}

}  // namespace model
}  // namespace orator
