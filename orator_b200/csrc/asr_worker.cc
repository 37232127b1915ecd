// AsrWorker / VadEvidenceStore / StreamBatcher (include/orator_b200/asr_worker.h).
//
// AsrWorker restates the reference's session scheduler
// (src/pipeline/asr_worker.cc:70-416): the VAD gate buffers audio ahead of
// the VAD decision frontier and feeds decided speech to the decoder in fixed
// quanta (with a lead before each onset and a trailing interval after the
// last speech), splits large spans into <= 8 s pieces, closes a segment at
// the trailing endpoint, the segment_sec cap or the max_audio_tokens cap, and
// publishes partial / final / retract events.
#include "orator_b200/asr_worker.h"

#include <algorithm>
#include <cstdio>
#include <limits>

namespace orator {
namespace pipeline {

// ---- VAD evidence -----------------------------------------------------------

void VadEvidenceStore::DepositVad(const VadSeg& seg) {
  if (!(std::isfinite(seg.start) && std::isfinite(seg.end) && seg.end > seg.start)) return;
  std::lock_guard<std::mutex> lock(mu_);
  for (const VadSeg& s : segs_)
    if (std::fabs(s.start - seg.start) < 1e-9 && std::fabs(s.end - seg.end) < 1e-9) return;
  auto at = std::lower_bound(segs_.begin(), segs_.end(), seg.start,
                             [](const VadSeg& s, double t) { return s.start < t; });
  segs_.insert(at, seg);
  ev_.segments = std::make_shared<const std::vector<VadSeg>>(segs_);
}

void VadEvidenceStore::AdvanceVadHorizon(double horizon_sec) {
  if (!std::isfinite(horizon_sec)) return;
  std::lock_guard<std::mutex> lock(mu_);
  ev_.horizon = std::max(ev_.horizon, horizon_sec);
}

void VadEvidenceStore::UpdateVadState(bool in_speech, double observed_at_sec,
                                      double active_start_sec, double active_horizon_sec) {
  if (!std::isfinite(observed_at_sec)) return;
  std::lock_guard<std::mutex> lock(mu_);
  if (observed_at_sec + 1e-9 < ev_.observed_at) return;  // stale update
  ev_.in_speech = in_speech;
  ev_.observed_at = observed_at_sec;
  const bool region = in_speech && std::isfinite(active_start_sec) &&
                      std::isfinite(active_horizon_sec) &&
                      active_horizon_sec + 1e-9 >= active_start_sec;
  ev_.active_start = region ? active_start_sec : -1e9;
  ev_.active_horizon = region ? active_horizon_sec : -1e9;
}

VadEvidenceStore::Evidence VadEvidenceStore::SnapshotVadEvidence() const {
  std::lock_guard<std::mutex> lock(mu_);
  return ev_;
}

// ---- AsrWorker ----------------------------------------------------------------

namespace {

using Clock = std::chrono::steady_clock;
using Evidence = VadEvidenceStore::Evidence;

Evidence Snapshot(const VadEvidenceStore* t) { return t ? t->SnapshotVadEvidence() : Evidence{}; }

// Seconds of [start, end) covered by finalized VAD speech.
double SpeechOverlap(double start, double end, const std::vector<VadEvidenceStore::VadSeg>& segs) {
  double sum = 0.0;
  for (const auto& s : segs) {
    const double lo = std::max(start, s.start), hi = std::min(end, s.end);
    if (hi > lo) sum += hi - lo;
  }
  return sum;
}

// Whether live text of [start, end) may be shown: finalized speech overlaps
// it, or the detector is in speech with an active region reaching it.
bool LiveTextBacked(double start, double end, const Evidence& v) {
  if (v.segments && SpeechOverlap(start, end, *v.segments) > 0.0) return true;
  return v.in_speech && v.active_start < end && v.active_horizon + 1e-9 >= start;
}

std::string EscapeJson(const std::string& s) {
  std::string o;
  o.reserve(s.size() + 8);
  for (unsigned char c : s) {
    switch (c) {
      case '"': o += "\\\""; break;
      case '\\': o += "\\\\"; break;
      case '\n': o += "\\n"; break;
      case '\r': o += "\\r"; break;
      case '\t': o += "\\t"; break;
      case '\b': o += "\\b"; break;
      case '\f': o += "\\f"; break;
      default:
        if (c < 0x20) {
          char b[8];
          std::snprintf(b, sizeof(b), "\\u%04x", c);
          o += b;
        } else {
          o += static_cast<char>(c);
        }
    }
  }
  return o;
}

std::string TextEvent(const char* type, long id, double start, double end, const std::string& text) {
  char head[192];
  std::snprintf(head, sizeof(head),
                "{\"type\":\"%s\",\"source\":\"qwen3_asr\",\"text_id\":%ld,\"start\":%.9f,"
                "\"end\":%.9f,\"text\":\"",
                type, id, start, end);
  return std::string(head) + EscapeJson(text) + "\"}";
}

struct Region {
  long start, end;
  bool finalized;
};

}  // namespace

AsrWorker::AsrWorker(core::IStreamAsr* asr, const Params& params, Emit emit, core::TimeBase tb,
                     cudaStream_t stream, const VadEvidenceStore* timeline)
    : asr_(asr), p_(params), emit_(std::move(emit)), tb_(tb), timeline_(timeline),
      stream_(stream) {}

void AsrWorker::ProcessSpan(const float* samples, int n) {
  if (!samples || n <= 0) return;
  if (!p_.asr_vad_gate) {
    ProcessIncremental(samples, n, false);
    processed_.fetch_add(n);
    return;
  }
  pending_.insert(pending_.end(), samples, samples + n);
  received_ += n;
  processed_.store(received_);
  DrainVadGate(false);
}

void AsrWorker::Finalize() {
  finalizing_ = true;
  if (p_.asr_vad_gate) DrainVadGate(true);
  ProcessIncremental(nullptr, 0, true);
  finalizing_ = false;
}

// Moves the gate cursor pos_ as far as the VAD evidence decides: silence is
// skipped (keeping `lead` samples before the next onset), speech is fed in
// quanta, and a segment closes once `trail` samples of decided silence
// follow its last speech.
void AsrWorker::DrainVadGate(bool final) {
  const Evidence v = Snapshot(timeline_);
  std::vector<Region> regions;
  long limit = -1;  // samples up to here are decided
  if (v.segments) {
    for (const auto& s : *v.segments) {
      const long a = std::max(0L, tb_.SampleAt(s.start)), b = std::min(received_, tb_.SampleAt(s.end));
      if (b <= a) continue;
      regions.push_back({a, b, true});
      limit = std::max(limit, b);
    }
  }
  if (v.horizon > -1e8) limit = std::max(limit, std::min(received_, tb_.SampleAt(v.horizon)));
  if (v.in_speech && v.active_start > -1e8 && v.active_horizon + 1e-9 >= v.active_start) {
    const long a = std::max(0L, tb_.SampleAt(v.active_start));
    const long b = std::min(received_, tb_.SampleAt(v.active_horizon));
    if (b > a) {
      regions.push_back({a, b, false});
      limit = std::max(limit, b);
    }
  }
  if (final) limit = received_;
  if (limit < pos_) return;
  limit = std::min(limit, received_);
  std::stable_sort(regions.begin(), regions.end(), [](const Region& x, const Region& y) {
    return x.start != y.start ? x.start < y.start : x.end < y.end;
  });
  const long lead = std::max<long>(0, static_cast<long>(p_.asr_vad_lead_ms) * p_.sample_rate / 1000);
  const long trail = std::max<long>(0, static_cast<long>(std::llround(p_.asr_vad_trail_sec * p_.sample_rate)));

  while (pos_ < limit && PendingSamples() > 0) {
    const Region* next = nullptr;
    for (const Region& r : regions)
      if (r.end > pos_ && r.start < limit) {
        next = &r;
        break;
      }
    if (in_seg_ && last_speech_end_ >= 0) {
      const long endpoint = last_speech_end_ + trail;
      const long next_start = next ? next->start : std::numeric_limits<long>::max();
      if (next_start > endpoint) {
        if (limit < endpoint && !final) break;  // the trailing interval is not decided yet
        // close at the endpoint; the gap samples stay pending (a later
        // onset may need them as its lead)
        seg_end_ = std::min(endpoint, received_);
        ProcessIncremental(nullptr, 0, true);
        last_speech_end_ = -1;
        continue;
      }
    }
    if (!next) {
      const long skip_to = final ? limit : std::max(pos_, limit - lead);
      if (skip_to <= pos_) break;
      SkipPendingUntil(skip_to);
      continue;
    }
    if (pos_ < next->start) {
      if (in_seg_) {  // speech resumes inside the trailing interval: keep the pause
        FeedPendingUntil(std::min(next->start, limit), true);
        continue;
      }
      const long lead_start = std::max(0L, next->start - lead);
      if (pos_ < lead_start) {
        SkipPendingUntil(std::min(lead_start, limit));
        continue;
      }
    }
    const long before = pos_;
    FeedPendingUntil(std::min(next->end, limit), next->finalized || final);
    if (pos_ == before) break;
    last_speech_end_ = pos_;
  }
}

void AsrWorker::FeedPendingUntil(long end_sample, bool exact_end) {
  const long quantum =
      std::max<long>(1, static_cast<long>(p_.asr_vad_gate_chunk_ms) * p_.sample_rate / 1000);
  while (pos_ < end_sample && PendingSamples() > 0) {
    const long left = end_sample - pos_;
    if (!exact_end && left < quantum) return;  // wait for a full quantum
    const int take = static_cast<int>(std::min({left, quantum, PendingSamples()}));
    if (take <= 0) return;
    ProcessIncremental(PendingData(), take, false);
    ConsumePending(take);
  }
}

void AsrWorker::SkipPendingUntil(long end_sample) {
  const long take = std::min(end_sample - pos_, PendingSamples());
  if (take <= 0) return;
  pos_ += take;
  ConsumePending(take);
}

void AsrWorker::ConsumePending(long n) {
  if (n <= 0) return;
  pending_off_ += static_cast<size_t>(n);
  if (pending_off_ == pending_.size()) {
    pending_.clear();
    pending_off_ = 0;
  } else if (pending_off_ >= 65536 && pending_off_ * 2 >= pending_.size()) {
    pending_.erase(pending_.begin(), pending_.begin() + static_cast<long>(pending_off_));
    pending_off_ = 0;
  }
}

void AsrWorker::ProcessIncremental(const float* samples, int n, bool finalize) {
  const int piece = 8 * p_.sample_rate;  // worker-level caps are checked between pieces
  for (int off = 0; off < n; off += piece)
    EmitIncrementalChunk(samples ? samples + off : nullptr, std::min(piece, n - off), false);
  if (finalize) EmitIncrementalChunk(nullptr, 0, true);
}

std::string AsrWorker::FinalizeDecoderSegment() {
  std::string text = asr_->StreamFinalize(stream_);
  if (!p_.final_full_context_decode) return text;
  if (seg_audio_.empty()) return "";
  return asr_->TranscribeFinal(seg_audio_.data(), static_cast<int>(seg_audio_.size()), stream_);
}

void AsrWorker::CloseSegment() {
  live_ = FinalizeDecoderSegment();
  in_seg_ = false;
}

void AsrWorker::EmitIncrementalChunk(const float* samples, int n, bool finalize) {
  const auto t0 = Clock::now();
  bool closed = false;
  if (n > 0) {
    if (!in_seg_) {
      seg_start_ = pos_;
      seg_samples_ = 0;
      live_.clear();
      seg_audio_.clear();
      asr_->StreamReset(seg_start_);
      in_seg_ = true;
    }
    if (p_.final_full_context_decode) seg_audio_.insert(seg_audio_.end(), samples, samples + n);
    live_ = asr_->StreamChunk(samples, n, stream_);
    seg_samples_ += n;
    pos_ += n;
    seg_end_ = pos_;
  }
  if (in_seg_ && finalize) {
    CloseSegment();
    closed = true;
  }
  if (in_seg_ && p_.segment_sec > 0.0 &&
      seg_samples_ >= static_cast<long>(p_.segment_sec * p_.sample_rate)) {
    CloseSegment();
    closed = true;
  }
  // decoder-cache cap: the segment closes before its audio tokens outgrow
  // the KV budget
  if (in_seg_ && p_.max_audio_tokens > 0 && asr_->stream_audio_tokens() >= p_.max_audio_tokens) {
    CloseSegment();
    closed = true;
  }
  {
    const double dt = std::chrono::duration<double>(Clock::now() - t0).count();
    double cur = compute_sec_.load(std::memory_order_relaxed);
    while (!compute_sec_.compare_exchange_weak(cur, cur + dt, std::memory_order_relaxed)) {
    }
  }

  if (closed && (p_.final_full_context_decode || !live_.empty())) {
    const double s0 = tb_.SecondsAt(seg_start_), s1 = tb_.SecondsAt(seg_end_);
    bool keep = true;
    if (p_.asr_vad_gate && timeline_) {
      const Evidence v = Snapshot(timeline_);
      if (!v.segments || v.segments->empty()) {
        keep = !(finalizing_ || v.horizon >= s0 + p_.asr_vad_trail_sec);
      } else if (SpeechOverlap(s0, s1, *v.segments) < p_.asr_vad_min_overlap_sec) {
        keep = !(finalizing_ || s1 <= v.horizon);  // rejected once VAD has decided the span
      }
    }
    if (!keep || live_.empty()) {
      if (emit_ && !delivered_.empty())
        emit_("{\"type\":\"asr_retract\",\"source\":\"qwen3_asr\",\"text_id\":" +
              std::to_string(text_id_) + "}");
    } else {
      const long id = text_id_++;
      if (text_sink_) text_sink_(id, s0, s1, live_, true);
      if (emit_) emit_(TextEvent("asr", id, s0, s1, live_));
    }
    live_.clear();
    delivered_.clear();
    seg_audio_.clear();
  } else if (in_seg_) {
    const double s0 = tb_.SecondsAt(seg_start_), s1 = tb_.SecondsAt(seg_end_);
    const bool expose = !(p_.asr_vad_gate && timeline_) || LiveTextBacked(s0, s1, Snapshot(timeline_));
    if (expose && live_ != delivered_) {
      if (text_sink_) text_sink_(text_id_, s0, s1, live_, false);
      if (emit_ && !live_.empty()) emit_(TextEvent("asr_partial", text_id_, s0, s1, live_));
      delivered_ = live_;
    }
  }
}

void AsrWorker::Reset() {
  in_seg_ = false;
  pos_ = 0;
  seg_samples_ = 0;
  live_.clear();
  seg_audio_.clear();
  text_id_ = 0;
  delivered_.clear();
  finalizing_ = false;
  processed_.store(0);
  compute_sec_.store(0.0, std::memory_order_relaxed);
  asr_->Reset();
  pending_.clear();
  pending_off_ = 0;
  received_ = 0;
  last_speech_end_ = -1;
}

// ---- StreamBatcher -------------------------------------------------------------

class StreamBatcher::Proxy final : public core::IStreamAsr {
 public:
  Proxy(StreamBatcher* b, int i) : b_(b), i_(i) {}
  void Reset() override {
    if (b_->ops_.reset) b_->ops_.reset(i_);
  }
  void StreamReset(long base) override {
    if (b_->ops_.stream_reset) b_->ops_.stream_reset(i_, base);
  }
  std::string StreamChunk(const float* pcm, int n, cudaStream_t) override {
    return b_->Submit({i_, false, pcm, n});
  }
  std::string StreamFinalize(cudaStream_t) override { return b_->Submit({i_, true, nullptr, 0}); }
  std::string TranscribeFinal(const float* pcm, int n, cudaStream_t) override {
    return b_->ops_.transcribe_final ? b_->ops_.transcribe_final(i_, pcm, n) : std::string();
  }
  int stream_audio_tokens() const override {
    return b_->ops_.audio_tokens ? b_->ops_.audio_tokens(i_) : 0;
  }

 private:
  StreamBatcher* b_;
  int i_;
};

StreamBatcher::StreamBatcher(int streams, BatchFn batch, StreamOps ops,
                             std::chrono::microseconds max_wait)
    : batch_(std::move(batch)), ops_(std::move(ops)), max_wait_(max_wait) {
  for (int i = 0; i < streams; ++i) proxies_.push_back(std::make_unique<Proxy>(this, i));
  dispatcher_ = std::thread([this] { Dispatch(); });
}

StreamBatcher::~StreamBatcher() {
  {
    std::lock_guard<std::mutex> lock(mu_);
    stop_ = true;
  }
  cv_work_.notify_all();
  dispatcher_.join();
}

core::IStreamAsr* StreamBatcher::Stream(int i) { return proxies_.at(static_cast<size_t>(i)).get(); }

void StreamBatcher::Enter(int) {
  std::lock_guard<std::mutex> lock(mu_);
  ++active_;
}

void StreamBatcher::Leave(int) {
  {
    std::lock_guard<std::mutex> lock(mu_);
    --active_;
  }
  cv_work_.notify_all();  // the streams still inside may now be complete
}

std::vector<int> StreamBatcher::batch_sizes() const {
  std::lock_guard<std::mutex> lock(mu_);
  return sizes_;
}

std::string StreamBatcher::Submit(const Request& r) {
  std::string text;
  bool done = false;
  std::unique_lock<std::mutex> lock(mu_);
  queue_.push_back(r);
  results_.push_back(&text);
  done_flags_.push_back(&done);
  cv_work_.notify_all();
  cv_done_.wait(lock, [&] { return done; });
  return text;
}

// One batch at a time: wait for a first request, then until every stream in
// a call window has submitted or max_wait has passed, then run the batch with
// the lock released.
void StreamBatcher::Dispatch() {
  std::unique_lock<std::mutex> lock(mu_);
  while (true) {
    cv_work_.wait(lock, [&] { return stop_ || !queue_.empty(); });
    if (queue_.empty() && stop_) return;
    const auto deadline = Clock::now() + max_wait_;
    cv_work_.wait_until(lock, deadline, [&] {
      return stop_ || static_cast<int>(queue_.size()) >= std::max(active_, 1);
    });
    std::vector<Request> reqs;
    std::vector<std::string*> outs;
    std::vector<bool*> flags;
    reqs.swap(queue_);
    outs.swap(results_);
    flags.swap(done_flags_);
    sizes_.push_back(static_cast<int>(reqs.size()));
    lock.unlock();
    std::vector<std::string> texts(reqs.size());
    batch_(reqs, &texts);
    lock.lock();
    for (size_t i = 0; i < reqs.size(); ++i) {
      *outs[i] = std::move(texts[i]);
      *flags[i] = true;
    }
    cv_done_.notify_all();
  }
}

}  // namespace pipeline
}  // namespace orator
