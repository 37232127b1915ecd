// Session scheduler of the streaming ASR path: the reference's per-session
// AsrWorker (include/pipeline/asr_worker.h, src/pipeline/asr_worker.cc) with
// the same Params, public methods, VAD gate, segment / audio-token caps and
// JSON events, plus a StreamBatcher that lets many workers (one host thread
// per live stream, as in the reference) share one batched GPU decoder: the
// decoder calls that the workers make at about the same time are coalesced
// into one batched call (AsrSessionPool::StepAll underneath) instead of
// running one session at a time.
//
// Types the reference takes from other modules are restated here with the
// subset this layer uses: core::TimeBase (sample <-> second mapping),
// core::IStreamAsr (the streaming methods of core::IAsr) and
// pipeline::VadEvidenceStore (the typed VAD track of ComprehensiveTimeline).
#pragma once

#include <cuda_runtime_api.h>

#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace orator {
namespace core {

// Sample positions on the session clock <-> seconds
// (include/core/time_base.h).
class TimeBase {
 public:
  TimeBase() = default;
  explicit TimeBase(int sample_rate, long origin_sample = 0)
      : sample_rate_(sample_rate), origin_(origin_sample) {}
  bool valid() const { return sample_rate_ > 0; }
  int sample_rate() const { return sample_rate_; }
  double SecondsAt(long abs_sample) const {
    return sample_rate_ > 0 ? static_cast<double>(abs_sample - origin_) / sample_rate_ : 0.0;
  }
  long SampleAt(double seconds) const {
    return origin_ + static_cast<long>(std::llround(seconds * sample_rate_));
  }

 private:
  int sample_rate_ = 0;
  long origin_ = 0;
};

// The streaming half of the reference's core::IAsr (include/core/stages.h):
// a session-scoped recognizer that accepts PCM pieces and returns the text
// decoded so far.
class IStreamAsr {
 public:
  virtual ~IStreamAsr() = default;
  virtual void Reset() = 0;
  virtual void StreamReset(long base_sample) = 0;
  virtual std::string StreamChunk(const float* pcm, int n, cudaStream_t stream) = 0;
  virtual std::string StreamFinalize(cudaStream_t stream) = 0;
  virtual std::string TranscribeFinal(const float* pcm, int n, cudaStream_t stream) = 0;
  virtual int stream_audio_tokens() const = 0;
};

}  // namespace core

namespace pipeline {

// Typed VAD evidence (the VAD track of the reference's ComprehensiveTimeline,
// src/pipeline/comprehensive_timeline.cc:162-208, 428-434): finalized speech
// segments, the decision horizon, and the live in-speech state with its
// provisional active region. Thread-safe; snapshots are immutable.
class VadEvidenceStore {
 public:
  struct VadSeg {
    double start = 0.0;
    double end = 0.0;
  };
  struct Evidence {
    std::shared_ptr<const std::vector<VadSeg>> segments;
    double horizon = -1e9;
    bool in_speech = false;
    double observed_at = -1e9;
    double active_start = -1e9;
    double active_horizon = -1e9;
  };
  void DepositVad(const VadSeg& seg);
  void AdvanceVadHorizon(double horizon_sec);
  void UpdateVadState(bool in_speech, double observed_at_sec, double active_start_sec = -1e9,
                      double active_horizon_sec = -1e9);
  Evidence SnapshotVadEvidence() const;

 private:
  mutable std::mutex mu_;
  std::vector<VadSeg> segs_;
  Evidence ev_;
};

class AsrWorker {
 public:
  // Defaults of the reference (include/pipeline/asr_worker.h:20-40).
  struct Params {
    int sample_rate = 16000;
    double segment_sec = 24.0;      // hard cap on one decoder segment (0 = off)
    int max_audio_tokens = 1500;    // decoder-cache cap: finalize at this many audio tokens
    bool asr_vad_gate = true;       // feed only VAD-decided speech
    int asr_vad_lead_ms = 200;      // audio kept before a speech onset
    int asr_vad_gate_chunk_ms = 100;  // feed quantum for decided speech
    double asr_vad_trail_sec = 1.5;   // silence after speech before the segment closes
    double asr_vad_min_overlap_sec = 0.12;  // VAD speech a final needs to be kept
    bool final_full_context_decode = false;
  };
  using Emit = std::function<void(const std::string&)>;
  using TextSegmentSink = std::function<void(long id, double start, double end,
                                             const std::string& text, bool is_final)>;

  AsrWorker(core::IStreamAsr* asr, const Params& params, Emit emit, core::TimeBase tb,
            cudaStream_t stream = 0, const VadEvidenceStore* timeline = nullptr);

  void set_text_sink(TextSegmentSink sink) { text_sink_ = std::move(sink); }
  void ProcessSpan(const float* samples, int n);
  void Finalize();
  void Reset();
  long processed_samples() const { return processed_.load(); }
  double compute_sec() const { return compute_sec_.load(); }

 private:
  void DrainVadGate(bool final);
  void FeedPendingUntil(long end_sample, bool exact_end);
  void SkipPendingUntil(long end_sample);
  void ConsumePending(long n);
  long PendingSamples() const { return static_cast<long>(pending_.size() - pending_off_); }
  const float* PendingData() const { return pending_.data() + pending_off_; }
  void ProcessIncremental(const float* samples, int n, bool finalize);
  void EmitIncrementalChunk(const float* samples, int n, bool finalize);
  std::string FinalizeDecoderSegment();
  void CloseSegment();

  core::IStreamAsr* asr_;
  Params p_;
  Emit emit_;
  TextSegmentSink text_sink_;
  core::TimeBase tb_;
  const VadEvidenceStore* timeline_;
  cudaStream_t stream_;

  std::atomic<long> processed_{0};
  std::atomic<double> compute_sec_{0.0};

  bool in_seg_ = false;
  long pos_ = 0;          // next sample the decoder would receive (session clock)
  long seg_start_ = 0, seg_end_ = 0, seg_samples_ = 0;
  std::string live_, delivered_;
  std::vector<float> seg_audio_;
  long text_id_ = 0;
  bool finalizing_ = false;

  std::vector<float> pending_;  // samples [pos_, received_)
  size_t pending_off_ = 0;
  long received_ = 0;
  long last_speech_end_ = -1;
};

// Coalesces the decoder calls of many streams into batched calls. Each stream
// gets an IStreamAsr proxy (Stream(i)) for its AsrWorker; StreamChunk and
// StreamFinalize block the calling thread until the batch holding them has
// run. A batch runs when every stream that is currently inside a decoder call
// window has submitted (Enter / Leave bracket a worker's ProcessSpan or
// Finalize) or `max_wait` after its first request, whichever comes first.
class StreamBatcher {
 public:
  struct Request {
    int stream = 0;
    bool finalize = false;     // StreamFinalize instead of StreamChunk
    const float* pcm = nullptr;
    int n = 0;
  };
  // The batched decoder: fills texts[i] for requests[i] (one call per batch).
  using BatchFn = std::function<void(const std::vector<Request>& requests,
                                     std::vector<std::string>* texts)>;
  // Per-stream calls that are not batched (reset, full-context final decode,
  // audio-token count).
  struct StreamOps {
    std::function<void(int stream)> reset;
    std::function<void(int stream, long base_sample)> stream_reset;
    std::function<std::string(int stream, const float* pcm, int n)> transcribe_final;
    std::function<int(int stream)> audio_tokens;
  };

  StreamBatcher(int streams, BatchFn batch, StreamOps ops,
                std::chrono::microseconds max_wait = std::chrono::microseconds(2000));
  ~StreamBatcher();
  StreamBatcher(const StreamBatcher&) = delete;
  StreamBatcher& operator=(const StreamBatcher&) = delete;

  core::IStreamAsr* Stream(int i);
  void Enter(int stream);
  void Leave(int stream);
  // Sizes of the batches run so far, in order.
  std::vector<int> batch_sizes() const;

 private:
  class Proxy;
  std::string Submit(const Request& r);
  void Dispatch();

  BatchFn batch_;
  StreamOps ops_;
  std::chrono::microseconds max_wait_;
  std::vector<std::unique_ptr<Proxy>> proxies_;
  mutable std::mutex mu_;
  std::condition_variable cv_work_, cv_done_;
  std::vector<Request> queue_;
  std::vector<std::string*> results_;
  std::vector<bool*> done_flags_;
  int active_ = 0;
  bool stop_ = false;
  std::vector<int> sizes_;
  std::thread dispatcher_;
};

}  // namespace pipeline
}  // namespace orator
