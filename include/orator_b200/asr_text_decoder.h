// C++ host classes of the B200 decoder, source-compatible with the
// reference's include/model/asr_text_decoder.h:30-113 (namespace
// orator::model, class AsrTextDecoder, same method names, signatures and
// argument meaning). They are thin owners over the C ABI in orx.h; errors
// become exceptions as in the reference: invalid arguments or state ->
// std::runtime_error, CUDA failures -> orator::model::GpuError (the
// reference's GpuMemoryException, src/gpu/memory.cc:14-20).
//
// Additions the reference does not have: LoadWeights from a checkpoint
// directory (instead of an io::ShardedSafeTensors object), InitSynthetic,
// and the multi-session AsrSessionPool (continuous batching over a paged KV
// pool: CreateSession / PrefillAt / StepAll / TruncateCache / FreeSession).
#pragma once

#include <cuda_runtime_api.h>

#include <stdexcept>
#include <string>
#include <vector>

#include "orx.h"

namespace orator {
namespace model {

#ifndef ORATOR_B200_GPU_ERROR_DEFINED
#define ORATOR_B200_GPU_ERROR_DEFINED
class GpuError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};
#endif

// AsrTextConfig (asr_text_decoder.h:30-43).
struct AsrTextConfig {
  int hidden_size = 2048;
  int num_layers = 28;
  int num_q_heads = 16;
  int num_kv_heads = 8;
  int head_dim = 128;
  int intermediate_size = 6144;
  int vocab_size = 151936;
  float rms_norm_eps = 1e-6f;
  float rope_theta = 1000000.0f;
  int max_seq_len = 2048;
  bool profile = false;
  bool cuda_graph_enabled = true;
};

class AsrTextDecoder {
 public:
  explicit AsrTextDecoder(const AsrTextConfig& config = {});
  ~AsrTextDecoder();
  AsrTextDecoder(const AsrTextDecoder&) = delete;
  AsrTextDecoder& operator=(const AsrTextDecoder&) = delete;

  // Weights: a checkpoint directory (model.safetensors[.index.json]) with
  // thinker.model.* tensors, one tensor at a time, or seeded synthetic ones.
  void LoadWeights(const std::string& model_dir);
  void SetTensor(const std::string& name, const void* data, bool bf16, size_t numel,
                 bool on_device = false);
  void InitSynthetic(int seed);

  void ResetCache();
  void Embed(int token_id, float* out) const;
  int hidden_size() const { return config_.hidden_size; }
  int vocab_size() const { return config_.vocab_size; }

  void Prefill(const float* embeds, int T, cudaStream_t stream = 0);
  void PrefillAt(const float* embeds, int T, int pos0, cudaStream_t stream = 0);
  void TruncateCache(int len);
  int cache_len() const;

  void DecodeStep(const float* embed, int pos, cudaStream_t stream = 0);
  void DecodeStepDevice(const int* d_token, int pos, cudaStream_t stream = 0);
  int Argmax(int ban0 = -1, int ban1 = -1, cudaStream_t stream = 0);
  void ArgmaxToDevice(int* d_out, int ban0, int ban1, cudaStream_t stream = 0);
  int ReadTokenId(const int* d_token, cudaStream_t stream = 0) const;
  std::vector<int> DecodeGreedy(int start_pos, int max_new, int eos0, int eos1,
                                int ban_steps = 3, int batch = 32, cudaStream_t stream = 0);
  std::vector<float> CopyLogits() const;

  orx_decoder* handle() const { return h_; }

 private:
  AsrTextConfig config_;
  orx_decoder* h_ = nullptr;
};

// Many independent sessions over one paged KV pool and the weights of an
// AsrTextDecoder (which must outlive the pool); one greedy token for every
// listed session per StepAll, batched on the GPU.
class AsrSessionPool {
 public:
  AsrSessionPool(const AsrTextDecoder& weights, int max_sessions, int max_batch, int pool_pages,
                 int max_pages_per_session);
  ~AsrSessionPool();
  AsrSessionPool(const AsrSessionPool&) = delete;
  AsrSessionPool& operator=(const AsrSessionPool&) = delete;

  int CreateSession();
  void FreeSession(int session);
  // Appends T rows [T, hidden] (host) to the session; leaves its next greedy
  // token pending. Several sessions at once: PrefillAt(sessions, lens, rows).
  void PrefillAt(int session, const float* embeds, int T, cudaStream_t stream = 0);
  void PrefillAt(const std::vector<int>& sessions, const std::vector<int>& lens,
                 const float* embeds, cudaStream_t stream = 0);
  std::vector<int> StepAll(const std::vector<int>& sessions, cudaStream_t stream = 0);
  std::vector<int> PendingTokens(const std::vector<int>& sessions, cudaStream_t stream = 0);
  void SetBan(int session, int ban0, int ban1, int steps, cudaStream_t stream = 0);
  void TruncateCache(int session, int len);
  int cache_len(int session) const;
  int free_pages() const;

 private:
  orx_batch* h_ = nullptr;
};

}  // namespace model
}  // namespace orator
