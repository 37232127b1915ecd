// Decoder engine: weights (Model), one-session decoder (Decoder, the
// AsrTextDecoder drop-in) and the paged KV pool they share.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <map>
#include <set>
#include <vector>

#include <cuda_runtime.h>

#include "graph_cache.h"
#include "kernels.h"

namespace orx {

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};
void check(cudaError_t e, const char* what);
#define ORX_CHECK(x) ::orx::check((x), #x)

template <typename T>
T* dalloc(size_t n) {
  void* p = nullptr;
  ORX_CHECK(cudaMalloc(&p, n * sizeof(T) ? n * sizeof(T) : 16));
  return static_cast<T*>(p);
}

struct ModelConfig {
  int num_layers = 28;
  int vocab_size = 151936;
  int max_seq_len = 2048;
  float rms_norm_eps = 1e-6f;
  float rope_theta = 1000000.0f;
};

// Device-resident weights of the 28-layer decoder (layout chosen for the
// streaming GEMV and the GEMM epilogues; see set_tensor for the mapping from
// the reference's thinker.model.* tensors).
// Split-K workspace of one stream's projections. `reserve` grows it (after a
// stream synchronize) and bumps `gen`, so owners of captured graphs can tell
// that the old address is gone.
struct GemmWs {
  static constexpr int kTickets = 1 << 15;  // split-K fixup tickets (tiles per projection)
  float* ws = nullptr;
  int* cnt = nullptr;  // kTickets zeroed ints, allocated with the first workspace
  size_t cap = 0;
  uint64_t gen = 0;
  void reserve(size_t floats, cudaStream_t s);
  GemmWs() = default;
  GemmWs(const GemmWs&) = delete;
  GemmWs& operator=(const GemmWs&) = delete;
  ~GemmWs();
};
// Split count run_proj picks for an N x K projection over T token rows, and
// the workspace floats it then needs (0 without a split).
int proj_splits(int N, int K, int T, int num_sms);
size_t proj_ws_floats(int N, int K, int T, int num_sms);
// norm_w / norm_out: RMSNorm of the residual output rows to bf16 right after
// the projection (fused into the split-K reduction when there is one).
void run_proj(GemmWs& w, const uint16_t* X, const uint16_t* W, int N, int K, int T, int epi,
              float* out_f32, uint16_t* out_bf16, int ldo, int* err, int num_sms, cudaStream_t s,
              const float* norm_w = nullptr, uint16_t* norm_out = nullptr, float eps = 0.f);

class Model {
 public:
  struct Layer {
    float *in_ln = nullptr, *post_ln = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    uint16_t *qkv = nullptr, *o = nullptr, *gateup = nullptr, *down = nullptr;
  };
  explicit Model(const ModelConfig& c);
  ~Model();
  Model(const Model&) = delete;
  Model& operator=(const Model&) = delete;

  // Place one reference-named tensor. dtype: 0 = fp32, 1 = bf16 bits.
  // `device` selects whether `src` is a device pointer.
  void set_tensor(const std::string& name, const void* src, int dtype, size_t numel, bool device);
  void init_synthetic(int seed, cudaStream_t s);
  bool complete() const;

  ModelConfig cfg;
  int num_sms = 148;
  uint16_t* embed = nullptr;  // [V, 2048], also the tied lm_head
  float* final_norm = nullptr;
  std::vector<Layer> layers;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  std::vector<uint8_t> have;  // per-tensor loaded flags
  int rope_positions = 0;
};

// Paged KV pool: [layer][page][K|V][kv head][16][128] bf16.
struct KvPool {
  KvPool(int layers, int pages);
  ~KvPool();
  uint16_t* layer(int l) const { return base + (size_t)l * pages * kPageElems; }
  int num_layers, pages;
  uint16_t* base = nullptr;
};

// One decode session with the reference AsrTextDecoder semantics
// (include/model/asr_text_decoder.h:45-113).
class Decoder {
 public:
  Decoder(Model* model, bool own_model);
  ~Decoder();

  void reset_cache() { cache_len_ = 0; }
  void truncate_cache(int len);
  int cache_len() const { return cache_len_; }
  void embed(int token, float* out) const;

  void prefill_at(const float* host_embeds, int T, int pos0, cudaStream_t s);
  void prefill_at_device(const float* dev_embeds, int T, int pos0, cudaStream_t s);
  void decode_step(const float* host_embed, int pos, cudaStream_t s);
  void decode_step_device(const int* d_token, int pos, cudaStream_t s);
  int argmax(int ban0, int ban1, cudaStream_t s);
  void argmax_to_device(int* d_out, int ban0, int ban1, cudaStream_t s);
  int read_token_id(const int* d_token, cudaStream_t s) const;
  std::vector<int> decode_greedy(int start_pos, int max_new, int eos0, int eos1, int ban_steps,
                                 int batch, cudaStream_t s);
  void copy_logits(float* host_out, cudaStream_t s) const;
  const float* logits_device() const { return logits_; }
  int device_error() const;

  // Records one decode body (embed -> layers -> lm_head + argmax) on `s`.
  void record_body(cudaStream_t s, const int* tok_ptr, bool record, bool finalize,
                   int only = -1);
  void profile_kernels(int iters, float* ms, cudaStream_t s);
  int trace_decode(int steps, unsigned long long* host_out, cudaStream_t s);
  int trace_ctas(int steps, unsigned long long* host_out, size_t out_len, cudaStream_t s);
  void launch_mk(const int* tok_ptr, int steps, int pos0, int count0, bool record, bool finalize,
                 int ban_steps, int ban0, int ban1, cudaStream_t s);
  bool use_mk_ = false;
  MkLayerW* mk_layers_ = nullptr;
  float* mk_part_ = nullptr;
  unsigned long long* mk_sync_ = nullptr;  // [best0, best1, barrier counter]
  unsigned long long* mk_trace_ = nullptr;
  unsigned long long* mk_trace_cta_ = nullptr;
  unsigned long long* trace_ = nullptr;

  Model* model;
  int graph_steps = 8;

 private:
  void ensure_prefill(int T);
  void forward_prefill(int T, int pos0, cudaStream_t s);
  void ensure_graphs(cudaStream_t s);

  bool own_model_;
  KvPool* kv_ = nullptr;
  int max_pages_ = 0;
  int* page_table_ = nullptr;
  int cache_len_ = 0;
  // decode buffers (fixed addresses, baked into graphs)
  float* dx_ = nullptr;
  float* dqkv_ = nullptr;
  uint16_t* dattn_ = nullptr;
  uint16_t* dact_ = nullptr;
  float* logits_ = nullptr;
  float* part_ = nullptr;
  int* counters_ = nullptr;
  StepState* st_ = nullptr;
  int* d_out_ = nullptr;
  int out_cap_ = 0;
  int* h_out_ = nullptr;  // pinned
  int* d_tmp_tok_ = nullptr;
  int* h_tok_ = nullptr;  // pinned
  // prefill buffers (grown on demand)
  int tcap_ = 0;
  float *px_ = nullptr, *pqkv_ = nullptr;
  uint16_t *pxn_ = nullptr, *pattn_ = nullptr, *pact_ = nullptr;
  int* pcounters_ = nullptr;
  float* ppart_ = nullptr;
  PrefillTile* d_tiles_ = nullptr;
  PrefillTile* h_tiles_ = nullptr;
  int tiles_cap_ = 0;
  float* h_stage_ = nullptr;
  size_t h_stage_cap_ = 0;
  cudaGraphExec_t g1_ = nullptr, gk_ = nullptr;
  GemmWs gws_;
  std::vector<uint16_t> embed_host_;
  bool embed_host_ready_ = false;
};

// Continuous-batching decoder over a shared paged KV pool (batch.cu).
class BatchDecoder {
 public:
  BatchDecoder(Model* model, int max_sessions, int max_batch, int pool_pages,
               int max_pages_per_session);
  ~BatchDecoder();
  int create_session();   // -1 when every slot is live
  void free_session(int sid);
  int cache_len(int sid) const;
  void truncate(int sid, int len);
  // Appends lens[i] rows of host embeddings (concatenated, [sum lens, 2048])
  // to each session and leaves its next greedy token on the device.
  void prefill(const int* sids, const int* lens, int n, const float* host_embeds, cudaStream_t s);
  // One greedy token for each listed session (ragged lengths), batched.
  void step(const int* sids, int n, int* host_tokens_out, cudaStream_t s);
  // The session's next `steps` argmaxes (prefill or step) exclude ban0/ban1.
  void set_ban(int sid, int ban0, int ban1, int steps, cudaStream_t s);
  // Each session's pending greedy token (the one its next step will feed).
  void next_tokens(const int* sids, int n, int* out, cudaStream_t s) const;
  int free_pages() const { return static_cast<int>(free_pages_.size()); }
  int device_error() const;
  Model* model;

 private:
  struct Session {
    bool live = false;
    int len = 0;
    std::vector<int> pages;
  };
  // Per-row activations of one pass over the layers. `rows` holds
  // [row_table (cap) | row_pos (cap) | last rows / session ids (2 * cap)].
  struct RowBufs {
    int cap = 0;
    float *x = nullptr, *qkv = nullptr, *part = nullptr, *logits = nullptr;
    uint16_t *xn = nullptr, *attn = nullptr, *act = nullptr;
    int *counters = nullptr, *rows = nullptr, *tokens = nullptr, *out = nullptr;
    int logits_cap = 0;
    void release();
  };
  void check_sid(int sid) const;
  bool reserve(int sid, int new_len);
  bool fits(const int* sids, const int* lens, int n) const;
  void upload_table(cudaStream_t s);
  void alloc_rows(RowBufs& b, int rows);
  void ensure_logits(RowBufs& b, int rows);
  void layers(RowBufs& b, GemmWs& ws, int rows, int max_len, bool fused, cudaStream_t s);
  void record_step(int n, cudaStream_t s);
  // Device memory a captured step graph may reference changes only with this.
  uint64_t step_epoch() const { return step_ws_.gen + step_realloc_; }

  int max_sessions_, max_batch_, mps_;
  KvPool* kv_ = nullptr;
  std::vector<int> free_pages_;
  std::vector<Session> sessions_;
  std::vector<int> h_table_;
  bool dirty_ = true;
  int* d_table_ = nullptr;
  int* d_next_tok_ = nullptr;
  int4* d_ban_ = nullptr;  // per session {ban0, ban1, argmaxes left to ban}
  unsigned long long* d_amax_keys_ = nullptr;  // split argmax: per-row packed best
  int* d_amax_cnt_ = nullptr;                  // split argmax: per-row CTA tickets
  StepState* st_ = nullptr;
  int* h_rows_ = nullptr;  // pinned staging
  // Decode steps use fixed buffers sized for max_batch at construction and a
  // workspace reserved for every batch size up front, so captured step graphs
  // never see a reallocation; prefill (any row count) has its own.
  RowBufs stepb_, preb_;
  GemmWs step_ws_, pre_ws_;
  uint64_t step_realloc_ = 0;
  PrefillTile* d_tiles_ = nullptr;
  PrefillTile* h_tiles_ = nullptr;
  int tiles_cap_ = 0, ntiles_ = 0;
  int* h_step_[2] = {nullptr, nullptr};
  int* h_tbl_[2] = {nullptr, nullptr};
  int* h_out_ = nullptr;
  cudaEvent_t ev_rows_[2] = {nullptr, nullptr};
  cudaEvent_t ev_table_[2] = {nullptr, nullptr};
  long long step_count_ = 0, table_count_ = 0;
  GraphCache<cudaGraphExec_t, cudaError_t (*)(cudaGraphExec_t)> graphs_{cudaGraphExecDestroy};
};

// Batched Silero-shaped speech detector (vad.cu): `streams` independent
// streams advance one 512-sample window per step; LSTM state and the 64-sample
// context are carried per stream across calls.
class BatchVad {
 public:
  explicit BatchVad(int streams);
  ~BatchVad();
  BatchVad(const BatchVad&) = delete;
  BatchVad& operator=(const BatchVad&) = delete;
  int streams() const;
  void set_tensor(const std::string& name, const float* data, size_t n);  // host fp32
  void init_synthetic(int seed);
  void reset();
  // pcm [streams][steps * 512] -> probs [streams][steps] (device / host).
  void run_device(const float* d_pcm, int steps, float* d_probs, cudaStream_t s);
  void run_host(const float* pcm, int steps, float* probs, cudaStream_t s);

 private:
  void upload();
  struct Impl;
  Impl* p_;
};

// Qwen3-ASR audio tower (tower.cu), batched over utterances: mel
// [128, frames] of each utterance -> [OutputLength(frames), 2048] rows.
class AudioTower {
 public:
  AudioTower(int layers, bool windowed);
  ~AudioTower();
  AudioTower(const AudioTower&) = delete;
  AudioTower& operator=(const AudioTower&) = delete;
  int layers() const;
  // By checkpoint name (thinker.audio_tower.*); dtype 0 fp32, 1 bf16 bits (host).
  void set_tensor(const std::string& name, const void* data, int dtype, size_t numel);
  void init_synthetic(int seed);
  bool complete() const;
  // d_mel: the utterances' [128, frames[u]] blocks back to back (device);
  // d_out: [sum of OutputLength(frames[u]), 2048] (device). Returns the rows.
  int forward_device(const float* d_mel, const int* frames, int n_utt, float* d_out,
                     cudaStream_t s);
  // One utterance from / to host memory (AsrAudioTower::Forward).
  int forward_host(const float* mel, int n_frames, float* out, cudaStream_t s);
  int device_error() const;
  static int output_length(int frames);

 private:
  struct Impl;
  Impl* p_;
};

// Streaming Sortformer diarizer network (sortformer.cu): pre-encode,
// FastConformer stack and transformer decoder with the speaker head.
class Sortformer {
 public:
  Sortformer(int conf_layers, int dec_layers);
  ~Sortformer();
  Sortformer(const Sortformer&) = delete;
  Sortformer& operator=(const Sortformer&) = delete;
  // fp32 tensor by checkpoint name, from host or device memory.
  void set_tensor(const std::string& name, const float* data, size_t numel, bool device);
  void load_safetensors(const std::string& path);
  void init_synthetic(int seed);
  bool complete() const;
  // mel [128, n_frames] freq-major (device) -> d_out [T2, 512]; returns T2.
  int pre_encode_device(const float* d_mel, int n_frames, int valid, float* d_out, int* valid_out,
                        cudaStream_t s);
  // emb [T, 512] -> preds [T, 4] (ForwardEncoderDecoder).
  void encode_decode_device(const float* d_emb, int T, int valid, float* d_preds, cudaStream_t s);
  // One streaming chunk: [cache rows | pre_encode(mel)] -> preds [T, 4]; returns T.
  int step_device(const float* d_mel, int n_frames, int valid, const float* d_cache, int n_cache,
                  float* d_preds, int* valid_out, cudaStream_t s);
  int device_error() const;

 private:
  struct Impl;
  Impl* p_;
};

// fp32 single decoder layer (layer32.cu): fp32 weights, activations and KV.
struct Layer32;
Layer32* layer32_create(int max_seq_len, float eps, float theta);
void layer32_destroy(Layer32* l);
void layer32_set_tensor(Layer32* l, const char* name, const float* src, size_t n, bool device_src);
void layer32_init_synthetic(Layer32* l, int seed, int layer);
void layer32_forward(Layer32* l, const float* d_in, int T, int pos0, float* d_out, cudaStream_t s);
int layer32_len(const Layer32* l);
void layer32_truncate(Layer32* l, int n);

}  // namespace orx
