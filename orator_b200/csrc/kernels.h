// Kernel launchers shared between the decoder engine and the C ABI.
#pragma once

#include <cstdint>
#include <utility>
#include <cuda_runtime.h>
#include <atomic>
#include <mutex>

namespace orx {

// Per-decode-step device state (one per decode stream). Replaces the
// reference's device scalars d_tok_/step_pos_/d_count_/d_out_
// (src/model/asr_text_decoder.cu:677-691).
struct StepState {
  int pos;        // absolute position of the token being decoded
  int count;      // tokens recorded into `out` so far
  int tok;        // current token id (argmax result of the previous step)
  int ban_steps;  // argmaxes producing token k < ban_steps exclude ban0/ban1
  int ban0, ban1;
  int out_cap;
  int done;       // CTA ticket for the last-CTA finalize of the argmax
  unsigned long long best;  // packed (value, index) running argmax
  int* out;       // recorded token ids [out_cap]
  int err;        // device error word (bounded waits etc.)
  int pad;
};

enum ActMode : int { kActNorm = 0, kActEmbedNorm = 1, kActBf16 = 2 };
enum EpiMode : int { kEpiStore = 0, kEpiResid = 1, kEpiSwiglu = 2, kEpiLogits = 3,
                     kEpiLinear = 4 };

struct GemvArgs {
  const uint16_t* W;  // [rows, K] bf16 row-major
  int K;              // multiple of 2048
  int units;          // output units (rows, or gate/up pairs for SwiGLU)
  int act_mode;
  const float* x;         // fp32 input row for kActNorm
  const float* norm_w;    // fp32 RMSNorm weight [2048]
  float eps;
  const uint16_t* act;    // bf16 activation [K] for kActBf16
  const uint16_t* embed;  // embedding table for kActEmbedNorm
  const int* tok_ptr;     // token id for kActEmbedNorm
  float* x_init;          // kActEmbedNorm: residual row initialised by CTA 0
  int record;             // kActEmbedNorm: append *tok_ptr to st->out
  int epi;
  float* out_f32;         // kEpiStore / kEpiLogits target, kEpiResid accumulator
  uint16_t* out_bf16;     // kEpiSwiglu target
  int finalize;           // kEpiLogits: write st->tok and advance st->pos
  StepState* st;
  unsigned long long* trace;  // optional debug timeline slot (3 words)
};

// Weight-streaming GEMV for one activation row (decode at batch 1).
void launch_gemv(const GemvArgs& a, int num_sms, cudaStream_t s);

// Paged decode / prefill attention (flash-decoding split over pages).
struct AttnArgs {
  const float* qkv;        // [rows, 4096] fp32 raw projections (decode) or
                           // normalised+roped q in cols [0,2048) (prefill)
  int qkv_stride;          // elements between rows
  const float* q_norm_w;   // [128]
  const float* k_norm_w;   // [128]
  const float* rope_cos;   // [max_pos, 64]
  const float* rope_sin;
  uint16_t* kv_layer;      // this layer's page pool base
  int kv_row0;             // first 128-wide row of this layer in the pool's tensor map
  long long layer_stride;  // elements between layers (for reference only)
  const int* page_table;   // [n_tables, max_pages]
  int max_pages;
  const int* row_table;    // [rows] page-table row of each query row (nullptr: 0)
  const int* row_pos;      // [rows] absolute position of each query row
  const int* pos_scalar;   // if non-null, position of row 0 (decode B=1)
  int pos_base;            // row_pos == nullptr: row r sits at pos_base + r
  int rows;
  int fused_kv;            // 1: q/k norm, RoPE and the K/V store happen here
  int nsplit_max;           // grid splits; >= ceil(pages / pages_per_split)
  int pages_per_split;
  float* part;             // split partials scratch
  int* counters;           // [rows * 8] split tickets (self-resetting)
  uint16_t* out;           // [rows, 2048] bf16
  int* err;
  unsigned long long* trace;  // optional debug timeline slot (3 words)
};
// kv_pool: pool base ([layers * pages * 2 * 8 * 16, 128] bf16 rows).
void launch_attention(const AttnArgs& a, const uint16_t* kv_pool, long long pool_rows,
                      cudaStream_t s);
// 2-D bf16 TMA map over a row-major [rows, cols] matrix, box box_cols x box_rows,
// 128-byte swizzle.
bool make_tmap_2d(void* map, const void* base, long long rows, int cols, int box_cols,
                  int box_rows);

// Causal prefill attention (attn_prefill.cu): tiles of up to prefill_tile_rows()
// consecutive query positions of one session.
struct PrefillTile {
  int tab;    // page-table row of the session
  int pos0;   // position of the tile's first row
  int nrows;  // rows in the tile
  int row0;   // first row in qkv / out
};
struct PrefillAttnArgs {
  const float* qkv;  // normalised + roped q in cols [0, 2048)
  int qkv_stride;
  const PrefillTile* tiles;
  const int* page_table;
  int max_pages;
  int kv_row0;       // first 128-wide row of this layer in the pool's tensor map
  uint16_t* out;     // [rows, 2048] bf16
  int* err;
};
void launch_attn_prefill(const PrefillAttnArgs& a, int ntiles, const uint16_t* kv_pool,
                         long long pool_rows, cudaStream_t s);
int prefill_tile_rows();

// q/k RMSNorm + RoPE + K/V store for T prefill rows (q normalised in place).
void launch_qk_norm_rope_store(float* qkv, int rows, const float* qn, const float* kn,
                               const float* cos, const float* sin, uint16_t* kv_layer,
                               const int* page_table, int max_pages, const int* row_table,
                               const int* row_pos, int pos_base, cudaStream_t s);

// Row-wise RMSNorm to bf16: out[r] = bf16(x[r] * rsqrt(mean(x^2)+eps) * w).
void launch_rmsnorm_bf16(const float* x, const float* w, uint16_t* out, int rows, float eps,
                         cudaStream_t s);

// tcgen05 GEMM (gemm_tc.cu): out[t, n] (op)= sum_k X[t, k] W[n, k].
struct TcArgs {
  // weight rows, depth, tokens. N is a multiple of 128 and K of 64 * splits
  // except under kEpiLinear (splits 1, any N, K a multiple of 8: the tensor
  // maps zero-fill the ragged tiles and the epilogue masks rows >= N).
  int N, K, T;
  int epi;             // kEpiStore / kEpiResid / kEpiSwiglu / kEpiLinear
  float* out_f32;      // [T, ldo]
  uint16_t* out_bf16;  // SwiGLU output [T, ldo]
  int ldo;
  int* err;
  float* ws;           // split-K partials [splits, T, N]
  // Optional RMSNorm of the (residual) output rows to bf16 (N == 2048):
  // fused into the split-K reduction, else a separate row kernel.
  const float* norm_w;
  uint16_t* norm_out;
  float eps;
  // kEpiLinear: y = act(acc + bias[n]); act 0 none, 1 GELU (erf), 2 ReLU,
  // 3 SiLU, 4 sigmoid. The row goes to out_bf16 (rounded) when it is set --
  // with `split3`, as [bf16(y) | bf16(y) | bf16(y - bf16(y))] at columns
  // n, N + n, 2N + n (ldo = 3N) -- else it is stored into out_f32, or added
  // to it when `resid` is 1 (half of it when 2).
  const float* bias;
  int act;
  int resid;
  int split3;
  int bn_hint;  // token-tile width to use (0: chosen by launch_gemm_tc)
};
// kEpiLinear with split K: token-tile width (*bn) and split count for an
// N x K Linear over T rows on `sms` CTAs; split counts divide K / 64. The
// partials need splits * T * N floats of workspace in TcArgs::ws.
int linear_plan(int N, int K, int T, int sms, int* bn);
// X: [T, K] bf16 row-major (device), W: [N, K] bf16. splits divides K / 64.
void launch_gemm_tc(const uint16_t* X, const uint16_t* W, const TcArgs& g, int splits,
                    cudaStream_t s);
bool tc_available();
// Token-tile width launch_gemm_tc uses for a projection (sms 0: powers of two only).
int tc_token_tile(int N, int T, int splits, int sms);
int tc_sms();

// Argmax over fp32 logits with up to two banned ids into st (finalize sets st->tok).
void launch_argmax(const float* logits, int n, int ban0, int ban1, StepState* st, int* out_dev,
                   cudaStream_t s);

// Free operators of the reference API (ops.cu).
void op_rms_norm(const float* x, const float* w, float* out, int rows, int dim, float eps,
                 cudaStream_t s);
void op_rope(float* x, const int* pos, int n_tokens, int n_heads, int head_dim, float theta,
             bool rotate_half, cudaStream_t s);
void op_swiglu(const float* g, const float* u, float* o, long long n, cudaStream_t s);
void op_argmax_banned(const float* x, int n, int ban0, int ban1, int* out, cudaStream_t s);
cudaError_t op_gqa_attention(const float* q, const float* k, const float* v, float* out, int T,
                             int Hq, int Hkv, int D, float scale, bool causal, cudaStream_t s);
// Linear without tensor maps (K not a multiple of 8): one warp per output.
void op_linear_simt(const uint16_t* X, const uint16_t* W, const float* bias, float* out, int M,
                    int K, int N, int act, cudaStream_t s);

void launch_rope_table(float* cos, float* sin, int max_pos, float theta, cudaStream_t s);
void launch_synth_bf16(uint16_t* dst, long long n, int seed, int tid, double std, float mean,
                       cudaStream_t s);
void launch_synth_f32(float* dst, long long n, int seed, int tid, double std, float mean,
                      int round_bf16, cudaStream_t s);
void launch_f32_to_bf16(const float* in, uint16_t* out, long long n, cudaStream_t s);
void launch_bf16_to_f32(const uint16_t* in, float* out, long long n, cudaStream_t s);
void launch_embed_rows(const uint16_t* table, const int* ids, float* out, int rows,
                       cudaStream_t s);

// Persistent cooperative decode kernel (decode_mk.cu).
constexpr int kMkMaxSplit = 32;  // attention splits per kv head: 32 x 8 pages = 4096 positions
constexpr int kMkPart = 2 * 132;
constexpr int kMkMaxLayers = 48;  // layers the persistent kernel keeps pointers for
constexpr int kMkOwnRows = 16;   // rows of x per CTA: needs a grid of at least 128 CTAs
struct MkLayerW {
  const uint16_t *qkv, *o, *gu, *down;
  const float *in_ln, *post_ln, *qn, *kn;
};
struct MkArgs {
  const MkLayerW* layers;
  int L;
  const uint16_t* embed;
  const float* final_norm;
  int vocab;
  const float* rope_cos;
  const float* rope_sin;
  uint16_t* kv;                // pool base; layer l at kv + l * kv_layer_stride
  long long kv_layer_stride;   // elements
  const int* page_table;       // identity or session table [max_pages]
  int max_pages;
  StepState* st;
  const int* tok_ptr;          // token of step 0
  int steps, record, finalize;
  int pos0, count0, ban_steps, ban0, ban1;
  float* x;                    // [2048] residual
  float* qkv;                  // [4096]
  float* part;                 // [8 * kMaxSplit * kPart]
  uint16_t* act_g;             // [6144]
  float* logits;               // [vocab]
  unsigned long long* best2;   // [2] packed argmax, double-buffered per token
  unsigned int* bar;           // arrival counter, zero at launch
  float eps;
  unsigned long long* trace;   // optional: CTA 0 barrier arrive/depart times
  unsigned long long* trace_cta;  // optional: per barrier k and CTA, {inputs ready, arrive}
};
cudaError_t launch_decode_mk(const MkArgs& a, int grid, cudaStream_t s);
int decode_mk_max_grid();
size_t decode_mk_smem();
void launch_decode_mk_config();

// Runs `f` once per CUDA device (kernel attributes belong to a device's
// context); thread-safe.
template <typename F>
inline void once_per_device(std::atomic<unsigned long long>& done, F&& f) {
  int dev = 0;
  cudaGetDevice(&dev);
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (done.load(std::memory_order_relaxed) & bit) return;
  f();
  done.fetch_or(bit, std::memory_order_release);
}

// Programmatic dependent launch is on unless ORX_NO_PDL=1 is set.
bool pdl_enabled();

// Launch helper: every kernel may start early under programmatic dependent
// launch and must call griddepcontrol.wait before reading predecessor data.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

}  // namespace orx
