// fp32 single-layer decoder (the correctness-first configuration): one
// Qwen3-1.7B-shaped layer with fp32 weights, fp32 activations and an fp32 KV
// cache, no bf16 rounding anywhere. Same math as the bf16 path with every
// quantization point removed:
//   x -> RMSNorm -> qkv -> q/k RMSNorm (per head) -> RoPE (rotate-half)
//     -> KV append -> GQA attention (fp32 softmax, expf) -> o + residual
//     -> RMSNorm -> gate/up -> SwiGLU (expf) -> down + residual
// following the per-layer body of src/model/asr_text_decoder.cu:360-431 and
// the reference ops it calls (asr_ops.cu RmsNorm :21-51, RopeHalf :92-111,
// SwiGLU :80-87). The reference has no fp32 GPU decoder; its fp32 check runs
// this layer through its CPU oracle.
//
// One row at a time (a prompt of T rows is T successive rows, causally), five
// launches per row: norm+qkv GEMV, q/k norm + RoPE + KV store, attention,
// o GEMV (+residual), norm+gate/up GEMV (+SwiGLU), down GEMV (+residual).
// The GEMVs stream fp32 weights with 16-byte non-allocating loads, eight in
// flight per lane; at 201 MB of weights per row they are HBM-bound.
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>

#include "common.cuh"
#include "engine.h"
#include "kernels.h"

namespace orx {
namespace {

constexpr int kThreads = 256;
constexpr int kLayerBase = 16, kLayerStride = 16;  // synthetic tensor ids, as in the bf16 model
constexpr int kWarps = kThreads / 32;

enum L32Epi : int { kL32Store = 0, kL32Resid = 1, kL32Swiglu = 2 };

__device__ __forceinline__ float4 ld_stream(const float4* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < kWarps; ++w) t += red[w];
  return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < kWarps; ++w) t = fmaxf(t, red[w]);
  return t;
}

// Dot product of fp32 weight row w[K] with xs[K] (shared), one warp.
__device__ __forceinline__ float row_dot(const float* w, const float* xs, int K) {
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  const int lane = threadIdx.x & 31;
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
  const int n4 = K / 4;
  int i = lane;
  for (; i + 32 * 7 < n4; i += 32 * 8) {
    float4 wv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) wv[j] = ld_stream(w4 + i + 32 * j);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 xv = x4[i + 32 * j];
      a0 = fmaf(wv[j].x, xv.x, a0);
      a1 = fmaf(wv[j].y, xv.y, a1);
      a2 = fmaf(wv[j].z, xv.z, a2);
      a3 = fmaf(wv[j].w, xv.w, a3);
    }
  }
  for (; i < n4; i += 32) {
    const float4 wv = ld_stream(w4 + i), xv = x4[i];
    a0 = fmaf(wv.x, xv.x, a0);
    a1 = fmaf(wv.y, xv.y, a1);
    a2 = fmaf(wv.z, xv.z, a2);
    a3 = fmaf(wv.w, xv.w, a3);
  }
  return warp_sum((a0 + a1) + (a2 + a3));
}

// out[r] (op)= W[r, :] . act, act = RMSNorm(x) when norm_w is given, else x.
// kL32Swiglu: rows r < N/2 pair gate row r with up row r + N/2.
template <int EPI>
__global__ void __launch_bounds__(kThreads) l32_gemv_kernel(const float* __restrict__ W,
                                                            const float* __restrict__ x,
                                                            const float* __restrict__ norm_w,
                                                            float eps, int K, int N,
                                                            const float* resid, float* out) {
  extern __shared__ float xs[];
  __shared__ float red[kWarps];
  for (int i = threadIdx.x; i < K; i += kThreads) xs[i] = x[i];
  if (norm_w) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += kThreads) ss += xs[i] * xs[i];
    const float inv = rsqrtf(block_sum(ss, red) / K + eps);
    for (int i = threadIdx.x; i < K; i += kThreads) xs[i] = xs[i] * inv * norm_w[i];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = EPI == kL32Swiglu ? N / 2 : N;
  for (int r = blockIdx.x * kWarps + warp; r < rows; r += gridDim.x * kWarps) {
    const float acc = row_dot(W + (size_t)r * K, xs, K);
    if (EPI == kL32Swiglu) {
      const float up = row_dot(W + (size_t)(r + rows) * K, xs, K);
      if (lane == 0) out[r] = (acc / (1.0f + expf(-acc))) * up;
    } else if (lane == 0) {
      out[r] = EPI == kL32Resid ? resid[r] + acc : acc;
    }
  }
}

// q/k RMSNorm per head + RoPE at `pos`, then q -> qout and (k, v) -> KV row
// `pos` ([pos][K 1024 | V 1024]). One warp per head: warps 0..15 q, 16..23 k.
__global__ void __launch_bounds__(768) l32_qk_kernel(const float* qkv, const float* qn,
                                                     const float* kn, const float* rc,
                                                     const float* rs, int pos, float eps,
                                                     float* qout, float* kv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool isq = warp < kQHeads;
  const int h = isq ? warp : warp - kQHeads;
  const float* src = qkv + (isq ? h * kHeadDim : kQDim + h * kHeadDim);
  const float* w = isq ? qn : kn;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = src[lane + 32 * i];
  const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
  const float inv = rsqrtf(ss / kHeadDim + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = v[i] * inv * w[lane + 32 * i];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int j = lane + 32 * i;
    const float c = rc[pos * 64 + j], s = rs[pos * 64 + j];
    const float lo = v[i], hi = v[i + 2];
    v[i] = lo * c - hi * s;
    v[i + 2] = hi * c + lo * s;
  }
  float* dst = isq ? qout + h * kHeadDim : kv + (size_t)pos * 2 * kKvDim + h * kHeadDim;
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = v[i];
  if (!isq) {
    float* vd = kv + (size_t)pos * 2 * kKvDim + kKvDim + h * kHeadDim;
    const float* vs = qkv + kQDim + kKvDim + h * kHeadDim;
#pragma unroll
    for (int i = 0; i < 4; ++i) vd[lane + 32 * i] = vs[lane + 32 * i];
  }
}

// One block per q head over positions [0, S): scores in shared memory,
// softmax with expf, out = (sum_j p_j v_j) * (1 / sum_j p_j).
__global__ void __launch_bounds__(kThreads) l32_attn_kernel(const float* q, const float* kv, int S,
                                                            float* out) {
  extern __shared__ float sc[];
  __shared__ float qs[kHeadDim];
  __shared__ float red[kWarps];
  __shared__ float acc2[kHeadDim];
  const int h = blockIdx.x, g = h / (kQHeads / kKvHeads);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x < kHeadDim) qs[threadIdx.x] = q[h * kHeadDim + threadIdx.x];
  __syncthreads();
  const float scale = 1.0f / sqrtf(static_cast<float>(kHeadDim));
  const float4 q4 = reinterpret_cast<const float4*>(qs)[lane];
  for (int p = warp; p < S; p += kWarps) {
    const float4 k = reinterpret_cast<const float4*>(kv + (size_t)p * 2 * kKvDim + g * kHeadDim)[lane];
    const float d = warp_sum(k.x * q4.x + k.y * q4.y + k.z * q4.z + k.w * q4.w);
    if (lane == 0) sc[p] = d * scale;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int p = threadIdx.x; p < S; p += kThreads) m = fmaxf(m, sc[p]);
  m = block_max(m, red);
  float sum = 0.f;
  for (int p = threadIdx.x; p < S; p += kThreads) {
    const float e = expf(sc[p] - m);
    sc[p] = e;
    sum += e;
  }
  sum = block_sum(sum, red);
  __syncthreads();
  const int d = threadIdx.x & (kHeadDim - 1), half = threadIdx.x >> 7;
  float acc = 0.f;
  for (int p = half; p < S; p += 2)
    acc = fmaf(sc[p], kv[(size_t)p * 2 * kKvDim + kKvDim + g * kHeadDim + d], acc);
  if (half == 1) acc2[d] = acc;
  __syncthreads();
  if (half == 0) out[h * kHeadDim + d] = (acc + acc2[d]) * (1.0f / sum);
}

int gemv_grid(int rows) {
  const int g = (rows + kWarps - 1) / kWarps;
  return g < 148 * 8 ? g : 148 * 8;
}

}  // namespace

struct Layer32 {
  int max_seq;
  float eps, theta;
  // weights: qkv [4096, 2048], o [2048, 2048], gateup [12288, 2048] (gate | up),
  // down [2048, 6144]; norms [2048] x 2, q/k norms [128] x 2
  float *qkv = nullptr, *o = nullptr, *gu = nullptr, *down = nullptr;
  float *in_ln = nullptr, *post_ln = nullptr, *qn = nullptr, *kn = nullptr;
  float *rc = nullptr, *rs = nullptr, *kv = nullptr;
  float *x = nullptr, *t_qkv = nullptr, *t_q = nullptr, *t_att = nullptr, *t_h = nullptr,
        *t_act = nullptr, *t_out = nullptr;
  unsigned set_mask = 0;
  int len = 0;

  Layer32(int max_seq_len, float eps_, float theta_) : max_seq(max_seq_len), eps(eps_), theta(theta_) {
    qkv = dalloc<float>((size_t)kQkvDim * kHidden);
    o = dalloc<float>((size_t)kHidden * kQDim);
    gu = dalloc<float>((size_t)2 * kInter * kHidden);
    down = dalloc<float>((size_t)kHidden * kInter);
    in_ln = dalloc<float>(kHidden);
    post_ln = dalloc<float>(kHidden);
    qn = dalloc<float>(kHeadDim);
    kn = dalloc<float>(kHeadDim);
    rc = dalloc<float>((size_t)max_seq * 64);
    rs = dalloc<float>((size_t)max_seq * 64);
    kv = dalloc<float>((size_t)max_seq * 2 * kKvDim);
    x = dalloc<float>(kHidden);
    t_qkv = dalloc<float>(kQkvDim);
    t_q = dalloc<float>(kQDim);
    t_att = dalloc<float>(kQDim);
    t_h = dalloc<float>(kHidden);
    t_act = dalloc<float>(kInter);
    t_out = dalloc<float>(kHidden);
    launch_rope_table(rc, rs, max_seq, theta, 0);
    ORX_CHECK(cudaMemset(kv, 0, (size_t)max_seq * 2 * kKvDim * 4));
    ORX_CHECK(cudaDeviceSynchronize());
  }
  ~Layer32() {
    for (float* p : {qkv, o, gu, down, in_ln, post_ln, qn, kn, rc, rs, kv, x, t_qkv, t_q, t_att,
                     t_h, t_act, t_out})
      if (p) cudaFree(p);
  }

  // Layer-relative tensor names as in thinker.model.layers.N.<name>.weight.
  void set_tensor(const std::string& name, const float* src, size_t n, bool device_src) {
    struct Slot { const char* name; float* dst; size_t off, n; int bit; };
    const Slot slots[] = {
        {"input_layernorm", in_ln, 0, (size_t)kHidden, 0},
        {"post_attention_layernorm", post_ln, 0, (size_t)kHidden, 1},
        {"self_attn.q_norm", qn, 0, (size_t)kHeadDim, 2},
        {"self_attn.k_norm", kn, 0, (size_t)kHeadDim, 3},
        {"self_attn.q_proj", qkv, 0, (size_t)kQDim * kHidden, 4},
        {"self_attn.k_proj", qkv, (size_t)kQDim * kHidden, (size_t)kKvDim * kHidden, 5},
        {"self_attn.v_proj", qkv, (size_t)(kQDim + kKvDim) * kHidden, (size_t)kKvDim * kHidden, 6},
        {"self_attn.o_proj", o, 0, (size_t)kHidden * kQDim, 7},
        {"mlp.gate_proj", gu, 0, (size_t)kInter * kHidden, 8},
        {"mlp.up_proj", gu, (size_t)kInter * kHidden, (size_t)kInter * kHidden, 9},
        {"mlp.down_proj", down, 0, (size_t)kHidden * kInter, 10},
    };
    for (const Slot& s : slots) {
      if (name != s.name) continue;
      if (n != s.n) throw std::invalid_argument("tensor " + name + ": wrong element count");
      ORX_CHECK(cudaMemcpy(s.dst + s.off, src, n * 4,
                           device_src ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice));
      set_mask |= 1u << s.bit;
      return;
    }
    throw std::invalid_argument("unknown layer tensor " + name);
  }
  bool complete() const { return set_mask == (1u << 11) - 1; }

  // Seeded synthetic fp32 weights of decoder layer `layer` (unrounded values
  // of the same generator as the bf16 model).
  void init_synthetic(int seed, int layer) {
    static const char* names[] = {"input_layernorm", "post_attention_layernorm", "self_attn.q_norm",
                                  "self_attn.k_norm", "self_attn.q_proj", "self_attn.k_proj",
                                  "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
                                  "mlp.up_proj", "mlp.down_proj"};
    const size_t numel[] = {(size_t)kHidden, (size_t)kHidden, (size_t)kHeadDim, (size_t)kHeadDim,
                            (size_t)kQDim * kHidden, (size_t)kKvDim * kHidden,
                            (size_t)kKvDim * kHidden, (size_t)kHidden * kQDim,
                            (size_t)kInter * kHidden, (size_t)kInter * kHidden,
                            (size_t)kHidden * kInter};
    float* tmp = dalloc<float>((size_t)kInter * kHidden);
    for (int j = 0; j < 11; ++j) {
      const bool norm = j < 4;
      launch_synth_f32(tmp, (long long)numel[j], seed, kLayerBase + layer * kLayerStride + j, 0.02,
                       norm ? 1.0f : 0.0f, 0, 0);
      ORX_CHECK(cudaDeviceSynchronize());
      set_tensor(names[j], tmp, numel[j], true);
    }
    cudaFree(tmp);
  }

  // One row: xin (device [2048]) at position pos -> xout (device [2048]).
  void row(const float* xin, int pos, float* xout, cudaStream_t s) {
    l32_gemv_kernel<kL32Store><<<gemv_grid(kQkvDim), kThreads, kHidden * 4, s>>>(
        qkv, xin, in_ln, eps, kHidden, kQkvDim, nullptr, t_qkv);
    l32_qk_kernel<<<1, 32 * (kQHeads + kKvHeads), 0, s>>>(t_qkv, qn, kn, rc, rs, pos, eps, t_q, kv);
    l32_attn_kernel<<<kQHeads, kThreads, (size_t)(pos + 1) * 4, s>>>(t_q, kv, pos + 1, t_att);
    l32_gemv_kernel<kL32Resid><<<gemv_grid(kHidden), kThreads, kQDim * 4, s>>>(
        o, t_att, nullptr, eps, kQDim, kHidden, xin, t_h);
    l32_gemv_kernel<kL32Swiglu><<<gemv_grid(kInter), kThreads, kHidden * 4, s>>>(
        gu, t_h, post_ln, eps, kHidden, 2 * kInter, nullptr, t_act);
    l32_gemv_kernel<kL32Resid><<<gemv_grid(kHidden), kThreads, kInter * 4, s>>>(
        down, t_act, nullptr, eps, kInter, kHidden, t_h, xout);
  }

  // T rows (device [T, 2048]) at positions pos0.. -> device [T, 2048].
  void forward(const float* d_in, int T, int pos0, float* d_out, cudaStream_t s) {
    if (T <= 0) return;
    if (!complete()) throw std::invalid_argument("layer weights not loaded");
    if (pos0 < 0 || pos0 > len || pos0 + T > max_seq)
      throw std::invalid_argument("position out of range");
    for (int t = 0; t < T; ++t) row(d_in + (size_t)t * kHidden, pos0 + t, d_out + (size_t)t * kHidden, s);
    ORX_CHECK(cudaGetLastError());
    len = pos0 + T;
  }
};

Layer32* layer32_create(int max_seq_len, float eps, float theta) {
  static std::atomic<unsigned long long> configured{0};
  once_per_device(configured, [] {
    cudaFuncSetAttribute(l32_gemv_kernel<kL32Resid>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kInter * 4);
    cudaFuncSetAttribute(l32_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  if (max_seq_len < 1 || (size_t)max_seq_len * 4 > 200 * 1024)
    throw std::invalid_argument("max_seq_len out of range for the fp32 layer");
  return new Layer32(max_seq_len, eps, theta);
}
void layer32_destroy(Layer32* l) { delete l; }
void layer32_set_tensor(Layer32* l, const char* name, const float* src, size_t n, bool dev) {
  l->set_tensor(name, src, n, dev);
}
void layer32_init_synthetic(Layer32* l, int seed, int layer) { l->init_synthetic(seed, layer); }
void layer32_forward(Layer32* l, const float* d_in, int T, int pos0, float* d_out, cudaStream_t s) {
  l->forward(d_in, T, pos0, d_out, s);
}
int layer32_len(const Layer32* l) { return l->len; }
void layer32_truncate(Layer32* l, int n) {
  if (n < 0 || n > l->len) throw std::invalid_argument("truncate length out of range");
  l->len = n;
}

}  // namespace orx
