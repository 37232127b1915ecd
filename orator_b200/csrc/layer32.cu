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
// launches per row chained by programmatic dependent launch: norm+qkv GEMV,
// attention (q/k norm + RoPE + KV store fused, split over positions), o GEMV
// (+residual), norm+gate/up GEMV (+SwiGLU), down GEMV (+residual). The GEMVs
// stream fp32 weights with 16-byte non-allocating loads, sixteen in flight per
// lane, the first chunk issued before waiting on the previous kernel; at
// 201 MB of weights per row they are HBM-bound.
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

// out[u] (op)= W[u, :] . act, act = RMSNorm(x) when norm_w is given, else x.
// kL32Swiglu: unit u pairs gate row u with up row u + N/2.
// One warp per unit; each chunk of the unit's row(s) is 16 float4 per lane in
// flight (2048 floats of one row, or 1024 of each of the two SwiGLU rows).
// Launched with programmatic dependent launch: the CTA releases its
// dependents at once, streams the first chunk of its first unit (weights do
// not depend on earlier kernels), and only then waits for the producer of x.
template <int EPI>
__global__ void __launch_bounds__(kThreads, 2) l32_gemv_kernel(const float* __restrict__ W,
                                                               const float* __restrict__ x,
                                                               const float* __restrict__ norm_w,
                                                               float eps, int K, int N,
                                                               const float* resid, float* out) {
  constexpr int R = EPI == kL32Swiglu ? 2 : 1;
  constexpr int V = 16 / R;
  constexpr int kChunk = V * 32 * 4;  // floats of one row per chunk
  extern __shared__ float xs[];
  __shared__ float red[kWarps];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int units = EPI == kL32Swiglu ? N / 2 : N;
  const int nchunks = K / kChunk;
  const int stride = gridDim.x * kWarps;
  int u = blockIdx.x * kWarps + warp;
  float4 buf[R][V];
  auto load = [&](int unit, int c) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float4* w4 = reinterpret_cast<const float4*>(
          W + (size_t)(unit + r * units) * K + (size_t)c * kChunk);
#pragma unroll
      for (int j = 0; j < V; ++j) buf[r][j] = ld_stream(w4 + lane + 32 * j);
    }
  };
  pdl_trigger();
  if (u < units) load(u, 0);
  pdl_wait();
  for (int i = threadIdx.x; i < K; i += kThreads) xs[i] = x[i];
  if (norm_w) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += kThreads) ss += xs[i] * xs[i];
    const float inv = rsqrtf(block_sum(ss, red) / K + eps);
    for (int i = threadIdx.x; i < K; i += kThreads) xs[i] = xs[i] * inv * norm_w[i];
  }
  __syncthreads();
  bool loaded = true;
  for (; u < units; u += stride) {
    float acc[R][4];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r][0] = acc[r][1] = acc[r][2] = acc[r][3] = 0.f;
    for (int c = 0; c < nchunks; ++c) {
      if (!loaded) load(u, c);
      loaded = false;
      const float4* x4 = reinterpret_cast<const float4*>(xs + c * kChunk);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float4 xv = x4[lane + 32 * j];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          acc[r][0] = fmaf(buf[r][j].x, xv.x, acc[r][0]);
          acc[r][1] = fmaf(buf[r][j].y, xv.y, acc[r][1]);
          acc[r][2] = fmaf(buf[r][j].z, xv.z, acc[r][2]);
          acc[r][3] = fmaf(buf[r][j].w, xv.w, acc[r][3]);
        }
      }
    }
    const float a = warp_sum((acc[0][0] + acc[0][1]) + (acc[0][2] + acc[0][3]));
    if (EPI == kL32Swiglu) {
      const float up = warp_sum((acc[R - 1][0] + acc[R - 1][1]) + (acc[R - 1][2] + acc[R - 1][3]));
      if (lane == 0) out[u] = (a / (1.0f + expf(-a))) * up;
    } else if (lane == 0) {
      out[u] = EPI == kL32Resid ? resid[u] + a : a;
    }
  }
}

// Decode attention of one row at position `pos`, split over positions:
// grid (splits of kAttnChunk positions, kv heads). Each CTA normalises and
// ropes the q rows of its kv head's two query heads and the new k row
// (q/k RMSNorm per head, rotate-half RoPE), takes the new v row, stages its
// positions' K / V rows in shared memory (the new row in place of position
// `pos`; the CTA holding `pos` also stores it into the cache), and writes a
// partial softmax (max, sum, weighted V) per query head. The last CTA of the
// kv head merges the partials in split order (deterministic).
constexpr int kAttnChunk = 64;

__global__ void __launch_bounds__(kThreads) l32_attn_kernel(const float* __restrict__ qkv,
                                                            const float* __restrict__ qn,
                                                            const float* __restrict__ kn,
                                                            const float* __restrict__ rc,
                                                            const float* __restrict__ rs, int pos,
                                                            float eps, float* kv, float* part,
                                                            int part_stride, int* counters,
                                                            float* out) {
  extern __shared__ float sm[];
  float* ks = sm;                                  // [kAttnChunk][128]
  float* vs = ks + kAttnChunk * kHeadDim;          // [kAttnChunk][128]
  __shared__ float qs[kGroup][kHeadDim];
  __shared__ float knew[kHeadDim], vnew[kHeadDim];
  __shared__ float sc[kGroup][kAttnChunk];
  __shared__ int last;
  const int split = blockIdx.x, g = blockIdx.y, splits = gridDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = pos + 1;
  const int s0 = split * kAttnChunk, n = min(kAttnChunk, S - s0);
  pdl_trigger();
  pdl_wait();
  if (warp <= kGroup) {  // q rows of the group (warps 0, 1) and the new k row (warp 2)
    const bool isq = warp < kGroup;
    const float* src = isq ? qkv + (g * kGroup + warp) * kHeadDim : qkv + kQDim + g * kHeadDim;
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
    float* dst = isq ? qs[warp] : knew;
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = v[i];
  } else if (warp == kGroup + 1) {
    const float* src = qkv + kQDim + kKvDim + g * kHeadDim;
#pragma unroll
    for (int i = 0; i < 4; ++i) vnew[lane + 32 * i] = src[lane + 32 * i];
  }
  // past positions of this split: K and V rows of head g
#pragma unroll
  for (int it = 0; it < kAttnChunk * (kHeadDim / 4) / kThreads; ++it) {
    const int idx = threadIdx.x + it * kThreads;
    const int j = idx / (kHeadDim / 4), d4 = idx - j * (kHeadDim / 4);
    if (j >= n || s0 + j == pos) continue;
    const float4* row = reinterpret_cast<const float4*>(kv + (size_t)(s0 + j) * 2 * kKvDim + g * kHeadDim);
    reinterpret_cast<float4*>(ks + j * kHeadDim)[d4] = row[d4];
    reinterpret_cast<float4*>(vs + j * kHeadDim)[d4] = row[kKvDim / 4 + d4];
  }
  __syncthreads();
  if (pos >= s0 && pos < s0 + n && threadIdx.x < kHeadDim) {
    const int j = pos - s0, d = threadIdx.x;
    ks[j * kHeadDim + d] = knew[d];
    vs[j * kHeadDim + d] = vnew[d];
    kv[(size_t)pos * 2 * kKvDim + g * kHeadDim + d] = knew[d];
    kv[(size_t)pos * 2 * kKvDim + kKvDim + g * kHeadDim + d] = vnew[d];
  }
  __syncthreads();
  const float scale = 1.0f / sqrtf(static_cast<float>(kHeadDim));
  for (int j = warp; j < n; j += kWarps) {
    const float4 k4 = reinterpret_cast<const float4*>(ks + j * kHeadDim)[lane];
#pragma unroll
    for (int h = 0; h < kGroup; ++h) {
      const float4 q4 = reinterpret_cast<const float4*>(qs[h])[lane];
      const float d = warp_sum(k4.x * q4.x + k4.y * q4.y + k4.z * q4.z + k4.w * q4.w);
      if (lane == 0) sc[h][j] = d * scale;
    }
  }
  __syncthreads();
  float* pb = part + (size_t)g * kGroup * part_stride * (kHeadDim + 2);
  if (warp < kGroup) {  // per-head max, exponentials and sum over this split
    const int h = warp;
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[h][j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float e = expf(sc[h][j] - m);
      sc[h][j] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      float* ph = pb + ((size_t)h * part_stride + split) * (kHeadDim + 2);
      ph[0] = m;
      ph[1] = l;
    }
  }
  __syncthreads();
  {
    const int h = threadIdx.x / kHeadDim, d = threadIdx.x % kHeadDim;  // 256 threads = 2 heads
    float acc = 0.f;
    for (int j = 0; j < n; ++j) acc = fmaf(sc[h][j], vs[j * kHeadDim + d], acc);
    pb[((size_t)h * part_stride + split) * (kHeadDim + 2) + 2 + d] = acc;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(&counters[g], 1) == splits - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  {
    const int h = threadIdx.x / kHeadDim, d = threadIdx.x % kHeadDim;
    const float* ph = pb + (size_t)h * part_stride * (kHeadDim + 2);
    float M = -INFINITY;
#pragma unroll 8
    for (int sp = 0; sp < splits; ++sp) M = fmaxf(M, __ldcg(ph + (size_t)sp * (kHeadDim + 2)));
    float L = 0.f, A = 0.f;
    for (int sp0 = 0; sp0 < splits; sp0 += 8) {  // eight splits' loads in flight
      float mv[8], lv[8], av[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float* q = ph + (size_t)min(sp0 + i, splits - 1) * (kHeadDim + 2);
        mv[i] = __ldcg(q);
        lv[i] = __ldcg(q + 1);
        av[i] = __ldcg(q + 2 + d);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (sp0 + i >= splits) break;
        const float e = expf(mv[i] - M);
        L = fmaf(lv[i], e, L);
        A = fmaf(av[i], e, A);
      }
    }
    out[(g * kGroup + h) * kHeadDim + d] = A * (1.0f / L);
  }
  if (threadIdx.x == 0) counters[g] = 0;
}

int g_gemv_slots = 148 * 2;  // GEMV grid cap: resident CTAs (set at configuration)

int gemv_grid(int units) {
  const int g = (units + kWarps - 1) / kWarps;
  return g < g_gemv_slots ? g : g_gemv_slots;
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
        *t_act = nullptr, *t_out = nullptr, *part = nullptr;
  int* counters = nullptr;
  int max_splits = 0;
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
    max_splits = (max_seq + kAttnChunk - 1) / kAttnChunk;
    part = dalloc<float>((size_t)kQHeads * max_splits * (kHeadDim + 2));
    counters = dalloc<int>(kKvHeads);
    ORX_CHECK(cudaMemset(counters, 0, kKvHeads * sizeof(int)));
    launch_rope_table(rc, rs, max_seq, theta, 0);
    ORX_CHECK(cudaMemset(kv, 0, (size_t)max_seq * 2 * kKvDim * 4));
    ORX_CHECK(cudaDeviceSynchronize());
  }
  ~Layer32() {
    for (float* p : {qkv, o, gu, down, in_ln, post_ln, qn, kn, rc, rs, kv, x, t_qkv, t_q, t_att,
                     t_h, t_act, t_out, part})
      if (p) cudaFree(p);
    if (counters) cudaFree(counters);
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
  // Five launches chained by programmatic dependent launch.
  void row(const float* xin, int pos, float* xout, cudaStream_t s) {
    ORX_CHECK(launch_pdl(l32_gemv_kernel<kL32Store>, dim3(gemv_grid(kQkvDim)), dim3(kThreads),
                         kHidden * 4, s, (const float*)qkv, xin, (const float*)in_ln, eps, kHidden,
                         kQkvDim, (const float*)nullptr, t_qkv));
    const int splits = (pos + 1 + kAttnChunk - 1) / kAttnChunk;
    ORX_CHECK(launch_pdl(l32_attn_kernel, dim3(splits, kKvHeads), dim3(kThreads),
                         (size_t)2 * kAttnChunk * kHeadDim * 4, s, (const float*)t_qkv,
                         (const float*)qn, (const float*)kn, (const float*)rc, (const float*)rs, pos,
                         eps, kv, part, max_splits, counters, t_att));
    ORX_CHECK(launch_pdl(l32_gemv_kernel<kL32Resid>, dim3(gemv_grid(kHidden)), dim3(kThreads),
                         kQDim * 4, s, (const float*)o, (const float*)t_att, (const float*)nullptr,
                         eps, kQDim, kHidden, xin, t_h));
    ORX_CHECK(launch_pdl(l32_gemv_kernel<kL32Swiglu>, dim3(gemv_grid(kInter)), dim3(kThreads),
                         kHidden * 4, s, (const float*)gu, (const float*)t_h, (const float*)post_ln,
                         eps, kHidden, 2 * kInter, (const float*)nullptr, t_act));
    ORX_CHECK(launch_pdl(l32_gemv_kernel<kL32Resid>, dim3(gemv_grid(kHidden)), dim3(kThreads),
                         kInter * 4, s, (const float*)down, (const float*)t_act,
                         (const float*)nullptr, eps, kInter, kHidden, (const float*)t_h, xout));
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
    cudaFuncSetAttribute(l32_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         2 * kAttnChunk * kHeadDim * 4);
    int per_sm = 0, dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, l32_gemv_kernel<kL32Swiglu>,
                                                      kThreads, kHidden * 4) == cudaSuccess &&
        per_sm > 0)
      g_gemv_slots = sms * per_sm;
  });
  if (max_seq_len < 1 || max_seq_len > (1 << 20))
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
