// The reference's free operators (asr_ops / asr_gemm) as standalone device
// launchers over caller-owned fp32 / bf16 device buffers: RMSNorm, RoPE
// (rotate_half and interleaved), SwiGLU, grouped-query attention, banned
// argmax, the bf16 casts and the bf16 Linear with bias + GELU / ReLU.
//
// Replaces include/model/asr_ops.cuh:24-62 (src/model/asr_ops.cu) and
// include/model/asr_gemm.h:24-41 (src/model/asr_gemm.cu). The decoder itself
// does not call these (its norms, RoPE, SwiGLU and argmax are fused into the
// projection and attention kernels); they exist for callers of the reference
// API outside the decoder (e.g. an aligner or an encoder built on the same
// operators). Every one is an HBM-bound elementwise / reduction kernel except
// the Linear, which runs on the tcgen05 GEMM (gemm_tc.cu) with a bias +
// activation epilogue.
#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace orx {
namespace {

// ---- RMSNorm: one CTA per row -------------------------------------------
// out = x * rsqrtf(mean(x^2) + eps) * w, the reference's order of operations
// (asr_ops.cu:21-49); the sum of squares is a warp-shuffle tree.
__global__ void __launch_bounds__(256) op_rmsnorm_kernel(const float* __restrict__ x,
                                                         const float* __restrict__ w,
                                                         float* __restrict__ out, int dim,
                                                         float eps, int vec) {
  __shared__ float red[8];
  const long long r = blockIdx.x;
  const float* xr = x + r * dim;
  float* yr = out + r * dim;
  float ss = 0.f;
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) {
      const float4 v = x4[i];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss += xr[i] * xr[i];
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / dim + eps);
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    float4* y4 = reinterpret_cast<float4*>(yr);
    for (int i = threadIdx.x; i < dim / 4; i += blockDim.x) {
      const float4 v = x4[i], g = w4[i];
      y4[i] = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
    }
  } else {
    for (int i = threadIdx.x; i < dim; i += blockDim.x) yr[i] = xr[i] * inv * w[i];
  }
}

// ---- RoPE: one CTA per (token, head), threads over the rotated pairs -----
// The angle is the reference's: pos * powf(base, -2 j / D) with precise
// cosf / sinf (asr_ops.cu:55-112).
template <bool kHalf>
__global__ void op_rope_kernel(float* __restrict__ x, const int* __restrict__ pos, int H, int D,
                               float base) {
  const int t = blockIdx.x, h = blockIdx.y;
  float* xr = x + (static_cast<long long>(t) * H + h) * D;
  const int half = D / 2;
  const float p = static_cast<float>(pos[t]);
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    const float inv_freq = powf(base, -2.0f * j / D);
    const float ang = p * inv_freq;
    const float c = cosf(ang), s = sinf(ang);
    if (kHalf) {
      const float a = xr[j], b = xr[j + half];
      xr[j] = a * c - b * s;
      xr[j + half] = b * c + a * s;
    } else {
      const float a = xr[2 * j], b = xr[2 * j + 1];
      xr[2 * j] = a * c - b * s;
      xr[2 * j + 1] = a * s + b * c;
    }
  }
}

// ---- SwiGLU: out = g / (1 + expf(-g)) * u --------------------------------
__global__ void op_swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u,
                                 float* __restrict__ o, long long n) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += stride) {
    const float gv = g[i];
    o[i] = (gv / (1.0f + expf(-gv))) * u[i];
  }
}

// ---- banned argmax: one CTA of 1024 threads, no scratch -------------------
// The tie rule of the reference's ArgmaxBannedKernel comes from argmax_key.
__global__ void __launch_bounds__(1024) op_argmax_kernel(const float* __restrict__ x, int n,
                                                         int ban0, int ban1, int* out) {
  __shared__ unsigned long long sb[32];
  unsigned long long best = 0ull;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (i == ban0 || i == ban1) continue;
    const unsigned long long k = argmax_key(x[i], i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if ((threadIdx.x & 31) == 0) sb[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x < 32) {
    unsigned long long b = sb[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ob = __shfl_xor_sync(0xffffffffu, b, o);
      b = ob > b ? ob : b;
    }
    if (threadIdx.x == 0) *out = argmax_key_index(b);
  }
}

// ---- grouped-query attention (fp32) ---------------------------------------
// q [T, Hq, D], k / v [T, Hkv, D], out [T, Hq, D]. A CTA serves one kv head
// and kGqaRows (query token, query head of the group) rows, one warp each;
// keys stream through shared memory in tiles of 32 shared by all its warps.
// Per tile, lane j scores key j against the warp's query (q broadcast from
// shared memory, K rows padded to D + 1 floats so the 32 lanes hit 32 banks),
// the tile's scores update the online softmax once, and each lane
// accumulates its D / 32 output dims over the tile's 32 value rows.
constexpr int kGqaRows = 8;
constexpr int kGqaTile = 32;

template <int E>  // E = D / 32 dims per lane
__global__ void __launch_bounds__(kGqaRows * 32) op_gqa_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    float* __restrict__ out, int T, int Hq, int Hkv, float scale, int causal) {
  constexpr int D = E * 32;
  extern __shared__ float gsm[];
  float* sq = gsm;                         // [kGqaRows][D]
  float* sk = sq + kGqaRows * D;           // [kGqaTile][D + 1]
  float* sv = sk + kGqaTile * (D + 1);     // [kGqaTile][D]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = Hq / Hkv, kvh = blockIdx.y;
  const int rows = T * G;
  const int r = blockIdx.x * kGqaRows + warp;
  const bool active = r < rows;
  const int i = active ? r / G : 0;
  const int h = kvh * G + (active ? r % G : 0);
  // the CTA's last query token bounds the causal key range of every warp
  const int r_last = min(rows - 1, blockIdx.x * kGqaRows + kGqaRows - 1);
  const int jend = causal ? r_last / G : T - 1;
  const int my_end = causal ? i : T - 1;
  if (active)
    for (int d = lane; d < D; d += 32) sq[warp * D + d] = q[(static_cast<long long>(i) * Hq + h) * D + d];
  float m = -1e30f, l = 0.f, acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  for (int j0 = 0; j0 <= jend; j0 += kGqaTile) {
    __syncthreads();  // previous tile consumed (and sq written on the first pass)
    for (int idx = threadIdx.x; idx < kGqaTile * D; idx += blockDim.x) {
      const int jj = idx / D, d = idx - jj * D, j = j0 + jj;
      const bool ok = j <= jend;
      const long long off = (static_cast<long long>(j) * Hkv + kvh) * D + d;
      sk[jj * (D + 1) + d] = ok ? k[off] : 0.f;
      sv[jj * D + d] = ok ? v[off] : 0.f;
    }
    __syncthreads();
    if (!active || j0 > my_end) continue;
    const float* qr = sq + warp * D;
    const float* kr = sk + lane * (D + 1);
    float s = 0.f;
#pragma unroll 8
    for (int d = 0; d < D; ++d) s += qr[d] * kr[d];
    const bool valid = j0 + lane <= my_end;
    s = valid ? s * scale : -INFINITY;
    const float mt = warp_max(s);
    const float mn = fmaxf(m, mt);
    const float corr = expf(m - mn);
    const float p = valid ? expf(s - mn) : 0.f;
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] *= corr;
    const int nj = min(kGqaTile, my_end - j0 + 1);
    for (int jj = 0; jj < nj; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] += pj * sv[jj * D + lane + 32 * e];
    }
    m = mn;
  }
  if (!active) return;
  const float invl = l > 0.f ? 1.0f / l : 0.f;
  float* orow = out + (static_cast<long long>(i) * Hq + h) * D;
#pragma unroll
  for (int e = 0; e < E; ++e) orow[lane + 32 * e] = acc[e] * invl;
}

// Head dims that are not a multiple of 32 or exceed 256: one warp per row,
// keys read from global memory (L2), per-key online softmax.
__global__ void op_gqa_generic_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                      const float* __restrict__ v, float* __restrict__ out, int T,
                                      int Hq, int Hkv, int D, float scale, int causal) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long r = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + warp;
  if (r >= static_cast<long long>(T) * Hq) return;
  const int i = static_cast<int>(r / Hq), h = static_cast<int>(r % Hq);
  const int kvh = h / (Hq / Hkv);
  const float* qr = q + r * D;
  float* orow = out + r * D;
  float m = -1e30f, l = 0.f;
  for (int d = lane; d < D; d += 32) orow[d] = 0.f;
  const int jend = causal ? i : T - 1;
  for (int j = 0; j <= jend; ++j) {
    const float* kr = k + (static_cast<long long>(j) * Hkv + kvh) * D;
    const float* vr = v + (static_cast<long long>(j) * Hkv + kvh) * D;
    float s = 0.f;
    for (int d = lane; d < D; d += 32) s += qr[d] * kr[d];
    s = warp_sum(s) * scale;
    const float mn = fmaxf(m, s);
    const float corr = expf(m - mn), p = expf(s - mn);
    l = l * corr + p;
    for (int d = lane; d < D; d += 32) orow[d] = orow[d] * corr + p * vr[d];
    m = mn;
  }
  const float invl = l > 0.f ? 1.0f / l : 0.f;
  for (int d = lane; d < D; d += 32) orow[d] *= invl;
}

// out[m, n] = act(sum_k X[m, k] W[n, k] + bias[n]): one warp per output,
// fp32 accumulation of exact bf16 products (shapes the tensor maps cannot
// describe: K not a multiple of 8).
__global__ void op_linear_simt_kernel(const uint16_t* __restrict__ X, const uint16_t* __restrict__ W,
                                      const float* __restrict__ bias, float* __restrict__ out,
                                      int M, int K, int N, int act) {
  const long long o = static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (o >= static_cast<long long>(M) * N) return;
  const int m = static_cast<int>(o / N), n = static_cast<int>(o % N);
  const uint16_t* xr = X + static_cast<long long>(m) * K;
  const uint16_t* wr = W + static_cast<long long>(n) * K;
  float acc = 0.f;
  for (int k = lane; k < K; k += 32) acc = fmaf(bf2f(xr[k]), bf2f(wr[k]), acc);
  acc = warp_sum(acc);
  if (lane == 0) {
    float y = acc + (bias ? bias[n] : 0.f);
    if (act == 1)
      y = 0.5f * y * (1.0f + erff(y * 0.70710678118654752440f));
    else if (act == 2)
      y = fmaxf(y, 0.0f);
    out[o] = y;
  }
}

template <int E>
cudaError_t launch_gqa_tiled(const float* q, const float* k, const float* v, float* out, int T,
                             int Hq, int Hkv, float scale, int causal, cudaStream_t s) {
  constexpr int D = E * 32;
  const size_t smem = sizeof(float) * (kGqaRows * D + kGqaTile * (D + 1) + kGqaTile * D);
  static std::atomic<unsigned long long> configured{0};
  once_per_device(configured, [&] {
    cudaFuncSetAttribute(op_gqa_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
  });
  const int G = Hq / Hkv;
  const dim3 grid((T * G + kGqaRows - 1) / kGqaRows, Hkv);
  op_gqa_kernel<E><<<grid, kGqaRows * 32, smem, s>>>(q, k, v, out, T, Hq, Hkv, scale, causal);
  return cudaGetLastError();
}

int grid_1d(long long n, int threads) {
  const long long b = (n + threads - 1) / threads;
  return static_cast<int>(b < 148 * 32 ? (b > 0 ? b : 1) : 148 * 32);
}

}  // namespace

void op_rms_norm(const float* x, const float* w, float* out, int rows, int dim, float eps,
                 cudaStream_t s) {
  const int vec = (dim % 4 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                  (reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                  (reinterpret_cast<uintptr_t>(out) % 16 == 0);
  op_rmsnorm_kernel<<<rows, 256, 0, s>>>(x, w, out, dim, eps, vec);
}

void op_rope(float* x, const int* pos, int n_tokens, int n_heads, int head_dim, float theta,
             bool rotate_half, cudaStream_t s) {
  const dim3 grid(n_tokens, n_heads);
  const int threads = head_dim / 2 < 256 ? (head_dim / 2 > 0 ? head_dim / 2 : 1) : 256;
  if (rotate_half)
    op_rope_kernel<true><<<grid, threads, 0, s>>>(x, pos, n_heads, head_dim, theta);
  else
    op_rope_kernel<false><<<grid, threads, 0, s>>>(x, pos, n_heads, head_dim, theta);
}

void op_swiglu(const float* g, const float* u, float* o, long long n, cudaStream_t s) {
  op_swiglu_kernel<<<grid_1d(n, 256), 256, 0, s>>>(g, u, o, n);
}

void op_argmax_banned(const float* x, int n, int ban0, int ban1, int* out, cudaStream_t s) {
  op_argmax_kernel<<<1, 1024, 0, s>>>(x, n, ban0, ban1, out);
}

cudaError_t op_gqa_attention(const float* q, const float* k, const float* v, float* out, int T,
                             int Hq, int Hkv, int D, float scale, bool causal, cudaStream_t s) {
  const int c = causal ? 1 : 0;
  switch (D) {
    case 32: return launch_gqa_tiled<1>(q, k, v, out, T, Hq, Hkv, scale, c, s);
    case 64: return launch_gqa_tiled<2>(q, k, v, out, T, Hq, Hkv, scale, c, s);
    case 96: return launch_gqa_tiled<3>(q, k, v, out, T, Hq, Hkv, scale, c, s);
    case 128: return launch_gqa_tiled<4>(q, k, v, out, T, Hq, Hkv, scale, c, s);
    case 256: return launch_gqa_tiled<8>(q, k, v, out, T, Hq, Hkv, scale, c, s);
    default: {
      const long long rows = static_cast<long long>(T) * Hq;
      op_gqa_generic_kernel<<<static_cast<int>((rows + 3) / 4), 128, 0, s>>>(q, k, v, out, T, Hq,
                                                                           Hkv, D, scale, c);
      return cudaGetLastError();
    }
  }
}

void op_linear_simt(const uint16_t* X, const uint16_t* W, const float* bias, float* out, int M,
                    int K, int N, int act, cudaStream_t s) {
  const long long outs = static_cast<long long>(M) * N;
  op_linear_simt_kernel<<<static_cast<int>((outs + 7) / 8), 256, 0, s>>>(X, W, bias, out, M, K, N,
                                                                         act);
}

}  // namespace orx
