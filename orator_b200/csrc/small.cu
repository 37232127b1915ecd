// Small kernels of the decoder path: prefill RMSNorm, argmax, RoPE table,
// casts, embedding gather and the synthetic-weight generator.
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace orx {
namespace {

// RMSNorm of rows of 2048 to bf16 (asr_ops.cu:21-51 + asr_gemm.cu:45-50).
__global__ void __launch_bounds__(256) rmsnorm_bf16_kernel(const float* x, const float* w,
                                                           uint16_t* out, float eps) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  const int row = blockIdx.x, t = threadIdx.x;
  const float4* xi = reinterpret_cast<const float4*>(x + (long long)row * kHidden) + t * 2;
  const float4 p0 = xi[0], p1 = xi[1];
  const float v[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  ss = warp_sum(ss);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / kHidden + eps);
  const float4* wi = reinterpret_cast<const float4*>(w) + t * 2;
  const float4 w0 = wi[0], w1 = wi[1];
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  uint32_t pk[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    pk[j] = static_cast<uint32_t>(f2bf(v[2 * j] * inv * wv[2 * j])) |
            (static_cast<uint32_t>(f2bf(v[2 * j + 1] * inv * wv[2 * j + 1])) << 16);
  reinterpret_cast<uint4*>(out + (long long)row * kHidden)[t] =
      make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// Multi-CTA banned argmax (replaces the single-block ArgmaxBannedKernel,
// asr_ops.cu:300-325); exact ties resolve as that kernel does (argmax_key).
__global__ void __launch_bounds__(256) argmax_kernel(const float* x, int n, int ban0, int ban1,
                                                     StepState* st, int* out_dev) {
  pdl_trigger();
  pdl_wait();
  __shared__ unsigned long long sb[8];
  unsigned long long best = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    if (i == ban0 || i == ban1) continue;
    const float v = x[i];
    if (v != v) continue;
    const unsigned long long k = argmax_key(v, i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if ((threadIdx.x & 31) == 0) sb[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < 8; ++w) b = sb[w] > b ? sb[w] : b;
    if (b) atomicMax(&st->best, b);
    __threadfence();
    if (atomicAdd(&st->done, 1) == gridDim.x - 1) {
      __threadfence();
      const unsigned long long fin = atomicExch(&st->best, 0ull);
      st->done = 0;
      const int idx = fin ? argmax_key_index(fin) : 0;
      st->tok = idx;
      if (out_dev) *out_dev = idx;
    }
  }
}

// cos/sin table with the reference's angle math (asr_ops.cu:101-105):
// inv_freq = powf(theta, -2j/128), angle = (float)pos * inv_freq.
__global__ void rope_table_kernel(float* c, float* s, int max_pos, float theta) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= max_pos * 64) return;
  const int p = i / 64, j = i % 64;
  const float inv_freq = powf(theta, -2.0f * j / kHeadDim);
  const float ang = static_cast<float>(p) * inv_freq;
  c[i] = cosf(ang);
  s[i] = sinf(ang);
}

__device__ __forceinline__ unsigned long long splitmix64(unsigned long long x) {
  x += 0x9E3779B97F4A7C15ull;
  unsigned long long z = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Bit-exact twin of oracle/synth.py normal_f32 (Irwin-Hall of four 16-bit fields).
__device__ __forceinline__ float synth_value(int seed, int tid, long long i, float scale,
                                             float mean) {
  const unsigned long long key = (static_cast<unsigned long long>(seed & 0xFFF) << 52) |
                                 (static_cast<unsigned long long>(tid & 0xFFFF) << 36) |
                                 static_cast<unsigned long long>(i);
  const unsigned long long h = splitmix64(key);
  const long long tot = static_cast<long long>((h & 0xFFFF) + ((h >> 16) & 0xFFFF) +
                                               ((h >> 32) & 0xFFFF) + (h >> 48)) -
                        131070;
  float v = __fmul_rn(static_cast<float>(tot), scale);
  if (mean != 0.0f) v = __fadd_rn(v, mean);
  return v;
}

__global__ void synth_bf16_kernel(uint16_t* dst, long long n, int seed, int tid, float scale,
                                  float mean) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    dst[i] = f2bf(synth_value(seed, tid, i, scale, mean));
}

__global__ void synth_f32_kernel(float* dst, long long n, int seed, int tid, float scale,
                                 float mean, int round_bf16) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const float v = synth_value(seed, tid, i, scale, mean);
    dst[i] = round_bf16 ? bf2f(f2bf(v)) : v;
  }
}

__global__ void f32_to_bf16_kernel(const float* in, uint16_t* out, long long n) {
  pdl_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = f2bf(in[i]);
}
__global__ void bf16_to_f32_kernel(const uint16_t* in, float* out, long long n) {
  pdl_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    out[i] = bf2f(in[i]);
}

__global__ void embed_rows_kernel(const uint16_t* table, const int* ids, float* out) {
  pdl_wait();
  const int row = blockIdx.x;
  const uint16_t* src = table + (long long)ids[row] * kHidden;
  for (int i = threadIdx.x; i < kHidden; i += blockDim.x)
    out[(long long)row * kHidden + i] = bf2f(src[i]);
}

inline int grid_for(long long n) {
  long long g = (n + 255) / 256;
  return static_cast<int>(g > 148 * 64 ? 148 * 64 : (g < 1 ? 1 : g));
}

}  // namespace

void launch_rmsnorm_bf16(const float* x, const float* w, uint16_t* out, int rows, float eps,
                         cudaStream_t s) {
  if (rows <= 0) return;
  launch_pdl(rmsnorm_bf16_kernel, dim3(rows), dim3(256), 0, s, x, w, out, eps);
}

void launch_argmax(const float* logits, int n, int ban0, int ban1, StepState* st, int* out_dev,
                   cudaStream_t s) {
  launch_pdl(argmax_kernel, dim3(148), dim3(256), 0, s, logits, n, ban0, ban1, st, out_dev);
}

void launch_rope_table(float* c, float* sn, int max_pos, float theta, cudaStream_t s) {
  const int n = max_pos * 64;
  rope_table_kernel<<<(n + 255) / 256, 256, 0, s>>>(c, sn, max_pos, theta);
}

void launch_synth_bf16(uint16_t* dst, long long n, int seed, int tid, double std, float mean,
                       cudaStream_t s) {
  synth_bf16_kernel<<<grid_for(n), 256, 0, s>>>(dst, n, seed, tid, static_cast<float>(std / 37837.227), mean);
}
void launch_synth_f32(float* dst, long long n, int seed, int tid, double std, float mean,
                      int round_bf16, cudaStream_t s) {
  synth_f32_kernel<<<grid_for(n), 256, 0, s>>>(dst, n, seed, tid, static_cast<float>(std / 37837.227), mean, round_bf16);
}
void launch_f32_to_bf16(const float* in, uint16_t* out, long long n, cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(f32_to_bf16_kernel, dim3(grid_for(n)), dim3(256), 0, s, in, out, n);
}
void launch_bf16_to_f32(const uint16_t* in, float* out, long long n, cudaStream_t s) {
  if (n <= 0) return;
  launch_pdl(bf16_to_f32_kernel, dim3(grid_for(n)), dim3(256), 0, s, in, out, n);
}
void launch_embed_rows(const uint16_t* table, const int* ids, float* out, int rows,
                       cudaStream_t s) {
  if (rows <= 0) return;
  launch_pdl(embed_rows_kernel, dim3(rows), dim3(256), 0, s, table, ids, out);
}

}  // namespace orx
