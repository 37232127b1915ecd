// Streaming Sortformer diarizer network on B200 (fp32 model, fp32-grade
// arithmetic): the pre-encode, the 17 FastConformer layers and the 18-layer
// transformer decoder with its speaker head.
//
// Replaces ConformerPreEncode (src/model/conformer_preencode.cu:196-279),
// ConformerLayer (src/model/conformer_layer.cu:330-452), SortformerDecoder
// (src/model/sortformer_decoder.cu:240-333) and the network part of
// SortformerDiarizer (ForwardEncoderDecoder, src/model/streaming_sortformer.cc
// :391-418; the [spkcache | fifo | chunk] concatenation of StreamMelChunk,
// :500-537).
//
// Every Linear / pointwise convolution runs on the tcgen05 GEMM (gemm_tc.cu)
// with fp32-grade accuracy from bf16 operands: an fp32 operand x is split into
// hi = bf16(x) and lo = bf16(x - hi), the activation row is stored as
// [hi | hi | lo] and the weight row as [Wh | Wl | Wh], so one GEMM of depth
// 3K sums xh*Wh + xh*Wl + xl*Wh in fp32 (relative error about 2^-16 per
// product, against 2^-24 for the reference's fp32 SGEMM). LayerNorms, the
// depthwise convolutions and the GEMM epilogues write activations directly
// in that split form. Attention (relative-position MHSA in the conformer,
// plain MHSA in the decoder), softmax, LayerNorm, BatchNorm and the
// convolutions of the pre-encode stay fp32 on the SIMT pipes.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "engine.h"
#include "kernels.h"
#include "safetensors.h"

namespace orx {
namespace {

constexpr int kD = 512, kHeads = 8, kDk = 64, kDff = 2048, kKc = 9, kCh = 256, kMel = 128;
constexpr int kDD = 192, kDHeads = 8, kDDk = 24, kDDff = 768, kSpk = 4;
constexpr int kF0 = 64, kF1 = 32, kF2 = 16;  // frequency bins after each stride-2 stage
constexpr float kEps = 1e-5f;
constexpr float kMaskScore = -1e30f;         // the reference's masked score

int conv_len(int x) { return (x + 2 - 3) / 2 + 1; }
int grid_for(long long n, int threads = 256) {
  const long long b = (n + threads - 1) / threads;
  return static_cast<int>(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

__device__ __forceinline__ void put_split(uint16_t* row, int K, int k, float v) {
  const uint16_t hi = f2bf(v);
  row[k] = hi;
  row[K + k] = hi;
  row[2 * K + k] = f2bf(v - bf2f(hi));
}

// x [M, K] fp32 -> [M, 3K] split bf16, optionally ReLU'd, scaled, or with rows
// >= valid zeroed.
__global__ void __launch_bounds__(256) sf_split_kernel(const float* __restrict__ x,
                                                       uint16_t* __restrict__ out, long long M,
                                                       int K, int relu, int valid) {
  const long long n = M * K;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / K;
    const int k = static_cast<int>(i - r * K);
    float v = x[i];
    if (relu) v = fmaxf(v, 0.f);
    if (r >= valid) v = 0.f;
    put_split(out + r * 3 * K, K, k, v);
  }
}

// LayerNorm of rows of D (<= 512) fp32, one warp per row (two-pass mean and
// variance); writes fp32 (out_f32, may alias x) and / or the split form.
__global__ void __launch_bounds__(256) sf_layernorm_kernel(const float* x, const float* __restrict__ g,
                                                           const float* __restrict__ b,
                                                           float* out_f32, uint16_t* out_split,
                                                           int M, int D) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r >= M) return;
  const float* xr = x + (long long)r * D;
  float v[16];
  const int per = D / 32;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (i < per) {
      v[i] = xr[lane + 32 * i];
      s += v[i];
    }
  const float mean = warp_sum(s) / D;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (i < per) {
      const float t = v[i] - mean;
      ss += t * t;
    }
  const float inv = rsqrtf(warp_sum(ss) / D + kEps);
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (i < per) {
      const int d = lane + 32 * i;
      const float y = (v[i] - mean) * inv * g[d] + b[d];
      if (out_f32) out_f32[(long long)r * D + d] = y;
      if (out_split) put_split(out_split + (long long)r * 3 * D, D, d, y);
    }
}

__global__ void sf_scale_kernel(const float* __restrict__ x, float* __restrict__ y, long long n,
                                float s) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    y[i] = x[i] * s;
}

__global__ void sf_mask_rows_kernel(float* x, int T, int D, int valid) {
  const long long n = (long long)T * D;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    if (i / D >= valid) x[i] = 0.f;
}

// ---- pre-encode ----------------------------------------------------------
// conv 1 -> 256, 3x3, stride 2, pad 1 over the time-major mel (frames >= valid
// read as zero) + bias, ReLU, rows >= valid0 zeroed. One CTA per output time
// row; output channel-last [H0][64][256].
__global__ void __launch_bounds__(256) sf_conv0_kernel(const float* __restrict__ mel, int n_frames,
                                                       int valid, const float* __restrict__ w,
                                                       const float* __restrict__ b, int valid0,
                                                       float* __restrict__ out) {
  __shared__ float xs[3][kMel + 2];
  __shared__ float ws[kCh * 9];
  __shared__ float bs[kCh];
  const int h = blockIdx.x;
  for (int i = threadIdx.x; i < kCh * 9; i += blockDim.x) ws[i] = w[i];
  for (int i = threadIdx.x; i < kCh; i += blockDim.x) bs[i] = b[i];
  for (int i = threadIdx.x; i < 3 * (kMel + 2); i += blockDim.x) {
    const int ky = i / (kMel + 2), f = i - ky * (kMel + 2) - 1;
    const int t = 2 * h - 1 + ky;
    float v = 0.f;
    if (t >= 0 && t < n_frames && t < valid && f >= 0 && f < kMel) v = mel[(long long)f * n_frames + t];
    xs[ky][f + 1] = v;
  }
  __syncthreads();
  float* o = out + (long long)h * kF0 * kCh;
  for (int idx = threadIdx.x; idx < kF0 * kCh; idx += blockDim.x) {
    const int wo = idx / kCh, c = idx - wo * kCh;
    float acc = bs[c];
#pragma unroll
    for (int ky = 0; ky < 3; ++ky)
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) acc += xs[ky][2 * wo + kx] * ws[c * 9 + ky * 3 + kx];
    o[idx] = h < valid0 ? fmaxf(acc, 0.f) : 0.f;
  }
}

// Depthwise 3x3 stride-2 pad-1 conv + bias over channel-last [Hi][Wi][256]
// (input time rows >= in_valid read as zero) -> split bf16 [Ho * Wo][3 * 256].
__global__ void __launch_bounds__(256) sf_dwconv_kernel(const float* __restrict__ in, int Hi, int Wi,
                                                        int in_valid, const float* __restrict__ w,
                                                        const float* __restrict__ b, int Ho, int Wo,
                                                        uint16_t* __restrict__ out) {
  const long long n = (long long)Ho * Wo * kCh;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = static_cast<int>(i % kCh);
    const long long r = i / kCh;
    const int wo = static_cast<int>(r % Wo), ho = static_cast<int>(r / Wo);
    float acc = b[c];
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
      const int hi = 2 * ho - 1 + ky;
      if (hi < 0 || hi >= Hi || hi >= in_valid) continue;
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const int wi = 2 * wo - 1 + kx;
        if (wi < 0 || wi >= Wi) continue;
        acc += in[((long long)hi * Wi + wi) * kCh + c] * w[c * 9 + ky * 3 + kx];
      }
    }
    put_split(out + r * 3 * kCh, kCh, c, acc);
  }
}

// ---- conformer attention with relative positions --------------------------
// score(i, j) = ((q_i + u) . k_j + (q_i + v) . p_{T-1-i+j}) / 8, keys >= valid
// at -1e30 (RelShiftScoresKernel + AttnSoftmaxKernel of the reference).
// qkv: [T][1536] fp32 (q | k | v), p: [2T-1][512] fp32. Output: split bf16
// [T][3 * 512] (input of linear_out).
// On tensor cores: a CTA serves one head and 64 query rows (4 warps x 16);
// keys stream in blocks of 64 with the 128 position rows that block needs.
// Per warp and block: AC = (Q + u) K^T and the 16 x 80 matrix (Q + v) P^T
// over the warp's position rows, staged in shared memory and read back along
// the shifted diagonal r = T-1-i+j (the rel_shift); then online softmax and
// O += P V. Every fp32 operand is split into bf16 high + remainder parts and
// each product uses three mma.sync m16n8k16 (ah.bh + ah.bl + al.bh:
// fp32-grade, error about 2^-16 relative).
constexpr int kRtRows = 64, kRtKeys = 64, kRtPos = 128, kRtLd = kDk + 8, kRtBd = 81;
struct RtSmem {
  uint16_t kh[kRtKeys][kRtLd], kl[kRtKeys][kRtLd];
  uint16_t vh[kDk][kRtLd], vl[kDk][kRtLd];  // V transposed: [dim][key]
  uint16_t ph[kRtPos][kRtLd], pl[kRtPos][kRtLd];
  float bd[4][16][kRtBd];
};

__device__ __forceinline__ void rt_split(float x, uint16_t& hi, uint16_t& lo) {
  hi = f2bf(x);
  lo = f2bf(x - bf2f(hi));
}
__device__ __forceinline__ uint32_t rt_pack(uint16_t a, uint16_t b) {
  return static_cast<uint32_t>(a) | (static_cast<uint32_t>(b) << 16);
}

__global__ void __launch_bounds__(128) sf_relattn_tc_kernel(const float* __restrict__ qkv,
                                                           const float* __restrict__ p,
                                                           const float* __restrict__ bu,
                                                           const float* __restrict__ bv, int T,
                                                           int valid, uint16_t* __restrict__ out,
                                                           float* __restrict__ part,
                                                           int* __restrict__ tick) {
  extern __shared__ __align__(16) uint8_t rt_raw[];
  __shared__ int rt_last;
  RtSmem& sm = *reinterpret_cast<RtSmem*>(rt_raw);
  const int h = blockIdx.y, i0 = blockIdx.x * kRtRows;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int iw = i0 + warp * 16;
  const bool wactive = iw < T;
  const float scale = 0.125f;  // 1 / sqrt(64)
  // A fragments of (q + u) and (q + v), high and low parts, 4 k-steps
  uint32_t uh[4][4], ul[4][4], vh[4][4], vl[4][4];
  {
    const int ra = iw + g, rb = iw + g + 8;
    const float* qa = qkv + (long long)ra * 3 * kD + h * kDk;
    const float* qb = qkv + (long long)rb * 3 * kD + h * kDk;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const int c = ks * 16 + 2 * tq;
      const int cols[4] = {c, c, c + 8, c + 8};
      float f[8];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const bool row_b = r & 1;
        const bool ok = (row_b ? rb : ra) < T;
        const float* q = row_b ? qb : qa;
        f[2 * r] = ok ? q[cols[r]] : 0.f;
        f[2 * r + 1] = ok ? q[cols[r] + 1] : 0.f;
      }
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        uint16_t h0, l0, h1, l1;
        const float bu0 = bu[h * kDk + cols[r]], bu1 = bu[h * kDk + cols[r] + 1];
        const float bv0 = bv[h * kDk + cols[r]], bv1 = bv[h * kDk + cols[r] + 1];
        rt_split(f[2 * r] + bu0, h0, l0);
        rt_split(f[2 * r + 1] + bu1, h1, l1);
        uh[ks][r] = rt_pack(h0, h1);
        ul[ks][r] = rt_pack(l0, l1);
        rt_split(f[2 * r] + bv0, h0, l0);
        rt_split(f[2 * r + 1] + bv1, h1, l1);
        vh[ks][r] = rt_pack(h0, h1);
        vl[ks][r] = rt_pack(l0, l1);
      }
    }
  }
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const int rw0 = 48 - 16 * warp;  // first position row of this warp within the staged rows
  // key blocks of this CTA: gridDim.z CTAs split the blocks of a query tile
  const int nb = (T + kRtKeys - 1) / kRtKeys, KS = gridDim.z, kz = blockIdx.z;
  const int jb0 = (kz * nb / KS) * kRtKeys, jb1 = min(T, ((kz + 1) * nb / KS) * kRtKeys);
  for (int j0 = jb0; j0 < jb1; j0 += kRtKeys) {
    __syncthreads();
    // stage K, V (transposed) and the block's position rows as bf16 high /
    // low parts; every load of the block is issued before the first store
    {
      constexpr int kKv4 = kRtKeys * (kDk / 4) / 128, kP4 = kRtPos * (kDk / 4) / 128;
      float4 rk[kKv4], rv[kKv4], rp[kP4];
      const int mbase = T - 1 - (i0 + kRtRows - 1) + j0;  // position row of (i0 + 63, j0)
#pragma unroll
      for (int e = 0; e < kKv4; ++e) {
        const int idx = threadIdx.x + e * 128, jj = idx >> 4, d4 = idx & 15, j = j0 + jj;
        rk[e] = rv[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < T) {
          const float4* base = reinterpret_cast<const float4*>(qkv + (long long)j * 3 * kD + h * kDk);
          rk[e] = base[kD / 4 + d4];
          rv[e] = base[2 * kD / 4 + d4];
        }
      }
#pragma unroll
      for (int e = 0; e < kP4; ++e) {
        const int idx = threadIdx.x + e * 128, rr = idx >> 4, d4 = idx & 15, mrow = mbase + rr;
        rp[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (mrow >= 0 && mrow < 2 * T - 1)
          rp[e] = reinterpret_cast<const float4*>(p + (long long)mrow * kD + h * kDk)[d4];
      }
#pragma unroll
      for (int e = 0; e < kKv4; ++e) {
        const int idx = threadIdx.x + e * 128, jj = idx >> 4, d = (idx & 15) * 4;
        const float kf[4] = {rk[e].x, rk[e].y, rk[e].z, rk[e].w};
        const float vf[4] = {rv[e].x, rv[e].y, rv[e].z, rv[e].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint16_t hi, lo;
          rt_split(kf[q], hi, lo);
          sm.kh[jj][d + q] = hi;
          sm.kl[jj][d + q] = lo;
          rt_split(vf[q], hi, lo);
          sm.vh[d + q][jj] = hi;
          sm.vl[d + q][jj] = lo;
        }
      }
#pragma unroll
      for (int e = 0; e < kP4; ++e) {
        const int idx = threadIdx.x + e * 128, rr = idx >> 4, d = (idx & 15) * 4;
        const float pf[4] = {rp[e].x, rp[e].y, rp[e].z, rp[e].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint16_t hi, lo;
          rt_split(pf[q], hi, lo);
          sm.ph[rr][d + q] = hi;
          sm.pl[rr][d + q] = lo;
        }
      }
    }
    __syncthreads();
    if (!wactive) continue;
    float sc[8][4];
    // AC = (q + u) K^T
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      const int key = nt * 8 + g;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int c = ks * 16 + 2 * tq;
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&sm.kh[key][c]);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&sm.kh[key][c + 8]);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&sm.kl[key][c]);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&sm.kl[key][c + 8]);
        mma_bf16(sc[nt], ul[ks][0], ul[ks][1], ul[ks][2], ul[ks][3], bh0, bh1);
        mma_bf16(sc[nt], uh[ks][0], uh[ks][1], uh[ks][2], uh[ks][3], bl0, bl1);
        mma_bf16(sc[nt], uh[ks][0], uh[ks][1], uh[ks][2], uh[ks][3], bh0, bh1);
      }
    }
    // (q + v) P^T over the warp's 80 position rows -> shared memory
#pragma unroll
    for (int nt = 0; nt < 10; ++nt) {
      float bd[4] = {0.f, 0.f, 0.f, 0.f};
      const int pr = rw0 + nt * 8 + g;  // < 128
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int c = ks * 16 + 2 * tq;
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&sm.ph[pr][c]);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&sm.ph[pr][c + 8]);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&sm.pl[pr][c]);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&sm.pl[pr][c + 8]);
        mma_bf16(bd, vl[ks][0], vl[ks][1], vl[ks][2], vl[ks][3], bh0, bh1);
        mma_bf16(bd, vh[ks][0], vh[ks][1], vh[ks][2], vh[ks][3], bl0, bl1);
        mma_bf16(bd, vh[ks][0], vh[ks][1], vh[ks][2], vh[ks][3], bh0, bh1);
      }
      const int col = nt * 8 + 2 * tq;
      sm.bd[warp][g][col] = bd[0];
      sm.bd[warp][g][col + 1] = bd[1];
      sm.bd[warp][g + 8][col] = bd[2];
      sm.bd[warp][g + 8][col + 1] = bd[3];
    }
    __syncwarp();
    // scores: BD of (row, key) sits at column 15 - row + key
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int kl = nt * 8 + 2 * tq + e, j = j0 + kl;
        const float b0 = sm.bd[warp][g][15 - g + kl];
        const float b1 = sm.bd[warp][g + 8][7 - g + kl];
        float s0 = j < valid ? (sc[nt][e] + b0) * scale : kMaskScore;
        float s1 = j < valid ? (sc[nt][2 + e] + b1) * scale : kMaskScore;
        if (j >= T) s0 = s1 = -INFINITY;
        sc[nt][e] = s0;
        sc[nt][2 + e] = s1;
        mx0 = fmaxf(mx0, s0);
        mx1 = fmaxf(mx1, s1);
      }
    }
    __syncwarp();  // bd is rewritten by the next block
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = expf(m0 - mn0), c1 = expf(m1 - mn1);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sc[nt][e] = sc[nt][e] == -INFINITY ? 0.f : expf(sc[nt][e] - mn0);
        sc[nt][2 + e] = sc[nt][2 + e] == -INFINITY ? 0.f : expf(sc[nt][2 + e] - mn1);
        s0 += sc[nt][e];
        s1 += sc[nt][2 + e];
      }
    }
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    l0 = l0 * c0 + s0;
    l1 = l1 * c1 + s1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= c0; o[i][1] *= c0;
      o[i][2] *= c1; o[i][3] *= c1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint16_t ph[8], pl[8];
      const float pv[8] = {sc[2 * kk][0], sc[2 * kk][1], sc[2 * kk][2], sc[2 * kk][3],
                           sc[2 * kk + 1][0], sc[2 * kk + 1][1], sc[2 * kk + 1][2], sc[2 * kk + 1][3]};
#pragma unroll
      for (int i = 0; i < 8; ++i) rt_split(pv[i], ph[i], pl[i]);
      const uint32_t ah0 = rt_pack(ph[0], ph[1]), ah1 = rt_pack(ph[2], ph[3]);
      const uint32_t ah2 = rt_pack(ph[4], ph[5]), ah3 = rt_pack(ph[6], ph[7]);
      const uint32_t al0 = rt_pack(pl[0], pl[1]), al1 = rt_pack(pl[2], pl[3]);
      const uint32_t al2 = rt_pack(pl[4], pl[5]), al3 = rt_pack(pl[6], pl[7]);
      const int c = kk * 16 + 2 * tq;
#pragma unroll
      for (int nd = 0; nd < 8; ++nd) {
        const int dim = nd * 8 + g;
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&sm.vh[dim][c]);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&sm.vh[dim][c + 8]);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&sm.vl[dim][c]);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&sm.vl[dim][c + 8]);
        mma_bf16(o[nd], al0, al1, al2, al3, bh0, bh1);
        mma_bf16(o[nd], ah0, ah1, ah2, ah3, bl0, bl1);
        mma_bf16(o[nd], ah0, ah1, ah2, ah3, bh0, bh1);
      }
    }
  }
  if (KS > 1) {
    // Publish this CTA's (m, l, unnormalised o) in fragment order; the CTA
    // that arrives last for the (tile, head) merges all key ranges in order
    // (the same sums whichever CTA is last).
    const int slot = blockIdx.y * gridDim.x + blockIdx.x;
    float* mine = part + (((long long)slot * KS + kz) * 128 + threadIdx.x) * 36;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd)
#pragma unroll
      for (int e = 0; e < 4; ++e) mine[nd * 4 + e] = o[nd][e];
    mine[32] = m0; mine[33] = m1; mine[34] = l0; mine[35] = l1;
    __syncthreads();
    if (threadIdx.x == 0) {
      int tk;
      asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(tk) : "l"(tick + slot) : "memory");
      rt_last = tk == KS - 1;
      if (tk == KS - 1) tick[slot] = 0;  // ready for the next launch
    }
    __syncthreads();
    if (!rt_last) return;
    float M0 = -INFINITY, M1 = -INFINITY;
    for (int z = 0; z < KS; ++z) {
      const float* pz = part + (((long long)slot * KS + z) * 128 + threadIdx.x) * 36;
      M0 = fmaxf(M0, __ldcg(pz + 32));
      M1 = fmaxf(M1, __ldcg(pz + 33));
    }
    float L0 = 0.f, L1 = 0.f;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.f;
    for (int z = 0; z < KS; ++z) {
      const float* pz = part + (((long long)slot * KS + z) * 128 + threadIdx.x) * 36;
      const float mz0 = __ldcg(pz + 32), mz1 = __ldcg(pz + 33);
      const float w0 = mz0 == -INFINITY ? 0.f : expf(mz0 - M0);
      const float w1 = mz1 == -INFINITY ? 0.f : expf(mz1 - M1);
      L0 += __ldcg(pz + 34) * w0;
      L1 += __ldcg(pz + 35) * w1;
#pragma unroll
      for (int nd = 0; nd < 8; ++nd) {
        o[nd][0] += __ldcg(pz + nd * 4 + 0) * w0;
        o[nd][1] += __ldcg(pz + nd * 4 + 1) * w0;
        o[nd][2] += __ldcg(pz + nd * 4 + 2) * w1;
        o[nd][3] += __ldcg(pz + nd * 4 + 3) * w1;
      }
    }
    l0 = L0;
    l1 = L1;
  }
  if (!wactive) return;
  const float i0f = 1.0f / l0, i1f = 1.0f / l1;
  const int ra = iw + g, rb = iw + g + 8;
#pragma unroll
  for (int nd = 0; nd < 8; ++nd) {
    const int col = h * kDk + nd * 8 + 2 * tq;
    if (ra < T) {
      uint16_t* orow = out + (long long)ra * 3 * kD;
      put_split(orow, kD, col, o[nd][0] * i0f);
      put_split(orow, kD, col + 1, o[nd][1] * i0f);
    }
    if (rb < T) {
      uint16_t* orow = out + (long long)rb * 3 * kD;
      put_split(orow, kD, col, o[nd][2] * i1f);
      put_split(orow, kD, col + 1, o[nd][3] * i1f);
    }
  }
}

// Decoder attention (8 heads of 24): score(i, j) = q_i . k_j / sqrt(24), keys
// >= valid at -1e30; qkv [T][576] fp32, output split bf16 [T][3 * 192]. On
// tensor cores with dims padded to 32 for the k16 steps; 64 query rows per CTA
// (4 warps x 16), keys in blocks of 64, split-bf16 products (fp32-grade)
// and online softmax, as in sf_relattn_tc_kernel.
constexpr int kDtLdK = 40, kDtLdV = 72;
__global__ void __launch_bounds__(128) sf_dattn_tc_kernel(const float* __restrict__ qkv, int T,
                                                         int valid, uint16_t* __restrict__ out) {
  __shared__ __align__(16) uint16_t kh[64][kDtLdK], kl[64][kDtLdK];
  __shared__ __align__(16) uint16_t vh[kDDk][kDtLdV], vl[kDDk][kDtLdV];  // V transposed
  const int h = blockIdx.y, i0 = blockIdx.x * 64;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int iw = i0 + warp * 16;
  const bool wactive = iw < T;
  const float scale = 1.0f / sqrtf(static_cast<float>(kDDk));
  for (int idx = threadIdx.x; idx < 64 * 8; idx += 128) {  // zero the pad dims 24..31 once
    kh[idx >> 3][kDDk + (idx & 7)] = 0;
    kl[idx >> 3][kDDk + (idx & 7)] = 0;
  }
  uint32_t qh[2][4], ql[2][4];
  {
    const int ra = iw + g, rb = iw + g + 8;
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
      const int c = ks * 16 + 2 * tq;
      const int cols[4] = {c, c, c + 8, c + 8};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = (r & 1) ? rb : ra;
        float f0 = 0.f, f1 = 0.f;
        if (row < T && cols[r] < kDDk) {
          const float* q = qkv + (long long)row * 3 * kDD + h * kDDk + cols[r];
          f0 = q[0];
          f1 = q[1];
        }
        uint16_t h0, l0, h1, l1;
        rt_split(f0, h0, l0);
        rt_split(f1, h1, l1);
        qh[ks][r] = rt_pack(h0, h1);
        ql[ks][r] = rt_pack(l0, l1);
      }
    }
  }
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float o[3][4];
#pragma unroll
  for (int i = 0; i < 3; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  for (int j0 = 0; j0 < T; j0 += 64) {
    __syncthreads();
    {
      constexpr int kN = 64 * (kDDk / 4) / 128;  // float4 of K (and V) per thread
      float4 rk[kN], rv[kN];
#pragma unroll
      for (int e = 0; e < kN; ++e) {
        const int idx = threadIdx.x + e * 128, jj = idx / (kDDk / 4), d4 = idx % (kDDk / 4), j = j0 + jj;
        rk[e] = rv[e] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < T) {
          const float4* base = reinterpret_cast<const float4*>(qkv + (long long)j * 3 * kDD + h * kDDk);
          rk[e] = base[kDD / 4 + d4];
          rv[e] = base[2 * kDD / 4 + d4];
        }
      }
#pragma unroll
      for (int e = 0; e < kN; ++e) {
        const int idx = threadIdx.x + e * 128, jj = idx / (kDDk / 4), d = (idx % (kDDk / 4)) * 4;
        const float kf[4] = {rk[e].x, rk[e].y, rk[e].z, rk[e].w};
        const float vf[4] = {rv[e].x, rv[e].y, rv[e].z, rv[e].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint16_t hi, lo;
          rt_split(kf[q], hi, lo);
          kh[jj][d + q] = hi;
          kl[jj][d + q] = lo;
          rt_split(vf[q], hi, lo);
          vh[d + q][jj] = hi;
          vl[d + q][jj] = lo;
        }
      }
    }
    __syncthreads();
    if (!wactive) continue;
    float sc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
      const int key = nt * 8 + g;
#pragma unroll
      for (int ks = 0; ks < 2; ++ks) {
        const int c = ks * 16 + 2 * tq;
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&kh[key][c]);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&kh[key][c + 8]);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&kl[key][c]);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&kl[key][c + 8]);
        mma_bf16(sc[nt], ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3], bh0, bh1);
        mma_bf16(sc[nt], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], bl0, bl1);
        mma_bf16(sc[nt], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], bh0, bh1);
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = j0 + nt * 8 + 2 * tq + e;
        float s0 = j < valid ? sc[nt][e] * scale : kMaskScore;
        float s1 = j < valid ? sc[nt][2 + e] * scale : kMaskScore;
        if (j >= T) s0 = s1 = -INFINITY;
        sc[nt][e] = s0;
        sc[nt][2 + e] = s1;
        mx0 = fmaxf(mx0, s0);
        mx1 = fmaxf(mx1, s1);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = expf(m0 - mn0), c1 = expf(m1 - mn1);
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        sc[nt][e] = sc[nt][e] == -INFINITY ? 0.f : expf(sc[nt][e] - mn0);
        sc[nt][2 + e] = sc[nt][2 + e] == -INFINITY ? 0.f : expf(sc[nt][2 + e] - mn1);
        s0 += sc[nt][e];
        s1 += sc[nt][2 + e];
      }
    }
    s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
    s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
    s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
    l0 = l0 * c0 + s0;
    l1 = l1 * c1 + s1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      o[i][0] *= c0; o[i][1] *= c0;
      o[i][2] *= c1; o[i][3] *= c1;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint16_t ph[8], pl[8];
      const float pv[8] = {sc[2 * kk][0], sc[2 * kk][1], sc[2 * kk][2], sc[2 * kk][3],
                           sc[2 * kk + 1][0], sc[2 * kk + 1][1], sc[2 * kk + 1][2], sc[2 * kk + 1][3]};
#pragma unroll
      for (int i = 0; i < 8; ++i) rt_split(pv[i], ph[i], pl[i]);
      const uint32_t ah0 = rt_pack(ph[0], ph[1]), ah1 = rt_pack(ph[2], ph[3]);
      const uint32_t ah2 = rt_pack(ph[4], ph[5]), ah3 = rt_pack(ph[6], ph[7]);
      const uint32_t al0 = rt_pack(pl[0], pl[1]), al1 = rt_pack(pl[2], pl[3]);
      const uint32_t al2 = rt_pack(pl[4], pl[5]), al3 = rt_pack(pl[6], pl[7]);
      const int c = kk * 16 + 2 * tq;
#pragma unroll
      for (int nd = 0; nd < 3; ++nd) {
        const int dim = nd * 8 + g;
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(&vh[dim][c]);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(&vh[dim][c + 8]);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(&vl[dim][c]);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(&vl[dim][c + 8]);
        mma_bf16(o[nd], al0, al1, al2, al3, bh0, bh1);
        mma_bf16(o[nd], ah0, ah1, ah2, ah3, bl0, bl1);
        mma_bf16(o[nd], ah0, ah1, ah2, ah3, bh0, bh1);
      }
    }
  }
  if (!wactive) return;
  const int ra = iw + g, rb = iw + g + 8;
#pragma unroll
  for (int nd = 0; nd < 3; ++nd) {
    const int col = h * kDDk + nd * 8 + 2 * tq;
    if (ra < T) {
      uint16_t* orow = out + (long long)ra * 3 * kDD;
      put_split(orow, kDD, col, o[nd][0] / l0);
      put_split(orow, kDD, col + 1, o[nd][1] / l0);
    }
    if (rb < T) {
      uint16_t* orow = out + (long long)rb * 3 * kDD;
      put_split(orow, kDD, col, o[nd][2] / l1);
      put_split(orow, kDD, col + 1, o[nd][3] / l1);
    }
  }
}


// Conv module middle: GLU of pointwise_conv1's output (rows >= valid zero),
// depthwise conv k9 (zero padding) + bias, BatchNorm (running statistics),
// SiLU -> split bf16 [T][3 * 512] (input of pointwise_conv2).
__global__ void __launch_bounds__(256) sf_convmod_kernel(const float* __restrict__ pw1, int T,
                                                         int valid, const float* __restrict__ dw,
                                                         const float* __restrict__ dwb,
                                                         const float* __restrict__ mean,
                                                         const float* __restrict__ var,
                                                         const float* __restrict__ gamma,
                                                         const float* __restrict__ beta,
                                                         uint16_t* __restrict__ out) {
  const long long n = (long long)T * kD;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = static_cast<int>(i % kD), t = static_cast<int>(i / kD);
    float acc = dwb[c];
#pragma unroll
    for (int kk = 0; kk < kKc; ++kk) {
      const int ti = t + kk - kKc / 2;
      if (ti < 0 || ti >= T || ti >= valid) continue;
      const float a = pw1[(long long)ti * 2 * kD + c], g = pw1[(long long)ti * 2 * kD + kD + c];
      acc += a * (1.0f / (1.0f + expf(-g))) * dw[c * kKc + kk];
    }
    const float y = (acc - mean[c]) * rsqrtf(var[c] + kEps) * gamma[c] + beta[c];
    put_split(out + (long long)t * 3 * kD, kD, c, y / (1.0f + expf(-y)));
  }
}

// Weight row of a Linear in split form: W3[n] = [Wh | Wl | Wh] of W[n]
// (columns permuted from c * F + f to f * C + c when C > 0).
__global__ void sf_make_w3_kernel(const float* __restrict__ W, uint16_t* __restrict__ W3, int N,
                                  int K, int C, int F) {
  const long long n = (long long)N * K;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / K;
    const int k = static_cast<int>(i - r * K);
    int src = k;
    if (C > 0) {
      const int f = k / C, c = k - f * C;
      src = c * F + f;
    }
    const float v = W[r * K + src];
    const uint16_t hi = f2bf(v);
    uint16_t* row = W3 + r * 3 * K;
    row[k] = hi;
    row[K + k] = f2bf(v - bf2f(hi));
    row[2 * K + k] = hi;
  }
}

}  // namespace

struct Sortformer::Impl {
  int L = 0, DL = 0;
  int* err = nullptr;
  // One entry per checkpoint tensor.
  enum Kind { kVec, kLin, kLinPerm };
  struct Entry {
    std::string name;
    Kind kind;
    void* dst;      // fp32 vector, or the W3 block (row offset applied)
    size_t numel;
    int N, K;       // Linear shape
    int tkind;      // synthetic init: 0 matrix, 1 bias, 2 gain, 3 BN variance
    size_t fan_in;
  };
  std::vector<Entry> entries;
  std::vector<bool> have;
  std::vector<void*> allocs;

  // pre-encode
  float *c0w, *c0b, *c2w, *c2b, *c3b, *c5w, *c5b, *c6b, *outb;
  uint16_t *c3w, *c6w, *outw;
  struct Conf {
    float *ln1g, *ln1b, *ff1b1, *ff1b2, *lnag, *lnab, *qkvb, *ob, *bu, *bv, *lncg, *lncb, *pw1b,
        *dww, *dwb, *bng, *bnb, *bnm, *bnv, *pw2b, *ln2g, *ln2b, *ff2b1, *ff2b2, *lnog, *lnob;
    uint16_t *ff1w1, *ff1w2, *qkvw, *ow, *posw, *pw1w, *pw2w, *ff2w1, *ff2w2;
  };
  std::vector<Conf> C;
  float *projb, *hidb, *spkb;
  uint16_t *projw, *hidw, *spkw;
  struct Dec {
    float *qkvb, *ob, *inb, *outb, *ln1g, *ln1b, *ln2g, *ln2b;
    uint16_t *qkvw, *ow, *inw, *outw;
  };
  std::vector<Dec> Dl;

  // scratch
  struct Buf {
    void* p = nullptr;
    size_t cap = 0;
    template <class T>
    T* get(size_t n) {
      if (n * sizeof(T) > cap) {
        ORX_CHECK(cudaDeviceSynchronize());
        if (p) cudaFree(p);
        cap = n * sizeof(T) + 4096;
        ORX_CHECK(cudaMalloc(&p, cap));
      }
      return static_cast<T*>(p);
    }
    ~Buf() {
      if (p) cudaFree(p);
    }
  };
  Buf b_a, b_b, b_s1, b_s2, b_x, b_qkv, b_p, b_pe, b_pes, b_big, b_mel, b_out, b_emb, b_ws, b_rpart, b_rtick;
  size_t rtick_n = 0;  // tickets known to be zero
  std::vector<float> pe_host;
  int pe_T = -1;

  float* F(size_t n) {
    float* p = dalloc<float>(n);
    allocs.push_back(p);
    return p;
  }
  uint16_t* B3(size_t N, size_t K) {
    uint16_t* p = dalloc<uint16_t>(N * 3 * K);
    allocs.push_back(p);
    return p;
  }
  void vec(const std::string& n, float* d, size_t numel, int tk) {
    entries.push_back({n, kVec, d, numel, 0, 0, tk, 0});
  }
  void lin(const std::string& n, uint16_t* w3, int N, int K, Kind k = kLin) {
    entries.push_back({n, k, w3, (size_t)N * K, N, K, 0, (size_t)K});
  }

  void build() {
    const std::string P = "encoder.pre_encode.";
    c0w = F(kCh * 9); c0b = F(kCh); c2w = F(kCh * 9); c2b = F(kCh); c3b = F(kCh);
    c5w = F(kCh * 9); c5b = F(kCh); c6b = F(kCh); outb = F(kD);
    c3w = B3(kCh, kCh); c6w = B3(kCh, kCh); outw = B3(kD, kCh * kF2);
    entries.push_back({P + "conv.0.weight", kVec, c0w, kCh * 9, 0, 0, 0, 9});
    vec(P + "conv.0.bias", c0b, kCh, 1);
    entries.push_back({P + "conv.2.weight", kVec, c2w, kCh * 9, 0, 0, 0, 9});
    vec(P + "conv.2.bias", c2b, kCh, 1);
    lin(P + "conv.3.weight", c3w, kCh, kCh);
    vec(P + "conv.3.bias", c3b, kCh, 1);
    entries.push_back({P + "conv.5.weight", kVec, c5w, kCh * 9, 0, 0, 0, 9});
    vec(P + "conv.5.bias", c5b, kCh, 1);
    lin(P + "conv.6.weight", c6w, kCh, kCh);
    vec(P + "conv.6.bias", c6b, kCh, 1);
    lin(P + "out.weight", outw, kD, kCh * kF2, kLinPerm);
    vec(P + "out.bias", outb, kD, 1);
    C.resize(L);
    for (int i = 0; i < L; ++i) {
      Conf& c = C[i];
      const std::string p = "encoder.layers." + std::to_string(i) + ".";
      c.ln1g = F(kD); c.ln1b = F(kD); c.ff1w1 = B3(kDff, kD); c.ff1b1 = F(kDff);
      c.ff1w2 = B3(kD, kDff); c.ff1b2 = F(kD);
      c.lnag = F(kD); c.lnab = F(kD); c.qkvw = B3(3 * kD, kD); c.qkvb = F(3 * kD);
      c.ow = B3(kD, kD); c.ob = F(kD); c.posw = B3(kD, kD); c.bu = F(kD); c.bv = F(kD);
      c.lncg = F(kD); c.lncb = F(kD); c.pw1w = B3(2 * kD, kD); c.pw1b = F(2 * kD);
      c.dww = F(kD * kKc); c.dwb = F(kD); c.bng = F(kD); c.bnb = F(kD); c.bnm = F(kD); c.bnv = F(kD);
      c.pw2w = B3(kD, kD); c.pw2b = F(kD);
      c.ln2g = F(kD); c.ln2b = F(kD); c.ff2w1 = B3(kDff, kD); c.ff2b1 = F(kDff);
      c.ff2w2 = B3(kD, kDff); c.ff2b2 = F(kD); c.lnog = F(kD); c.lnob = F(kD);
      vec(p + "norm_feed_forward1.weight", c.ln1g, kD, 2);
      vec(p + "norm_feed_forward1.bias", c.ln1b, kD, 1);
      lin(p + "feed_forward1.linear1.weight", c.ff1w1, kDff, kD);
      vec(p + "feed_forward1.linear1.bias", c.ff1b1, kDff, 1);
      lin(p + "feed_forward1.linear2.weight", c.ff1w2, kD, kDff);
      vec(p + "feed_forward1.linear2.bias", c.ff1b2, kD, 1);
      vec(p + "norm_self_att.weight", c.lnag, kD, 2);
      vec(p + "norm_self_att.bias", c.lnab, kD, 1);
      const char* qkvn[3] = {"linear_q", "linear_k", "linear_v"};
      for (int j = 0; j < 3; ++j) {
        lin(p + "self_attn." + qkvn[j] + ".weight", c.qkvw + (size_t)j * kD * 3 * kD, kD, kD);
        vec(p + "self_attn." + qkvn[j] + ".bias", c.qkvb + j * kD, kD, 1);
      }
      lin(p + "self_attn.linear_out.weight", c.ow, kD, kD);
      vec(p + "self_attn.linear_out.bias", c.ob, kD, 1);
      lin(p + "self_attn.linear_pos.weight", c.posw, kD, kD);
      vec(p + "self_attn.pos_bias_u", c.bu, kD, 1);
      vec(p + "self_attn.pos_bias_v", c.bv, kD, 1);
      vec(p + "norm_conv.weight", c.lncg, kD, 2);
      vec(p + "norm_conv.bias", c.lncb, kD, 1);
      lin(p + "conv.pointwise_conv1.weight", c.pw1w, 2 * kD, kD);
      vec(p + "conv.pointwise_conv1.bias", c.pw1b, 2 * kD, 1);
      entries.push_back({p + "conv.depthwise_conv.weight", kVec, c.dww, (size_t)kD * kKc, 0, 0, 0,
                         (size_t)kKc});
      vec(p + "conv.depthwise_conv.bias", c.dwb, kD, 1);
      vec(p + "conv.batch_norm.weight", c.bng, kD, 2);
      vec(p + "conv.batch_norm.bias", c.bnb, kD, 1);
      vec(p + "conv.batch_norm.running_mean", c.bnm, kD, 1);
      vec(p + "conv.batch_norm.running_var", c.bnv, kD, 3);
      lin(p + "conv.pointwise_conv2.weight", c.pw2w, kD, kD);
      vec(p + "conv.pointwise_conv2.bias", c.pw2b, kD, 1);
      vec(p + "norm_feed_forward2.weight", c.ln2g, kD, 2);
      vec(p + "norm_feed_forward2.bias", c.ln2b, kD, 1);
      lin(p + "feed_forward2.linear1.weight", c.ff2w1, kDff, kD);
      vec(p + "feed_forward2.linear1.bias", c.ff2b1, kDff, 1);
      lin(p + "feed_forward2.linear2.weight", c.ff2w2, kD, kDff);
      vec(p + "feed_forward2.linear2.bias", c.ff2b2, kD, 1);
      vec(p + "norm_out.weight", c.lnog, kD, 2);
      vec(p + "norm_out.bias", c.lnob, kD, 1);
    }
    const std::string S = "sortformer_modules.";
    projw = B3(kDD, kD); projb = F(kDD); hidw = B3(kDD, kDD); hidb = F(kDD);
    spkw = B3(kSpk, kDD); spkb = F(kSpk);
    lin(S + "encoder_proj.weight", projw, kDD, kD);
    vec(S + "encoder_proj.bias", projb, kDD, 1);
    lin(S + "first_hidden_to_hidden.weight", hidw, kDD, kDD);
    vec(S + "first_hidden_to_hidden.bias", hidb, kDD, 1);
    lin(S + "single_hidden_to_spks.weight", spkw, kSpk, kDD);
    vec(S + "single_hidden_to_spks.bias", spkb, kSpk, 1);
    Dl.resize(DL);
    for (int i = 0; i < DL; ++i) {
      Dec& d = Dl[i];
      const std::string p = "transformer_encoder.layers." + std::to_string(i) + ".";
      d.qkvw = B3(3 * kDD, kDD); d.qkvb = F(3 * kDD); d.ow = B3(kDD, kDD); d.ob = F(kDD);
      d.inw = B3(kDDff, kDD); d.inb = F(kDDff); d.outw = B3(kDD, kDDff); d.outb = F(kDD);
      d.ln1g = F(kDD); d.ln1b = F(kDD); d.ln2g = F(kDD); d.ln2b = F(kDD);
      const char* qkvn[3] = {"query_net", "key_net", "value_net"};
      for (int j = 0; j < 3; ++j) {
        lin(p + "first_sub_layer." + qkvn[j] + ".weight", d.qkvw + (size_t)j * kDD * 3 * kDD, kDD, kDD);
        vec(p + "first_sub_layer." + qkvn[j] + ".bias", d.qkvb + j * kDD, kDD, 1);
      }
      lin(p + "first_sub_layer.out_projection.weight", d.ow, kDD, kDD);
      vec(p + "first_sub_layer.out_projection.bias", d.ob, kDD, 1);
      lin(p + "second_sub_layer.dense_in.weight", d.inw, kDDff, kDD);
      vec(p + "second_sub_layer.dense_in.bias", d.inb, kDDff, 1);
      lin(p + "second_sub_layer.dense_out.weight", d.outw, kDD, kDDff);
      vec(p + "second_sub_layer.dense_out.bias", d.outb, kDD, 1);
      vec(p + "layer_norm_1.weight", d.ln1g, kDD, 2);
      vec(p + "layer_norm_1.bias", d.ln1b, kDD, 1);
      vec(p + "layer_norm_2.weight", d.ln2g, kDD, 2);
      vec(p + "layer_norm_2.bias", d.ln2b, kDD, 1);
    }
    have.assign(entries.size(), false);
  }

  // Linear on the split operands: out = act(X3 . W3^T + bias), X3 [M][3K].
  void gemm(const uint16_t* X3, const uint16_t* W3, int M, int K, int N, const float* bias, int act,
            float* out_f32, uint16_t* out_split, int resid, cudaStream_t s) {
    TcArgs g = {};
    g.N = N;
    g.K = 3 * K;
    g.T = M;
    g.epi = kEpiLinear;
    g.out_f32 = out_f32;
    g.out_bf16 = out_split;
    g.split3 = out_split ? 1 : 0;
    g.ldo = out_split ? 3 * N : N;
    g.err = err;
    g.bias = bias;
    g.act = act;
    g.resid = resid;
    // split K where the Linear has too few tiles to cover the SMs
    int bn = 0;
    const int splits = linear_plan(N, 3 * K, M, tc_sms(), &bn);
    g.bn_hint = bn;
    if (splits > 1) g.ws = b_ws.get<float>((size_t)splits * M * N);
    launch_gemm_tc(X3, W3, g, splits, s);
    check(cudaGetLastError(), "sortformer gemm");
  }
  void ln(const float* x, const float* g, const float* b, float* of, uint16_t* os, int M, int Dm,
          cudaStream_t s) {
    sf_layernorm_kernel<<<(M + 7) / 8, 256, 0, s>>>(x, g, b, of, os, M, Dm);
    check(cudaGetLastError(), "sortformer layernorm");
  }
};

Sortformer::Sortformer(int conf_layers, int dec_layers) : p_(new Impl) {
  if (conf_layers < 0 || conf_layers > 64 || dec_layers < 0 || dec_layers > 64)
    throw std::invalid_argument("layer counts must be in [0, 64]");
  p_->L = conf_layers;
  p_->DL = dec_layers;
  p_->err = dalloc<int>(1);
  ORX_CHECK(cudaMemset(p_->err, 0, sizeof(int)));
  ORX_CHECK(cudaFuncSetAttribute(sf_relattn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(RtSmem))));
  p_->build();
}

Sortformer::~Sortformer() {
  cudaDeviceSynchronize();
  for (void* q : p_->allocs) cudaFree(q);
  cudaFree(p_->err);
  delete p_;
}

bool Sortformer::complete() const {
  for (bool b : p_->have)
    if (!b) return false;
  return true;
}

void Sortformer::set_tensor(const std::string& name, const float* data, size_t numel, bool device) {
  Impl& p = *p_;
  for (size_t i = 0; i < p.entries.size(); ++i) {
    const auto& e = p.entries[i];
    if (e.name != name) continue;
    if (numel != e.numel)
      throw std::invalid_argument("tensor " + name + " has " + std::to_string(numel) +
                                  " elements, expected " + std::to_string(e.numel));
    const cudaMemcpyKind kind = device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    if (e.kind == Impl::kVec) {
      ORX_CHECK(cudaMemcpy(e.dst, data, numel * 4, kind));
    } else {
      float* tmp = dalloc<float>(numel);
      ORX_CHECK(cudaMemcpy(tmp, data, numel * 4, kind));
      sf_make_w3_kernel<<<grid_for((long long)numel), 256>>>(
          tmp, static_cast<uint16_t*>(e.dst), e.N, e.K, e.kind == Impl::kLinPerm ? kCh : 0, kF2);
      ORX_CHECK(cudaGetLastError());
      ORX_CHECK(cudaDeviceSynchronize());
      cudaFree(tmp);
    }
    p.have[i] = true;
    return;
  }
  throw std::invalid_argument("unknown Sortformer tensor " + name);
}

void Sortformer::load_safetensors(const std::string& path) {
  SafeTensorsFile f(path);
  for (const auto& kv : f.tensors()) {
    if (kv.second.dtype != "F32") continue;
    bool known = false;
    for (const auto& e : p_->entries)
      if (e.name == kv.first) known = true;
    if (!known) continue;  // tensors of other modules, or of layers beyond the configured counts
    set_tensor(kv.first, static_cast<const float*>(kv.second.data), kv.second.nbytes / 4, false);
  }
  if (!complete()) throw std::invalid_argument("checkpoint is missing Sortformer tensors");
}

void Sortformer::init_synthetic(int seed) {
  Impl& p = *p_;
  size_t big = 0;
  for (const auto& e : p.entries) big = std::max(big, e.numel);
  float* tmp = dalloc<float>(big);
  for (size_t i = 0; i < p.entries.size(); ++i) {
    const auto& e = p.entries[i];
    const int tid = 90000 + static_cast<int>(i);
    double sd = 0.02;
    float mean = 0.f;
    if (e.fan_in) sd = 1.0 / std::sqrt(static_cast<double>(e.fan_in));
    else if (e.tkind == 2) mean = 1.f;
    else if (e.tkind == 3) sd = 0.1;
    launch_synth_f32(tmp, (long long)e.numel, seed, tid, sd, mean, 0, 0);
    ORX_CHECK(cudaGetLastError());
    if (e.tkind == 3) {  // running variance 1 + |N(0, 0.1^2)|
      std::vector<float> h(e.numel);
      ORX_CHECK(cudaMemcpy(h.data(), tmp, e.numel * 4, cudaMemcpyDeviceToHost));
      for (auto& v : h) v = 1.0f + std::fabs(v);
      ORX_CHECK(cudaMemcpy(tmp, h.data(), e.numel * 4, cudaMemcpyHostToDevice));
    }
    set_tensor(e.name, tmp, e.numel, true);
  }
  cudaFree(tmp);
}

int Sortformer::pre_encode_device(const float* d_mel, int n_frames, int valid, float* d_out,
                                  int* valid_out, cudaStream_t s) {
  Impl& p = *p_;
  if (!complete()) throw std::invalid_argument("Sortformer weights are incomplete");
  if (n_frames <= 0) throw std::invalid_argument("n_frames must be positive");
  valid = std::max(0, std::min(valid, n_frames));
  const int H0 = conv_len(n_frames), H1 = conv_len(H0), H2 = conv_len(H1);
  const int v0 = conv_len(valid), v1 = conv_len(v0), v2 = conv_len(v1);
  float* a = p.b_a.get<float>((size_t)H0 * kF0 * kCh);
  uint16_t* sp = p.b_s1.get<uint16_t>((size_t)H1 * kF1 * 3 * kCh);
  float* b = p.b_b.get<float>((size_t)H1 * kF1 * kCh);
  sf_conv0_kernel<<<H0, 256, 0, s>>>(d_mel, n_frames, valid, p.c0w, p.c0b, v0, a);
  check(cudaGetLastError(), "sortformer conv0");
  sf_dwconv_kernel<<<grid_for((long long)H1 * kF1 * kCh), 256, 0, s>>>(a, H0, kF0, v0, p.c2w, p.c2b,
                                                                      H1, kF1, sp);
  check(cudaGetLastError(), "sortformer dwconv");
  p.gemm(sp, p.c3w, H1 * kF1, kCh, kCh, p.c3b, 2, b, nullptr, 0, s);
  sf_dwconv_kernel<<<grid_for((long long)H2 * kF2 * kCh), 256, 0, s>>>(b, H1, kF1, v1, p.c5w, p.c5b,
                                                                      H2, kF2, sp);
  check(cudaGetLastError(), "sortformer dwconv");
  p.gemm(sp, p.c6w, H2 * kF2, kCh, kCh, p.c6b, 2, a, nullptr, 0, s);  // [H2][16][256] = [H2][4096]
  uint16_t* fs = p.b_s2.get<uint16_t>((size_t)H2 * 3 * kCh * kF2);
  sf_split_kernel<<<grid_for((long long)H2 * kCh * kF2), 256, 0, s>>>(a, fs, H2, kCh * kF2, 0, v2);
  check(cudaGetLastError(), "sortformer split");
  p.gemm(fs, p.outw, H2, kCh * kF2, kD, p.outb, 0, d_out, nullptr, 0, s);
  if (valid_out) *valid_out = v2;
  return H2;
}

void Sortformer::encode_decode_device(const float* d_emb, int T, int valid, float* d_preds,
                                      cudaStream_t s) {
  Impl& p = *p_;
  if (!complete()) throw std::invalid_argument("Sortformer weights are incomplete");
  if (T <= 0) throw std::invalid_argument("T must be positive");
  valid = std::max(0, std::min(valid, T));
  const int P = 2 * T - 1;
  float* x = p.b_x.get<float>((size_t)T * kD);
  uint16_t* s1 = p.b_s1.get<uint16_t>((size_t)T * 3 * kDff);
  uint16_t* s2 = p.b_s2.get<uint16_t>((size_t)T * 3 * kDff);
  float* qkv = p.b_qkv.get<float>((size_t)T * 3 * kD);
  float* pp = p.b_p.get<float>((size_t)P * kD);
  float* big = p.b_big.get<float>((size_t)T * 2 * kD);
  // relative positional encoding (ConformerLayer::BuildPosEmb), in fp32 as
  // the reference computes it, cached per T
  if (p.pe_T != T) {
    p.pe_host.assign((size_t)P * kD, 0.f);
    for (int idx = 0; idx < P; ++idx) {
      const float pos = static_cast<float>(T - 1 - idx);
      for (int i = 0; i < kD; i += 2) {
        const float div = std::exp(-(std::log(10000.0f)) * static_cast<float>(i) / kD);
        p.pe_host[(size_t)idx * kD + i] = std::sin(pos * div);
        p.pe_host[(size_t)idx * kD + i + 1] = std::cos(pos * div);
      }
    }
    float* pe = p.b_pe.get<float>((size_t)P * kD);
    ORX_CHECK(cudaMemcpyAsync(pe, p.pe_host.data(), (size_t)P * kD * 4, cudaMemcpyHostToDevice, s));
    uint16_t* pes = p.b_pes.get<uint16_t>((size_t)P * 3 * kD);
    sf_split_kernel<<<grid_for((long long)P * kD), 256, 0, s>>>(pe, pes, P, kD, 0, P);
    check(cudaGetLastError(), "sortformer split");
    ORX_CHECK(cudaStreamSynchronize(s));  // the host table is reused next call
    p.pe_T = T;
  }
  const uint16_t* pes = static_cast<const uint16_t*>(p.b_pes.p);
  sf_scale_kernel<<<grid_for((long long)T * kD), 256, 0, s>>>(d_emb, x, (long long)T * kD,
                                                              std::sqrt(static_cast<float>(kD)));
  check(cudaGetLastError(), "sortformer scale");
  // relative-position attention: query tiles x heads x key ranges, about
  // two CTAs per SM (each holds 94 KB of shared memory)
  const int rt_tiles = (T + kRtRows - 1) / kRtRows, rt_nb = (T + kRtKeys - 1) / kRtKeys;
  const int rt_ks = std::max(1, std::min({4, rt_nb, (2 * tc_sms()) / (rt_tiles * kHeads)}));
  float* rt_part = p.b_rpart.get<float>((size_t)rt_tiles * kHeads * rt_ks * 128 * 36);
  int* rt_tick = p.b_rtick.get<int>((size_t)rt_tiles * kHeads);
  if ((size_t)rt_tiles * kHeads > p.rtick_n) {  // grown (or first use): tickets start at zero
    ORX_CHECK(cudaMemsetAsync(rt_tick, 0, p.b_rtick.cap, s));
    p.rtick_n = p.b_rtick.cap / sizeof(int);
  }
  for (int li = 0; li < p.L; ++li) {
    const Impl::Conf& c = p.C[li];
    p.ln(x, c.ln1g, c.ln1b, nullptr, s1, T, kD, s);
    p.gemm(s1, c.ff1w1, T, kD, kDff, c.ff1b1, 3, nullptr, s2, 0, s);
    p.gemm(s2, c.ff1w2, T, kDff, kD, c.ff1b2, 0, x, nullptr, 2, s);
    p.ln(x, c.lnag, c.lnab, nullptr, s1, T, kD, s);
    p.gemm(s1, c.qkvw, T, kD, 3 * kD, c.qkvb, 0, qkv, nullptr, 0, s);
    p.gemm(pes, c.posw, P, kD, kD, nullptr, 0, pp, nullptr, 0, s);
    sf_relattn_tc_kernel<<<dim3(rt_tiles, kHeads, rt_ks), 128, sizeof(RtSmem), s>>>(
        qkv, pp, c.bu, c.bv, T, valid, s2, rt_part, rt_tick);
    check(cudaGetLastError(), "sortformer attention");
    p.gemm(s2, c.ow, T, kD, kD, c.ob, 0, x, nullptr, 1, s);
    p.ln(x, c.lncg, c.lncb, nullptr, s1, T, kD, s);
    p.gemm(s1, c.pw1w, T, kD, 2 * kD, c.pw1b, 0, big, nullptr, 0, s);
    sf_convmod_kernel<<<grid_for((long long)T * kD), 256, 0, s>>>(big, T, valid, c.dww, c.dwb, c.bnm,
                                                                  c.bnv, c.bng, c.bnb, s2);
    check(cudaGetLastError(), "sortformer conv module");
    p.gemm(s2, c.pw2w, T, kD, kD, c.pw2b, 0, x, nullptr, 1, s);
    p.ln(x, c.ln2g, c.ln2b, nullptr, s1, T, kD, s);
    p.gemm(s1, c.ff2w1, T, kD, kDff, c.ff2b1, 3, nullptr, s2, 0, s);
    p.gemm(s2, c.ff2w2, T, kDff, kD, c.ff2b2, 0, x, nullptr, 2, s);
    p.ln(x, c.lnog, c.lnob, x, nullptr, T, kD, s);
  }
  // ---- decoder ----
  float* xd = big;  // [T][192]
  sf_split_kernel<<<grid_for((long long)T * kD), 256, 0, s>>>(x, s1, T, kD, 0, T);
  check(cudaGetLastError(), "sortformer split");
  p.gemm(s1, p.projw, T, kD, kDD, p.projb, 0, xd, nullptr, 0, s);
  sf_split_kernel<<<grid_for((long long)T * kDD), 256, 0, s>>>(xd, s1, T, kDD, 0, T);
  check(cudaGetLastError(), "sortformer split");
  for (int li = 0; li < p.DL; ++li) {
    const Impl::Dec& d = p.Dl[li];
    p.gemm(s1, d.qkvw, T, kDD, 3 * kDD, d.qkvb, 0, qkv, nullptr, 0, s);
    sf_dattn_tc_kernel<<<dim3((T + 63) / 64, kDHeads), 128, 0, s>>>(qkv, T, valid, s2);
    check(cudaGetLastError(), "sortformer decoder attention");
    p.gemm(s2, d.ow, T, kDD, kDD, d.ob, 0, xd, nullptr, 1, s);
    p.ln(xd, d.ln1g, d.ln1b, xd, s1, T, kDD, s);
    p.gemm(s1, d.inw, T, kDD, kDDff, d.inb, 2, nullptr, s2, 0, s);
    p.gemm(s2, d.outw, T, kDDff, kDD, d.outb, 0, xd, nullptr, 1, s);
    p.ln(xd, d.ln2g, d.ln2b, xd, s1, T, kDD, s);
  }
  sf_split_kernel<<<grid_for((long long)T * kDD), 256, 0, s>>>(xd, s1, T, kDD, 1, T);
  check(cudaGetLastError(), "sortformer split");
  p.gemm(s1, p.hidw, T, kDD, kDD, p.hidb, 2, nullptr, s2, 0, s);
  p.gemm(s2, p.spkw, T, kDD, kSpk, p.spkb, 4, d_preds, nullptr, 0, s);
  sf_mask_rows_kernel<<<grid_for((long long)T * kSpk), 256, 0, s>>>(d_preds, T, kSpk, valid);
  check(cudaGetLastError(), "sortformer mask");
}

int Sortformer::step_device(const float* d_mel, int n_frames, int valid, const float* d_cache,
                            int n_cache, float* d_preds, int* valid_out, cudaStream_t s) {
  Impl& p = *p_;
  if (n_cache < 0) throw std::invalid_argument("cache rows must be >= 0");
  const int H2 = conv_len(conv_len(conv_len(n_frames)));
  float* emb = p.b_emb.get<float>((size_t)(n_cache + H2) * kD);
  if (n_cache > 0)
    ORX_CHECK(cudaMemcpyAsync(emb, d_cache, (size_t)n_cache * kD * 4, cudaMemcpyDeviceToDevice, s));
  int v2 = 0;
  pre_encode_device(d_mel, n_frames, valid, emb + (size_t)n_cache * kD, &v2, s);
  const int T = n_cache + H2, vcat = n_cache + v2;
  encode_decode_device(emb, T, vcat, d_preds, s);
  if (valid_out) *valid_out = vcat;
  return T;
}

int Sortformer::device_error() const {
  int e = 0;
  ORX_CHECK(cudaMemcpy(&e, p_->err, sizeof(int), cudaMemcpyDeviceToHost));
  return e;
}

}  // namespace orx
