// Paged GQA attention for decode and prefill (flash-decoding split over pages).
//
// Replaces GqaDecodeAttnKernel / GqaCacheAttnKernel / WriteKvCacheKernel and
// the per-head RmsNorm + RopeHalf launches of the reference
// (src/model/asr_text_decoder.cu:62-213,404-418; src/model/asr_ops.cu:92-111).
// Differences by design: the cache is paged (16 tokens per page, one page
// table per session) instead of one contiguous [max_seq, 8, 128] buffer, there
// is no 2048-position cap, and one CTA serves both query heads of a GQA group
// so each K/V page is read once per group.  Math is the reference's: fp32 q,
// bf16 K/V, scores scaled by 1/sqrt(128), exp-normalised in fp32, output
// rounded to bf16 (the cast the reference does before o_proj).
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace orx {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kPartStride = 2 * 132;  // per split: 2 heads x (128 acc, m, l, pad)
constexpr int kMaxSplits = 64;       // nsplit_max limit (2 * kMaxSplits <= 128 threads)

__device__ __forceinline__ float block_sum128(float v, float* red, int t) {
  v = warp_sum(v);
  __syncthreads();
  if ((t & 31) == 0) red[t >> 5] = v;
  __syncthreads();
  return red[0] + red[1] + red[2] + red[3];
}

__global__ void __launch_bounds__(kAttnThreads) attn_kernel(AttnArgs a) {
  const int split = blockIdx.x, h = blockIdx.y, row = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  pdl_trigger();
  pdl_wait();
  const int pos = a.pos_scalar ? *a.pos_scalar : (a.row_pos ? a.row_pos[row] : a.pos_base + row);
  const int tab = a.row_table ? a.row_table[row] : 0;
  const int* pt = a.page_table + (long long)tab * a.max_pages;
  const int npages = (pos + kPage) / kPage;  // pages holding positions [0, pos]
  const int nsplit = npages < a.nsplit_max ? npages : a.nsplit_max;
  if (split >= nsplit) return;
  const int p_begin = split * npages / nsplit;
  const int p_end = (split + 1) * npages / nsplit;

  __shared__ float qs[2][kHeadDim];
  __shared__ float tmp[3][kHeadDim];
  __shared__ float red[8];
  __shared__ float sm_m[4][2], sm_l[4][2];
  __shared__ float sm_acc[4][2][kHeadDim];
  __shared__ int sm_last;

  const float* qrow = a.qkv + (long long)row * a.qkv_stride;
  if (a.fused_kv) {
    // q_norm / k_norm (RMSNorm over head_dim) then rotate-half RoPE.
    const bool owner = (p_end == npages);  // this split holds position `pos`
    float q0 = qrow[(2 * h) * kHeadDim + t];
    float q1 = qrow[(2 * h + 1) * kHeadDim + t];
    const float qw = a.q_norm_w[t];
    float s0 = block_sum128(q0 * q0, red, t);
    float s1 = block_sum128(q1 * q1, red + 4, t);
    tmp[0][t] = q0 * rsqrtf(s0 / kHeadDim + 1e-6f) * qw;
    tmp[1][t] = q1 * rsqrtf(s1 / kHeadDim + 1e-6f) * qw;
    float kval = 0.f, vval = 0.f;
    if (owner) {
      kval = qrow[kQDim + h * kHeadDim + t];
      vval = qrow[kQDim + kKvDim + h * kHeadDim + t];
      const float sk = block_sum128(kval * kval, red, t);
      tmp[2][t] = kval * rsqrtf(sk / kHeadDim + 1e-6f) * a.k_norm_w[t];
    }
    __syncthreads();
    const int j = t & 63;
    const float c = a.rope_cos[pos * 64 + j], sn = a.rope_sin[pos * 64 + j];
    auto rope = [&](const float* x) {
      return t < 64 ? x[t] * c - x[t + 64] * sn : x[t] * c + x[t - 64] * sn;
    };
    qs[0][t] = rope(tmp[0]);
    qs[1][t] = rope(tmp[1]);
    if (owner) {
      const float kr = rope(tmp[2]);
      const int page = pt[pos / kPage];
      uint16_t* base = a.kv_layer + (long long)page * kPageElems +
                       (h * kPage + pos % kPage) * kHeadDim + t;
      base[0] = f2bf(kr);
      base[kHalfPageElems] = f2bf(vval);
    }
  } else {
    qs[0][t] = qrow[(2 * h) * kHeadDim + t];
    qs[1][t] = qrow[(2 * h + 1) * kHeadDim + t];
  }
  __syncthreads();

  const float scale = 0.08838834764831845f;  // 1/sqrt(128) as float
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const int r = lane & 15, hh = lane >> 4;
  for (int p = p_begin + warp; p < p_end; p += 4) {
    const int page = pt[p];
    const uint16_t* K = a.kv_layer + (long long)page * kPageElems + h * kPage * kHeadDim;
    const uint16_t* V = K + kHalfPageElems;
    const uint4* krow = reinterpret_cast<const uint4*>(K + r * kHeadDim);
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint4 w = krow[i];
      const float* q = &qs[hh][i * 8];
      dot = fmaf(q[0], bf_lo(w.x), dot);
      dot = fmaf(q[1], bf_hi(w.x), dot);
      dot = fmaf(q[2], bf_lo(w.y), dot);
      dot = fmaf(q[3], bf_hi(w.y), dot);
      dot = fmaf(q[4], bf_lo(w.z), dot);
      dot = fmaf(q[5], bf_hi(w.z), dot);
      dot = fmaf(q[6], bf_lo(w.w), dot);
      dot = fmaf(q[7], bf_hi(w.w), dot);
    }
    const bool valid = p * kPage + r <= pos;
    const float s = valid ? dot * scale : -INFINITY;
    float mx = s;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mx_other = __shfl_xor_sync(0xffffffffu, mx, 16);
    const float mxh[2] = {hh ? mx_other : mx, hh ? mx : mx_other};
    float mnew[2], corr[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      mnew[k] = fmaxf(m[k], mxh[k]);
      corr[k] = expf(m[k] - mnew[k]);
    }
    const float pl = valid ? expf(s - mnew[hh]) : 0.f;
    float ps = pl;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    const float ps_other = __shfl_xor_sync(0xffffffffu, ps, 16);
    const float psh[2] = {hh ? ps_other : ps, hh ? ps : ps_other};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      l[k] = l[k] * corr[k] + psh[k];
      m[k] = mnew[k];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[k][i] *= corr[k];
    }
#pragma unroll 4
    for (int r2 = 0; r2 < kPage; ++r2) {
      const uint2 vv = reinterpret_cast<const uint2*>(V + r2 * kHeadDim)[lane];
      const float p0 = __shfl_sync(0xffffffffu, pl, r2);
      const float p1 = __shfl_sync(0xffffffffu, pl, 16 + r2);
      const float v4[4] = {bf_lo(vv.x), bf_hi(vv.x), bf_lo(vv.y), bf_hi(vv.y)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[0][i] = fmaf(p0, v4[i], acc[0][i]);
        acc[1][i] = fmaf(p1, v4[i], acc[1][i]);
      }
    }
  }
  if (lane == 0) {
    sm_m[warp][0] = m[0]; sm_m[warp][1] = m[1];
    sm_l[warp][0] = l[0]; sm_l[warp][1] = l[1];
  }
#pragma unroll
  for (int k = 0; k < 2; ++k)
#pragma unroll
    for (int i = 0; i < 4; ++i) sm_acc[warp][k][lane * 4 + i] = acc[k][i];
  __syncthreads();

  float A[2], M[2], L[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    float mm = -INFINITY;
    for (int w = 0; w < 4; ++w) mm = fmaxf(mm, sm_m[w][k]);
    float ll = 0.f, aa = 0.f;
    for (int w = 0; w < 4; ++w) {
      const float e = sm_l[w][k] > 0.f ? expf(sm_m[w][k] - mm) : 0.f;
      ll += sm_l[w][k] * e;
      aa += sm_acc[w][k][t] * e;
    }
    A[k] = aa; M[k] = mm; L[k] = ll;
  }
  uint16_t* orow = a.out + (long long)row * kQDim + (2 * h) * kHeadDim + t;
  if (nsplit == 1) {
    orow[0] = f2bf(A[0] * (1.0f / L[0]));
    orow[kHeadDim] = f2bf(A[1] * (1.0f / L[1]));
    return;
  }
  const long long slot = ((long long)row * kKvHeads + h) * a.nsplit_max;
  float* part = a.part + (slot + split) * kPartStride;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    part[k * 132 + t] = A[k];
    if (t == 0) { part[k * 132 + 128] = M[k]; part[k * 132 + 129] = L[k]; }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const int ticket = atomicAdd(&a.counters[row * kKvHeads + h], 1);
    sm_last = (ticket == nsplit - 1);
  }
  __syncthreads();
  if (!sm_last) return;
  __threadfence();
  // Combine the splits: per-split (m, l) staged in shared memory, then every
  // thread sums its own output dimension over the splits (independent loads).
  __shared__ float sw[2][kMaxSplits];
  __shared__ float sl[2];
  if (t < 2 * nsplit) {
    const int k = t / nsplit, s2 = t % nsplit;
    sw[k][s2] = __ldcg(a.part + (slot + s2) * kPartStride + k * 132 + 128);
  }
  __syncthreads();
  if (t < 2) {
    float mm = -INFINITY;
    for (int s2 = 0; s2 < nsplit; ++s2) mm = fmaxf(mm, sw[t][s2]);
    float ll = 0.f;
    for (int s2 = 0; s2 < nsplit; ++s2) {
      const float e = expf(sw[t][s2] - mm);
      ll += __ldcg(a.part + (slot + s2) * kPartStride + t * 132 + 129) * e;
      sw[t][s2] = e;
    }
    sl[t] = ll;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    float aa = 0.f;
    for (int s2 = 0; s2 < nsplit; ++s2)
      aa += __ldcg(a.part + (slot + s2) * kPartStride + k * 132 + t) * sw[k][s2];
    orow[k * kHeadDim] = f2bf(aa * (1.0f / sl[k]));
  }
  if (t == 0) a.counters[row * kKvHeads + h] = 0;
}

// Prefill: one CTA per token row, warp per head. Lane holds d = lane + 32*i,
// so the rotate-half partner (d +/- 64) sits in the same lane.
__global__ void __launch_bounds__(256) qk_norm_rope_store_kernel(
    float* qkv, const float* qn, const float* kn, const float* cosT, const float* sinT,
    uint16_t* kv, const int* page_table, int max_pages, const int* row_table, const int* row_pos, int pos_base) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = row_pos ? row_pos[row] : pos_base + row;
  const int tab = row_table ? row_table[row] : 0;
  const int page = page_table[(long long)tab * max_pages + pos / kPage];
  float* x = qkv + (long long)row * kQkvDim;
  for (int hd = warp; hd < kQHeads + kKvHeads; hd += 8) {
    const bool isk = hd >= kQHeads;
    float* xh = x + hd * kHeadDim;
    const float* w = isk ? kn : qn;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = xh[lane + 32 * i];
    const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
    const float inv = rsqrtf(ss / kHeadDim + 1e-6f);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = v[i] * inv * w[lane + 32 * i];
    float o[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int j = lane + 32 * i;
      const float c = cosT[pos * 64 + j], s = sinT[pos * 64 + j];
      o[i] = v[i] * c - v[i + 2] * s;
      o[i + 2] = v[i + 2] * c + v[i] * s;
    }
    if (!isk) {
#pragma unroll
      for (int i = 0; i < 4; ++i) xh[lane + 32 * i] = o[i];
    } else {
      const int kh = hd - kQHeads;
      uint16_t* dst = kv + (long long)page * kPageElems + (kh * kPage + pos % kPage) * kHeadDim;
#pragma unroll
      for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = f2bf(o[i]);
    }
  }
  {
    const int kh = warp;  // 8 warps, 8 V heads
    const float* vh = x + kQDim + kKvDim + kh * kHeadDim;
    uint16_t* dst = kv + (long long)page * kPageElems + kHalfPageElems +
                    (kh * kPage + pos % kPage) * kHeadDim;
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = f2bf(vh[lane + 32 * i]);
  }
}

}  // namespace

void launch_attention(const AttnArgs& a, cudaStream_t s) {
  launch_pdl(attn_kernel, dim3(a.nsplit_max < kMaxSplits ? a.nsplit_max : kMaxSplits, kKvHeads, a.rows),
             dim3(kAttnThreads), 0, s, a);
}

void launch_qk_norm_rope_store(float* qkv, int rows, const float* qn, const float* kn,
                               const float* cos, const float* sin, uint16_t* kv_layer,
                               const int* page_table, int max_pages, const int* row_table,
                               const int* row_pos, int pos_base, cudaStream_t s) {
  if (rows <= 0) return;
  launch_pdl(qk_norm_rope_store_kernel, dim3(rows), dim3(256), 0, s, qkv, qn, kn, cos, sin,
             kv_layer, page_table, max_pages, row_table, row_pos, pos_base);
}

}  // namespace orx
