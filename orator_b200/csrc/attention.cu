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

constexpr int kAttnWarps = 8;          // one page per warp per group
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kPartStride = 2 * 132;   // per split: 2 heads x (128 acc, m, l, pad)
constexpr int kMaxSplits = 128;        // 2 * kMaxSplits <= threads
constexpr int kKRow = kHeadDim * 2 + 16;  // padded K row in shared memory (bytes)
constexpr int kKTile = kPage * kKRow;     // 4352
constexpr int kVTile = kPage * kHeadDim * 2;  // 4096
constexpr int kGroupBytes = kAttnWarps * (kKTile + kVTile);
constexpr int kAttnSmem = 2 * kGroupBytes + 128;  // double-buffered page groups

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n cp.async.wait_all;" ::: "memory");
}

// RMSNorm (eps 1e-6) + rotate-half RoPE of one 128-wide head held by a warp:
// lane holds d = lane + 32*i, so the RoPE partner d +/- 64 is in the same lane.
__device__ __forceinline__ void head_norm_rope(float v[4], const float* w, const float* cosT,
                                               const float* sinT, int pos, int lane) {
  const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
  const float inv = rsqrtf(ss / kHeadDim + 1e-6f);
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = v[i] * inv * w[lane + 32 * i];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int j = lane + 32 * i;
    const float c = cosT[pos * 64 + j], s = sinT[pos * 64 + j];
    const float lo = v[i], hi = v[i + 2];
    v[i] = lo * c - hi * s;
    v[i + 2] = hi * c + lo * s;
  }
}

// Stage pages [g0, g1) (at most kAttnWarps) of kv head h into shared memory.
__device__ __forceinline__ void stage_pages(uint8_t* sm, const uint16_t* kv, const int* pt,
                                            int h, int g0, int g1, int t) {
  const int n = (g1 - g0) * 2 * kPage * 16;  // 16-byte pieces (K and V)
  for (int i = t; i < n; i += kAttnThreads) {
    const int pg = i / (2 * kPage * 16), rem = i % (2 * kPage * 16);
    const int isv = rem / (kPage * 16), r = (rem / 16) % kPage, c = rem % 16;
    const uint16_t* src = kv + (long long)pt[g0 + pg] * kPageElems + (isv ? kHalfPageElems : 0) +
                          (h * kPage + r) * kHeadDim + c * 8;
    uint8_t* base = sm + pg * (kKTile + kVTile);
    const uint32_t dst = smem_u32(isv ? base + kKTile + r * kHeadDim * 2 + c * 16
                                      : base + r * kKRow + c * 16);
    cp_async16(dst, src);
  }
}

// Flash-decoding over a paged cache. Grid (splits, kv heads, rows); split s
// covers pages [s*P, (s+1)*P) of its row's page table (P = pages_per_split).
// In decode mode (fused_kv) the first page group is prefetched BEFORE
// griddepcontrol.wait using a speculative read of the position: cache entries
// older than the current position never change, and the one page that may be
// missing (when the position just crossed a page) is fetched after the wait.
__global__ void __launch_bounds__(kAttnThreads, 1) attn_kernel(AttnArgs a) {
  extern __shared__ uint8_t attn_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(attn_smem_raw) + 127) & ~uintptr_t(127));
  const int split = blockIdx.x, h = blockIdx.y, row = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int P = a.pages_per_split;
  trace_mark(a.trace, 0);
  const int tab = a.row_table ? a.row_table[row] : 0;
  const int* pt = a.page_table + (long long)tab * a.max_pages;
  const int* pos_ptr = a.pos_scalar ? a.pos_scalar : (a.row_pos ? a.row_pos + row : nullptr);
  const int pb = split * P;
  int staged_end = pb;  // pages [pb, staged_end) already requested
  if (a.fused_kv && pos_ptr) {
    const int pos_g = *reinterpret_cast<const volatile int*>(pos_ptr);
    int e = (pos_g + kPage) / kPage;
    e = e < pb + P ? e : pb + P;
    e = e < pb + kAttnWarps ? e : pb + kAttnWarps;
    if (e > pb && e <= a.max_pages) {
      stage_pages(sm, a.kv_layer, pt, h, pb, e, t);
      staged_end = e;
    }
  }
  pdl_trigger();
  pdl_wait();
  trace_mark(a.trace, 1);
  const int pos = pos_ptr ? *pos_ptr : a.pos_base + row;
  const int npages = (pos + kPage) / kPage;  // pages holding positions [0, pos]
  const int nsplit = (npages + P - 1) / P;
  if (split >= nsplit) {
    cp_async_wait_all();
    return;
  }
  const int pe = pb + P < npages ? pb + P : npages;

  __shared__ float qs[2][kHeadDim];
  __shared__ float sm_m[kAttnWarps][2], sm_l[kAttnWarps][2];
  __shared__ float sm_acc[kAttnWarps][2][kHeadDim];
  __shared__ int sm_last;

  const float* qrow = a.qkv + (long long)row * a.qkv_stride;
  const bool owner = a.fused_kv && pe == npages;  // this split holds position `pos`
  float knew[4], vnew[4];
  if (warp < 2) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = qrow[(2 * h + warp) * kHeadDim + lane + 32 * i];
    if (a.fused_kv) head_norm_rope(v, a.q_norm_w, a.rope_cos, a.rope_sin, pos, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) qs[warp][lane + 32 * i] = v[i];
  } else if (warp == 2 && owner) {
    // normalise, rotate and store K; store V (bf16, as the reference cache)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      knew[i] = qrow[kQDim + h * kHeadDim + lane + 32 * i];
      vnew[i] = qrow[kQDim + kKvDim + h * kHeadDim + lane + 32 * i];
    }
    head_norm_rope(knew, a.k_norm_w, a.rope_cos, a.rope_sin, pos, lane);
    uint16_t* dst = a.kv_layer + (long long)pt[pos / kPage] * kPageElems +
                    (h * kPage + pos % kPage) * kHeadDim;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      dst[lane + 32 * i] = f2bf(knew[i]);
      dst[kHalfPageElems + lane + 32 * i] = f2bf(vnew[i]);
    }
  }

  const float scale = 0.08838834764831845f;  // 1/sqrt(128) as float
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  const int r = lane & 15, hh = lane >> 4;
  // Page groups of kAttnWarps pages, double-buffered: group i+1 is in flight
  // while group i is consumed.
  if (staged_end < (pb + kAttnWarps < pe ? pb + kAttnWarps : pe)) {
    const int g1 = pb + kAttnWarps < pe ? pb + kAttnWarps : pe;
    stage_pages(sm + (staged_end - pb) * (kKTile + kVTile), a.kv_layer, pt, h, staged_end, g1, t);
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int g0 = pb; g0 < pe; g0 += kAttnWarps) {
    const int g1 = g0 + kAttnWarps < pe ? g0 + kAttnWarps : pe;
    uint8_t* buf = sm + (((g0 - pb) / kAttnWarps) & 1) * kGroupBytes;
    const bool more = g1 < pe;
    if (more) {
      const int n0 = g1, n1 = g1 + kAttnWarps < pe ? g1 + kAttnWarps : pe;
      stage_pages(sm + ((((g0 - pb) / kAttnWarps) + 1) & 1) * kGroupBytes, a.kv_layer, pt, h, n0,
                  n1, t);
      asm volatile("cp.async.commit_group;" ::: "memory");
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // every thread's copies of this group have landed
    if (owner && warp == 2 && g1 == pe) {
      // the staged copy of the newest slot may predate this step: patch it
      uint8_t* base = buf + (pos / kPage - g0) * (kKTile + kVTile);
      uint16_t* kd = reinterpret_cast<uint16_t*>(base + (pos % kPage) * kKRow);
      uint16_t* vd = reinterpret_cast<uint16_t*>(base + kKTile + (pos % kPage) * kHeadDim * 2);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kd[lane + 32 * i] = f2bf(knew[i]);
        vd[lane + 32 * i] = f2bf(vnew[i]);
      }
    }
    __syncthreads();
    const int p = g0 + warp;
    if (p < g1) {
      const uint8_t* base = buf + warp * (kKTile + kVTile);
      const uint4* krow = reinterpret_cast<const uint4*>(base + r * kKRow);
      const uint16_t* V = reinterpret_cast<const uint16_t*>(base + kKTile);
      float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const uint4 w = krow[i];
        const float* q = &qs[hh][i * 8];
        float& dot = d4[i & 3];
        dot = fmaf(q[0], bf_lo(w.x), dot);
        dot = fmaf(q[1], bf_hi(w.x), dot);
        dot = fmaf(q[2], bf_lo(w.y), dot);
        dot = fmaf(q[3], bf_hi(w.y), dot);
        dot = fmaf(q[4], bf_lo(w.z), dot);
        dot = fmaf(q[5], bf_hi(w.z), dot);
        dot = fmaf(q[6], bf_lo(w.w), dot);
        dot = fmaf(q[7], bf_hi(w.w), dot);
      }
      const float dot = (d4[0] + d4[1]) + (d4[2] + d4[3]);
      const bool valid = p * kPage + r <= pos;
      const float s = valid ? dot * scale : -INFINITY;
      float mx = s;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mx_other = __shfl_xor_sync(0xffffffffu, mx, 16);
      const float mx0 = hh ? mx_other : mx, mx1 = hh ? mx : mx_other;
      const float mn0 = fmaxf(m[0], mx0), mn1 = fmaxf(m[1], mx1);
      const float c0 = expf(m[0] - mn0), c1 = expf(m[1] - mn1);
      const float pl = valid ? expf(s - (hh ? mn1 : mn0)) : 0.f;
      float ps = pl;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      const float ps_other = __shfl_xor_sync(0xffffffffu, ps, 16);
      l[0] = l[0] * c0 + (hh ? ps_other : ps);
      l[1] = l[1] * c1 + (hh ? ps : ps_other);
      m[0] = mn0;
      m[1] = mn1;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[0][i] *= c0;
        acc[1][i] *= c1;
      }
#pragma unroll
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
    __syncthreads();  // this buffer is restaged two groups later
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
  const bool own = t < 2 * kHeadDim;  // threads 0..255 own (head kk, dim d)
  const int kk = (t >> 7) & 1, d = t & 127;
  float mm = -INFINITY, ll = 0.f, aa = 0.f;
  if (own) {
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, sm_m[w][kk]);
    for (int w = 0; w < kAttnWarps; ++w) {
      const float e = sm_l[w][kk] > 0.f ? expf(sm_m[w][kk] - mm) : 0.f;
      ll += sm_l[w][kk] * e;
      aa += sm_acc[w][kk][d] * e;
    }
  }
  uint16_t* orow = a.out + (long long)row * kQDim + (2 * h + kk) * kHeadDim + d;
  if (nsplit == 1) {
    if (own) *orow = f2bf(aa * (1.0f / ll));
    trace_mark(a.trace, 2);
    return;
  }
  const long long slot = ((long long)row * kKvHeads + h) * a.nsplit_max;
  if (own) {
    float* part = a.part + (slot + split) * kPartStride + kk * 132;
    part[d] = aa;
    if (d == 0) { part[128] = mm; part[129] = ll; }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const int ticket = atomicAdd(&a.counters[row * kKvHeads + h], 1);
    sm_last = (ticket == nsplit - 1);
  }
  __syncthreads();
  if (!sm_last) {
    trace_mark(a.trace, 2);
    return;
  }
  __threadfence();
  // Combine the splits: per-split (m, l) staged in shared memory, then every
  // owning thread sums its output dimension over the splits.
  __shared__ float sw[2][kMaxSplits];
  __shared__ float sl[2];
  if (t < 2 * nsplit) {
    const int k = t / nsplit, s2 = t % nsplit;
    sw[k][s2] = __ldcg(a.part + (slot + s2) * kPartStride + k * 132 + 128);
  }
  __syncthreads();
  if (t < 2) {
    float m2 = -INFINITY;
    for (int s2 = 0; s2 < nsplit; ++s2) m2 = fmaxf(m2, sw[t][s2]);
    float l2 = 0.f;
    for (int s2 = 0; s2 < nsplit; ++s2) {
      const float e = expf(sw[t][s2] - m2);
      l2 += __ldcg(a.part + (slot + s2) * kPartStride + t * 132 + 129) * e;
      sw[t][s2] = e;
    }
    sl[t] = l2;
  }
  __syncthreads();
  if (own) {
    float a2 = 0.f;
    for (int s2 = 0; s2 < nsplit; ++s2)
      a2 += __ldcg(a.part + (slot + s2) * kPartStride + kk * 132 + d) * sw[kk][s2];
    *orow = f2bf(a2 * (1.0f / sl[kk]));
  }
  if (t == 0) a.counters[row * kKvHeads + h] = 0;
  trace_mark(a.trace, 2);
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
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
    configured = true;
  }
  launch_pdl(attn_kernel, dim3(a.nsplit_max < kMaxSplits ? a.nsplit_max : kMaxSplits, kKvHeads, a.rows),
             dim3(kAttnThreads), kAttnSmem, s, a);
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
