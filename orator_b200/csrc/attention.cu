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

constexpr int kAttnWarps = 4;          // one page per warp per group
constexpr int kAttnThreads = kAttnWarps * 32;
constexpr int kPartStride = 2 * 132;   // per split: 2 heads x (128 acc, m, l, pad)
constexpr int kMaxSplits = 128;        // 2 * kMaxSplits <= threads
constexpr int kKRow = kHeadDim * 2;       // K / V row in shared memory (bytes)
constexpr int kKTile = kPage * kKRow;     // 4 KiB: one (page, kv head) K tile, as in HBM
constexpr int kVTile = kPage * kKRow;
constexpr int kGroupBytes = kAttnWarps * (kKTile + kVTile);
constexpr int kAttnSmem = 2 * kGroupBytes + 128;  // double-buffered page groups

__device__ __forceinline__ void mma_bf16(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  return static_cast<uint32_t>(f2bf(lo)) | (static_cast<uint32_t>(f2bf(hi)) << 16);
}
// bf16 part of x for rows 0-1 (hi) or its remainder for rows 2-3 (lo):
// hi + lo represents x to about 2^-16 relative, so bf16 MMAs give fp32-grade dots.
__device__ __forceinline__ float split_part(float x, bool lo) {
  const float h = bf2f(f2bf(x));
  return lo ? x - h : h;
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

// Stage pages [g0, g1) (at most kAttnWarps) of kv head h: one 1-D bulk copy
// (TMA engine) per 4 KiB K or V tile, completion counted on `bar`. Called by
// one thread; arrives on `bar` with the byte count.
__device__ __forceinline__ void stage_pages(uint8_t* sm, const uint16_t* kv, const int* pt,
                                            int h, int g0, int g1, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, static_cast<uint32_t>((g1 - g0) * (kKTile + kVTile)));
  for (int p = g0; p < g1; ++p) {
    const uint16_t* src = kv + (long long)pt[p] * kPageElems + h * kPage * kHeadDim;
    uint8_t* base = sm + (p - g0) * (kKTile + kVTile);
    bulk_g2s(base, src, kKTile, bar);
    bulk_g2s(base + kKTile, src + kHalfPageElems, kVTile, bar);
  }
}

// Flash-decoding over a paged cache. Grid (splits, kv heads, rows); split s
// covers pages [s*P, (s+1)*P) of its row's page table (P = pages_per_split).
// In decode mode (fused_kv) the first page group is prefetched BEFORE
// griddepcontrol.wait using a speculative read of the position: cache entries
// older than the current position never change, and the one page that may be
// missing (when the position just crossed a page) is fetched after the wait.
__global__ void __launch_bounds__(kAttnThreads, 3) attn_kernel(AttnArgs a) {
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
  // bar[0]: first group (2 arrivals: speculative + completion), bar[1], bar[2]:
  // later groups in buffers 0 / 1 (1 arrival each).
  __shared__ uint64_t bar[3];
  __shared__ int staged_end_s;
  if (t == 0) {
    mbar_init(&bar[0], 2);
    mbar_init(&bar[1], 1);
    mbar_init(&bar[2], 1);
    fence_mbar_init();
    int e = pb;
    if (a.fused_kv && pos_ptr) {
      const int pos_g = *reinterpret_cast<const volatile int*>(pos_ptr);
      e = (pos_g + kPage) / kPage;
      e = e < pb + P ? e : pb + P;
      e = e < pb + kAttnWarps ? e : pb + kAttnWarps;
      if (e < pb || e > a.max_pages) e = pb;
    }
    stage_pages(sm, a.kv_layer, pt, h, pb, e, &bar[0]);  // e == pb: arrival only
    staged_end_s = e;
  }
  pdl_trigger();
  pdl_wait();
  trace_mark(a.trace, 1);
  const int pos = pos_ptr ? *pos_ptr : a.pos_base + row;
  const int npages = (pos + kPage) / kPage;  // pages holding positions [0, pos]
  const int nsplit = (npages + P - 1) / P;
  __syncthreads();
  const int staged_end = staged_end_s;
  if (split >= nsplit) {
    if (t == 0) {  // do not leave with copies in flight
      mbar_arrive_expect_tx(&bar[0], 0);
      mbar_wait(&bar[0], 0, a.err, 41);
    }
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
  // Lane roles in the m16n8k16 fragments: row g = lane / 4. Rows 0-1 carry the
  // bf16 "hi" parts of query heads 0-1, rows 2-3 their "lo" remainders.
  const int g = lane >> 2;
  const bool qrow_ok = g < 4;
  float m_r = -INFINITY, l_r = 0.f;  // softmax state of head (g & 1)
  float acc16[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc16[i][0] = acc16[i][1] = acc16[i][2] = acc16[i][3] = 0.f;
  __syncthreads();  // qs written by warps 0-1
  uint32_t qa[8][2];  // A fragments (a0, a2) of the 8 K-steps; a1 = a3 = 0 (rows 8-15)
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int dim = ks * 16 + (lane & 3) * 2;
    if (qrow_ok) {
      const float* qv = qs[g & 1];
      const bool lo = g >= 2;
      qa[ks][0] = pack_bf16(split_part(qv[dim], lo), split_part(qv[dim + 1], lo));
      qa[ks][1] = pack_bf16(split_part(qv[dim + 8], lo), split_part(qv[dim + 9], lo));
    } else {
      qa[ks][0] = qa[ks][1] = 0u;
    }
  }
  // Page groups of kAttnWarps pages, double-buffered: group i+1 is in flight
  // while group i is consumed.
  if (t == 0) {
    const int g1 = pb + kAttnWarps < pe ? pb + kAttnWarps : pe;
    if (staged_end < g1)
      stage_pages(sm + (staged_end - pb) * (kKTile + kVTile), a.kv_layer, pt, h, staged_end, g1,
                  &bar[0]);
    else
      mbar_arrive_expect_tx(&bar[0], 0);
  }
  for (int g0 = pb; g0 < pe; g0 += kAttnWarps) {
    const int gi = (g0 - pb) / kAttnWarps;
    const int g1 = g0 + kAttnWarps < pe ? g0 + kAttnWarps : pe;
    uint8_t* buf = sm + (gi & 1) * kGroupBytes;
    if (g1 < pe && t == 0) {
      const int n1 = g1 + kAttnWarps < pe ? g1 + kAttnWarps : pe;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      stage_pages(sm + ((gi + 1) & 1) * kGroupBytes, a.kv_layer, pt, h, g1, n1,
                  &bar[1 + ((gi + 1) & 1)]);
    }
    // group gi >= 1 lives in buffer gi & 1 with barrier 1 + (gi & 1), phase (gi - 1) / 2
    if (gi == 0)
      mbar_wait(&bar[0], 0, a.err, 42);
    else
      mbar_wait(&bar[1 + (gi & 1)], ((gi - 1) >> 1) & 1, a.err, 43);
    __syncthreads();  // every thread's copies of this group have landed
    if (owner && warp == 2 && g1 == pe) {
      // the staged copy of the newest slot may predate this step: patch it
      uint8_t* base = buf + (pos / kPage - g0) * (kKTile + kVTile);
      uint16_t* kd = reinterpret_cast<uint16_t*>(base + (pos % kPage) * kKRow);
      uint16_t* vd = reinterpret_cast<uint16_t*>(base + kKTile + (pos % kPage) * kKRow);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        kd[lane + 32 * i] = f2bf(knew[i]);
        vd[lane + 32 * i] = f2bf(vnew[i]);
      }
    }
    __syncthreads();
    const int p = g0 + warp;
    if (p < g1) {
      // Tensor-core page: scores[16 rows x 16 positions] = Q~ K^T with Q~ rows
      // {q0 hi, q1 hi, q0 lo, q1 lo, 0...}; out += P~ V likewise.
      const uint8_t* base = buf + warp * (kKTile + kVTile);
      float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const uint8_t* kr = base + (nt * 8 + (lane >> 2)) * kKRow + (ks * 16 + (lane & 3) * 2) * 2;
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr);
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + 16);
          mma_bf16(d[nt], qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
        }
      }
      // combine hi + lo rows (lane ^ 8 holds the partner row g ^ 2)
      float sc[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const float v = d[nt][j] + __shfl_xor_sync(0xffffffffu, d[nt][j], 8);
          const int ppos = p * kPage + nt * 8 + (lane & 3) * 2 + j;
          sc[nt * 2 + j] = (ppos <= pos) ? v * scale : -INFINITY;
        }
      float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      // rows 4-15 (lanes 16-31) are zero rows: their state is computed but unused
      const float mn = fmaxf(m_r, mx);
      const float corr = expf(m_r - mn);
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pr[i] = sc[i] == -INFINITY ? 0.f : expf(sc[i] - mn);
      float ps = (pr[0] + pr[1]) + (pr[2] + pr[3]);
      ps += __shfl_xor_sync(0xffffffffu, ps, 1);
      ps += __shfl_xor_sync(0xffffffffu, ps, 2);
      l_r = l_r * corr + ps;
      m_r = mn;
      const bool lo = (lane >> 2) >= 2;
      uint32_t pa0 = 0u, pa2 = 0u;
      if (qrow_ok) {
        pa0 = pack_bf16(split_part(pr[0], lo), split_part(pr[1], lo));
        pa2 = pack_bf16(split_part(pr[2], lo), split_part(pr[3], lo));
      }
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        acc16[nt][0] *= corr;
        acc16[nt][1] *= corr;
      }
      const uint8_t* vb = base + kKTile;
#pragma unroll
      for (int nt = 0; nt < 16; nt += 2) {
        // matrices: (pos 0-7, dims 8nt..), (pos 8-15, dims 8nt..), (pos 0-7, dims 8nt+8..), (pos 8-15, ...)
        const int vrow = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int vcol = nt * 8 + (lane >> 4) * 8;
        const uint32_t addr = smem_u32(vb + vrow * kKRow + vcol * 2);
        uint32_t b0, b1, b2, b3;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3)
                     : "r"(addr));
        mma_bf16(acc16[nt], pa0, 0u, pa2, 0u, b0, b1);
        mma_bf16(acc16[nt + 1], pa0, 0u, pa2, 0u, b2, b3);
      }
    }
    __syncthreads();  // this buffer is restaged two groups later
  }
  // out rows: head (g&1) = row g + row g^2 (hi + lo)
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    acc16[nt][0] += __shfl_xor_sync(0xffffffffu, acc16[nt][0], 8);
    acc16[nt][1] += __shfl_xor_sync(0xffffffffu, acc16[nt][1], 8);
  }
  if (g < 2) {
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      sm_acc[warp][g][nt * 8 + (lane & 3) * 2] = acc16[nt][0];
      sm_acc[warp][g][nt * 8 + (lane & 3) * 2 + 1] = acc16[nt][1];
    }
    if ((lane & 3) == 0) {
      sm_m[warp][g] = m_r;
      sm_l[warp][g] = l_r;
    }
  }
  __syncthreads();
  // Outputs (head kk, dim d), o = kk * 128 + d, strided over the threads.
  constexpr int kOut = 2 * kHeadDim / kAttnThreads;
  float mmv[kOut], llv[kOut], aav[kOut];
#pragma unroll
  for (int q = 0; q < kOut; ++q) {
    const int o = t + q * kAttnThreads, kk = o >> 7, d = o & 127;
    float mm = -INFINITY, ll = 0.f, aa = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) mm = fmaxf(mm, sm_m[w][kk]);
    for (int w = 0; w < kAttnWarps; ++w) {
      const float e = sm_l[w][kk] > 0.f ? expf(sm_m[w][kk] - mm) : 0.f;
      ll += sm_l[w][kk] * e;
      aa += sm_acc[w][kk][d] * e;
    }
    mmv[q] = mm; llv[q] = ll; aav[q] = aa;
  }
  uint16_t* orow = a.out + (long long)row * kQDim + (2 * h) * kHeadDim;
  if (nsplit == 1) {
#pragma unroll
    for (int q = 0; q < kOut; ++q) orow[t + q * kAttnThreads] = f2bf(aav[q] * (1.0f / llv[q]));
    trace_mark(a.trace, 2);
    return;
  }
  const long long slot = ((long long)row * kKvHeads + h) * a.nsplit_max;
#pragma unroll
  for (int q = 0; q < kOut; ++q) {
    const int o = t + q * kAttnThreads, kk = o >> 7, d = o & 127;
    float* part = a.part + (slot + split) * kPartStride + kk * 132;
    part[d] = aav[q];
    if (d == 0) { part[128] = mmv[q]; part[129] = llv[q]; }
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
  // thread sums its output dimensions over the splits.
  __shared__ float sw[2][kMaxSplits];
  __shared__ float sl[2];
  for (int i2 = t; i2 < 2 * nsplit; i2 += kAttnThreads) {
    const int k = i2 / nsplit, s2 = i2 % nsplit;
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
#pragma unroll
  for (int q = 0; q < kOut; ++q) {
    const int o = t + q * kAttnThreads, kk = o >> 7, d = o & 127;
    float a2 = 0.f;
    for (int s2 = 0; s2 < nsplit; ++s2)
      a2 += __ldcg(a.part + (slot + s2) * kPartStride + kk * 132 + d) * sw[kk][s2];
    orow[o] = f2bf(a2 * (1.0f / sl[kk]));
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
