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
#include <cuda.h>

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
constexpr int kAttnSmem = kAttnWarps * 2 * (kKTile + kVTile) + 1024;  // 2-slot ring per warp

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
__global__ void __launch_bounds__(kAttnThreads, 3)
    attn_kernel(const __grid_constant__ CUtensorMap kvmap, AttnArgs a) {
  extern __shared__ uint8_t attn_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(attn_smem_raw) + 1023) & ~uintptr_t(1023));
  const int split = blockIdx.x, h = blockIdx.y, row = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int P = a.pages_per_split;
  trace_mark(a.trace, 0);
  const int tab = a.row_table ? a.row_table[row] : 0;
  const int* pt = a.page_table + (long long)tab * a.max_pages;
  const int* pos_ptr = a.pos_scalar ? a.pos_scalar : (a.row_pos ? a.row_pos + row : nullptr);
  const int pb = split * P;
  // Each warp streams its own pages (pb + warp, pb + warp + kAttnWarps, ...)
  // through a private 2-slot ring: K and V tiles by 2-D TMA with 128-byte
  // swizzle (conflict-free fragment loads), one mbarrier per slot.
  __shared__ uint64_t bar[kAttnWarps][2];
  uint8_t* ring = sm + warp * 2 * (kKTile + kVTile);
  auto issue = [&](int page_idx, int slot) {  // lane 0
    uint8_t* dst = ring + slot * (kKTile + kVTile);
    const int r0 = a.kv_row0 + (pt[page_idx] * 2 * kKvHeads + h) * kPage;   // K rows
    const int r1 = r0 + kKvHeads * kPage;                                     // V rows
    mbar_arrive_expect_tx(&bar[warp][slot], kKTile + kVTile);
    tma_2d(dst, &kvmap, 0, r0, &bar[warp][slot]);
    tma_2d(dst + 2048, &kvmap, 64, r0, &bar[warp][slot]);
    tma_2d(dst + kKTile, &kvmap, 0, r1, &bar[warp][slot]);
    tma_2d(dst + kKTile + 2048, &kvmap, 64, r1, &bar[warp][slot]);
  };
  int issued = 0;  // pages of this warp already requested (lane 0's view)
  if (lane == 0) {
    mbar_init(&bar[warp][0], 1);
    mbar_init(&bar[warp][1], 1);
    fence_mbar_init();
    if (a.fused_kv && pos_ptr) {
      // speculative: entries older than the current position never change
      const int pos_g = *reinterpret_cast<const volatile int*>(pos_ptr);
      int e = (pos_g + kPage) / kPage;
      e = e < pb + P ? e : pb + P;
      if (e <= a.max_pages)
        for (; issued < 2 && pb + warp + issued * kAttnWarps < e; ++issued)
          issue(pb + warp + issued * kAttnWarps, issued);
    }
  }
  pdl_trigger();
  pdl_wait();
  trace_mark(a.trace, 1);
  const int pos = pos_ptr ? *pos_ptr : a.pos_base + row;
  const int npages = (pos + kPage) / kPage;  // pages holding positions [0, pos]
  const int nsplit = (npages + P - 1) / P;
  const int pe = pb + P < npages ? pb + P : npages;
  const int nw = pe > pb + warp ? (pe - pb - warp + kAttnWarps - 1) / kAttnWarps : 0;
  if (lane == 0)
    for (; issued < 2 && issued < nw; ++issued) issue(pb + warp + issued * kAttnWarps, issued);
  issued = __shfl_sync(0xffffffffu, issued, 0);
  if (split >= nsplit) {
    // drain speculative copies before leaving
    for (int j = 0; j < issued; ++j) mbar_wait(&bar[warp][j], 0, a.err, 41);
    return;
  }

  __shared__ float qs[2][kHeadDim];
  __shared__ uint16_t knew_s[kHeadDim], vnew_s[kHeadDim];
  __shared__ float sm_m[kAttnWarps][2], sm_l[kAttnWarps][2];
  __shared__ float sm_acc[kAttnWarps][2][kHeadDim];
  __shared__ int sm_last;

  const float* qrow = a.qkv + (long long)row * a.qkv_stride;
  const bool owner = a.fused_kv && pe == npages;  // this split holds position `pos`
  if (warp < 2) {
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = qrow[(2 * h + warp) * kHeadDim + lane + 32 * i];
    if (a.fused_kv) head_norm_rope(v, a.q_norm_w, a.rope_cos, a.rope_sin, pos, lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) qs[warp][lane + 32 * i] = v[i];
  } else if (warp == 2 && owner) {
    // normalise, rotate and store K; store V (bf16, as the reference cache)
    float knew[4], vnew[4];
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
      const uint16_t kb = f2bf(knew[i]), vb = f2bf(vnew[i]);
      dst[lane + 32 * i] = kb;
      dst[kHalfPageElems + lane + 32 * i] = vb;
      knew_s[lane + 32 * i] = kb;
      vnew_s[lane + 32 * i] = vb;
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
  __syncthreads();  // qs / knew_s / vnew_s written
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

  for (int j = 0; j < nw; ++j) {
    const int p = pb + warp + j * kAttnWarps;
    const int slot = j & 1;
    mbar_wait(&bar[warp][slot], (j >> 1) & 1, a.err, 42);
    uint8_t* base = ring + slot * (kKTile + kVTile);
    if (owner && p == pos / kPage) {
      // the staged copy of the newest slot may predate this step: patch it
      const int r = pos % kPage;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = lane + 32 * i;
        *reinterpret_cast<uint16_t*>(base + sw_off(r, c)) = knew_s[c];
        *reinterpret_cast<uint16_t*>(base + kKTile + sw_off(r, c)) = vnew_s[c];
      }
      __syncwarp();
    }
    {
      // Tensor-core page: scores[16 rows x 16 positions] = Q~ K^T with Q~ rows
      // {q0 hi, q1 hi, q0 lo, q1 lo, 0...}; out += P~ V likewise.
      float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int r = nt * 8 + (lane >> 2), c = ks * 16 + (lane & 3) * 2;
          const uint32_t b0 = *reinterpret_cast<const uint32_t*>(base + sw_off(r, c));
          const uint32_t b1 = *reinterpret_cast<const uint32_t*>(base + sw_off(r, c + 8));
          mma_bf16(d[nt], qa[ks][0], 0u, qa[ks][1], 0u, b0, b1);
        }
      }
      // combine hi + lo rows (lane ^ 8 holds the partner row g ^ 2)
      float sc[4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const float v = d[nt][jj] + __shfl_xor_sync(0xffffffffu, d[nt][jj], 8);
          const int ppos = p * kPage + nt * 8 + (lane & 3) * 2 + jj;
          sc[nt * 2 + jj] = (ppos <= pos) ? v * scale : -INFINITY;
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
      const bool lo = g >= 2;
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
        const uint32_t addr = smem_u32(vb + sw_off(vrow, vcol));
        uint32_t b0, b1, b2, b3;
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                     : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3)
                     : "r"(addr));
        mma_bf16(acc16[nt], pa0, 0u, pa2, 0u, b0, b1);
        mma_bf16(acc16[nt + 1], pa0, 0u, pa2, 0u, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0 && j + 2 < nw) {  // the slot is free again: next page of this warp
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(pb + warp + (j + 2) * kAttnWarps, slot);
    }
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
  // One acquire-release ticket per CTA publishes the partial written by all
  // its threads (ordered before it by the barrier) and, for the last CTA of
  // the (row, head), acquires every other split's partial.
  __syncthreads();
  if (t == 0) {
    int ticket;
    asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;"
                 : "=r"(ticket)
                 : "l"(&a.counters[row * kKvHeads + h])
                 : "memory");
    sm_last = (ticket == nsplit - 1);
  }
  __syncthreads();
  if (!sm_last) {
    trace_mark(a.trace, 2);
    return;
  }
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
  // grid.y 0-2: heads 8y .. 8y+7 (16 q heads, then 8 k heads), one per warp;
  // grid.y 3: the V rows
  for (int hd = blockIdx.y * 8 + warp; blockIdx.y < 3 && hd < kQHeads + kKvHeads; hd += 24) {
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
  if (blockIdx.y == 3) {
    const int kh = warp;  // 8 warps, 8 V heads
    const float* vh = x + kQDim + kKvDim + kh * kHeadDim;
    uint16_t* dst = kv + (long long)page * kPageElems + kHalfPageElems +
                    (kh * kPage + pos % kPage) * kHeadDim;
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[lane + 32 * i] = f2bf(vh[lane + 32 * i]);
  }
}

}  // namespace

void launch_attention(const AttnArgs& a, const uint16_t* kv_pool, long long pool_rows,
                      cudaStream_t s) {
  static std::atomic<unsigned long long> configured{0};
  once_per_device(configured, [] {
    cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
  });
  // one map per pool; encoding is a host-side operation of about a microsecond
  CUtensorMap map;
  if (!make_tmap_2d(&map, kv_pool, pool_rows, kHeadDim, 64, kPage)) return;
  launch_pdl(attn_kernel, dim3(a.nsplit_max < kMaxSplits ? a.nsplit_max : kMaxSplits, kKvHeads, a.rows),
             dim3(kAttnThreads), kAttnSmem, s, map, a);
}

void launch_qk_norm_rope_store(float* qkv, int rows, const float* qn, const float* kn,
                               const float* cos, const float* sin, uint16_t* kv_layer,
                               const int* page_table, int max_pages, const int* row_table,
                               const int* row_pos, int pos_base, cudaStream_t s) {
  if (rows <= 0) return;
  launch_pdl(qk_norm_rope_store_kernel, dim3(rows, 4), dim3(256), 0, s, qkv, qn, kn, cos, sin,
             kv_layer, page_table, max_pages, row_table, row_pos, pos_base);
}

}  // namespace orx
