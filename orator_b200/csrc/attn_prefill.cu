// Causal prefill attention over the paged cache, flash-attention style.
//
// Replaces GqaCacheAttnKernel (src/model/asr_text_decoder.cu:88-142: one warp
// per (token, head) walking every key of the cache). Here a CTA owns a tile of
// up to 16 consecutive query positions of one session and one kv head (its 2
// query heads = 32 query vectors); the session's K/V pages stream once per
// tile through an 8-slot ring of swizzled 2-D TMA tiles and feed tensor-core
// MMAs. Four warps per query head take every fourth page each (online
// softmax per warp) and merge their states at the end in a fixed order. Precision: q and the softmax probabilities are split into bf16 hi +
// lo parts (hi + lo carries about 16 more bits), so QK^T and PV on bf16 MMAs
// track the reference's fp32 dots against the bf16 cache.
#include <cuda.h>

#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace orx {
namespace {

constexpr int kKeyGroups = 4;                 // warps per query head, each on every 4th page
constexpr int kPfWarps = 2 * kKeyGroups;      // warp w: query head (w & 1), key group (w >> 1)
constexpr int kPfThreads = kPfWarps * 32;
constexpr int kPfRows = 16;  // query positions per tile
constexpr int kTileB = kPage * kHeadDim * 2;  // 4 KiB K or V tile
constexpr int kPtStage = 1024;                // page ids staged in shared memory
constexpr int kMergeFloats = 68;              // per lane: acc[16][4] + m0, m1, l0, l1
constexpr int kQFragB = 8 * 4 * 32 * 4 * 2;   // one warp's q fragments (hi + lo), bytes
// Two shapes of the kernel:
//  WIDE = false (launches of less than two waves): q fragments in registers,
//    two groups of pages in flight, one CTA per SM -- the shortest path for
//    one CTA;
//  WIDE = true (many tiles, e.g. a batch of joining sessions): q fragments
//    in shared memory and one group of pages in flight, so that two CTAs
//    (16 warps) fit on an SM -- more throughput per SM.
template <bool WIDE>
struct PfShape {
  static constexpr int kSlots = WIDE ? kKeyGroups : 2 * kKeyGroups;
  static constexpr int kRingB = kSlots * 2 * kTileB;
  static constexpr int kSmem = kRingB + (WIDE ? kPfWarps * kQFragB : 0) + 1024;
};
static_assert((kPfWarps - 2) * 32 * kMergeFloats * 4 <= PfShape<false>::kRingB,
              "merge buffer reuses the ring");
static_assert((kPfWarps - 2) * 32 * kMergeFloats * 4 <= kPfWarps * kQFragB,
              "merge buffer reuses the q fragments");

template <bool WIDE>
__global__ void __launch_bounds__(kPfThreads, WIDE ? 2 : 1)
    attn_prefill_kernel(const __grid_constant__ CUtensorMap kvmap, PrefillAttnArgs a) {
  constexpr int kSlots = PfShape<WIDE>::kSlots;
  constexpr int kRingB = PfShape<WIDE>::kRingB;
  extern __shared__ uint8_t pf_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(pf_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar[kSlots];
  // items in tile-major order (tiles arrive longest-first): blocks of one
  // launch wave take whole tiles, heaviest first
  const int tile = blockIdx.x / kKvHeads, h = blockIdx.x % kKvHeads;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const PrefillTile ti = a.tiles[tile];
  const int* pt = a.page_table + (long long)ti.tab * a.max_pages;
  const int npages = (ti.pos0 + ti.nrows - 1) / kPage + 1;  // keys [0, last position]
  // The session's page ids, staged in shared memory: a global load per TMA
  // issue would serialise one memory round trip per page on thread 0.
  __shared__ int spt[kPtStage];
  const bool staged = npages <= kPtStage;
  auto issue = [&](int p, int slot) {  // thread 0
    uint8_t* dst = sm + slot * 2 * kTileB;
    const int r0 = a.kv_row0 + ((staged ? spt[p] : pt[p]) * 2 * kKvHeads + h) * kPage;
    const int r1 = r0 + kKvHeads * kPage;
    mbar_arrive_expect_tx(&bar[slot], 2 * kTileB);
    tma_2d(dst, &kvmap, 0, r0, &bar[slot]);
    tma_2d(dst + 2048, &kvmap, 64, r0, &bar[slot]);
    tma_2d(dst + kTileB, &kvmap, 0, r1, &bar[slot]);
    tma_2d(dst + kTileB + 2048, &kvmap, 64, r1, &bar[slot]);
  };
  if (t == 0) {
    for (int i = 0; i < kSlots; ++i) mbar_init(&bar[i], 1);
    fence_mbar_init();
  }
  pdl_trigger();
  pdl_wait();  // K/V of this prefill are stored by the previous kernel
  if (staged)
    for (int i = t; i < npages; i += kPfThreads) spt[i] = pt[i];
  __syncthreads();
  if (t == 0)
    for (int p = 0; p < kSlots && p < npages; ++p) issue(p, p);

  // Q fragments of this warp's 16 rows: hi and lo bf16 parts.
  const int hh = warp & 1, kg = warp >> 1, rbase = 0;
  const int g = lane >> 2, tig = lane & 3;
  // q fragments: registers, or shared memory ([ks][r][lane], hi then lo)
  uint32_t qh[WIDE ? 1 : 8][4], ql[WIDE ? 1 : 8][4];
  uint32_t* qf = reinterpret_cast<uint32_t*>(sm + kRingB + warp * kQFragB);
  {
    const float* q0 = a.qkv + (long long)(ti.row0 + rbase + g) * a.qkv_stride + (2 * h + hh) * kHeadDim;
    const float* q1 = q0 + 8LL * a.qkv_stride;
    const bool v0 = rbase + g < ti.nrows, v1 = rbase + g + 8 < ti.nrows;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int c = ks * 16 + tig * 2;
      float x[8];
      x[0] = v0 ? q0[c] : 0.f;     x[1] = v0 ? q0[c + 1] : 0.f;
      x[2] = v1 ? q1[c] : 0.f;     x[3] = v1 ? q1[c + 1] : 0.f;
      x[4] = v0 ? q0[c + 8] : 0.f; x[5] = v0 ? q0[c + 9] : 0.f;
      x[6] = v1 ? q1[c + 8] : 0.f; x[7] = v1 ? q1[c + 9] : 0.f;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const uint32_t hv = pack_bf16(split_part(x[2 * r], false), split_part(x[2 * r + 1], false));
        const uint32_t lv = pack_bf16(split_part(x[2 * r], true), split_part(x[2 * r + 1], true));
        if constexpr (WIDE) {
          qf[(ks * 4 + r) * 32 + lane] = hv;
          qf[1024 + (ks * 4 + r) * 32 + lane] = lv;
        } else {
          qh[ks][r] = hv;
          ql[ks][r] = lv;
        }
      }
    }
  }
  const int qpos0 = ti.pos0 + rbase + g, qpos1 = qpos0 + 8;  // positions of rows g, g + 8
  const float scale = 0.08838834764831845f;  // 1/sqrt(128) as float
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

  for (int p0 = 0; p0 < npages; p0 += kKeyGroups) {
    const int p = p0 + kg;
    const int slot = p % kSlots;
    if (p < npages) {
    mbar_wait(&bar[slot], (p / kSlots) & 1, a.err, 51);
    const uint8_t* base = sm + slot * 2 * kTileB;
    // S = Q K^T for 16 rows x 16 positions
    float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int r = nt * 8 + g, c = ks * 16 + tig * 2;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(base + sw_off(r, c));
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(base + sw_off(r, c + 8));
        if constexpr (WIDE) {
          const uint32_t* qhk = qf + ks * 128 + lane;
          const uint32_t* qlk = qhk + 1024;
          mma_bf16(d[nt], qhk[0], qhk[32], qhk[64], qhk[96], b0, b1);
          mma_bf16(d[nt], qlk[0], qlk[32], qlk[64], qlk[96], b0, b1);
        } else {
          mma_bf16(d[nt], qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3], b0, b1);
          mma_bf16(d[nt], ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3], b0, b1);
        }
      }
    float s0[4], s1[4];  // rows g and g + 8; columns nt * 2 + j
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kp = p * kPage + nt * 8 + tig * 2 + j;
        s0[nt * 2 + j] = kp <= qpos0 ? d[nt][j] * scale : -INFINITY;
        s1[nt * 2 + j] = kp <= qpos1 ? d[nt][2 + j] * scale : -INFINITY;
      }
    float mx0 = fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s0[2], s0[3]));
    float mx1 = fmaxf(fmaxf(s1[0], s1[1]), fmaxf(s1[2], s1[3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // a page entirely in a row's future leaves that row's state unchanged
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float c0 = n0 == -INFINITY ? 1.f : expf(m0 - n0);
    const float c1 = n1 == -INFINITY ? 1.f : expf(m1 - n1);
    float p0[4], p1[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      p0[i] = s0[i] == -INFINITY ? 0.f : expf(s0[i] - n0);
      p1[i] = s1[i] == -INFINITY ? 0.f : expf(s1[i] - n1);
    }
    float ps0 = (p0[0] + p0[1]) + (p0[2] + p0[3]);
    float ps1 = (p1[0] + p1[1]) + (p1[2] + p1[3]);
    ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
    ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
    ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
    ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
    l0 = l0 * c0 + ps0;
    l1 = l1 * c1 + ps1;
    m0 = n0;
    m1 = n1;
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      acc[nt][0] *= c0; acc[nt][1] *= c0;
      acc[nt][2] *= c1; acc[nt][3] *= c1;
    }
    // P fragments (A of the PV MMA): a0 row g pos 0-7, a1 row g+8, a2 / a3 pos 8-15
    const uint32_t ph0 = pack_bf16(split_part(p0[0], false), split_part(p0[1], false));
    const uint32_t ph1 = pack_bf16(split_part(p1[0], false), split_part(p1[1], false));
    const uint32_t ph2 = pack_bf16(split_part(p0[2], false), split_part(p0[3], false));
    const uint32_t ph3 = pack_bf16(split_part(p1[2], false), split_part(p1[3], false));
    const uint32_t pl0 = pack_bf16(split_part(p0[0], true), split_part(p0[1], true));
    const uint32_t pl1 = pack_bf16(split_part(p1[0], true), split_part(p1[1], true));
    const uint32_t pl2 = pack_bf16(split_part(p0[2], true), split_part(p0[3], true));
    const uint32_t pl3 = pack_bf16(split_part(p1[2], true), split_part(p1[3], true));
    const uint8_t* vb = base + kTileB;
#pragma unroll
    for (int nt = 0; nt < 16; nt += 2) {
      const int vrow = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int vcol = nt * 8 + (lane >> 4) * 8;
      uint32_t b0, b1, b2, b3;
      asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                   : "=r"(b0), "=r"(b1), "=r"(b2), "=r"(b3)
                   : "r"(smem_u32(vb + sw_off(vrow, vcol))));
      mma_bf16(acc[nt], ph0, ph1, ph2, ph3, b0, b1);
      mma_bf16(acc[nt], pl0, pl1, pl2, pl3, b0, b1);
      mma_bf16(acc[nt + 1], ph0, ph1, ph2, ph3, b2, b3);
      mma_bf16(acc[nt + 1], pl0, pl1, pl2, pl3, b2, b3);
    }
    }
    __syncthreads();  // every warp is done with this group's slots
    if (t == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      for (int q = p0; q < p0 + kKeyGroups; ++q)
        if (q + kSlots < npages) issue(q + kSlots, q % kSlots);
    }
  }
  // Merge the key groups of each head in group order (deterministic): groups
  // 1..3 park their state in the (now idle) ring, group 0 combines.
  {
    float* mb = reinterpret_cast<float*>(WIDE ? sm + kRingB : sm);
    if (kg > 0) {
      float* dst = mb + ((size_t)(warp - 2) * 32 + lane) * kMergeFloats;
#pragma unroll
      for (int i = 0; i < 16; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) dst[i * 4 + j] = acc[i][j];
      dst[64] = m0;
      dst[65] = m1;
      dst[66] = l0;
      dst[67] = l1;
    }
    __syncthreads();
    if (kg > 0) return;
    float M0 = m0, M1 = m1;
#pragma unroll
    for (int k = 1; k < kKeyGroups; ++k) {
      const float* src = mb + ((size_t)(2 * k + hh - 2) * 32 + lane) * kMergeFloats;
      M0 = fmaxf(M0, src[64]);
      M1 = fmaxf(M1, src[65]);
    }
    auto w = [](float m, float M) { return m == -INFINITY ? 0.f : expf(m - M); };
    const float e0 = w(m0, M0), e1 = w(m1, M1);
    l0 *= e0;
    l1 *= e1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      acc[i][0] *= e0; acc[i][1] *= e0;
      acc[i][2] *= e1; acc[i][3] *= e1;
    }
#pragma unroll
    for (int k = 1; k < kKeyGroups; ++k) {
      const float* src = mb + ((size_t)(2 * k + hh - 2) * 32 + lane) * kMergeFloats;
      const float f0 = w(src[64], M0), f1 = w(src[65], M1);
      l0 = fmaf(src[66], f0, l0);
      l1 = fmaf(src[67], f1, l1);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        acc[i][0] = fmaf(src[i * 4 + 0], f0, acc[i][0]);
        acc[i][1] = fmaf(src[i * 4 + 1], f0, acc[i][1]);
        acc[i][2] = fmaf(src[i * 4 + 2], f1, acc[i][2]);
        acc[i][3] = fmaf(src[i * 4 + 3], f1, acc[i][3]);
      }
    }
  }
  // normalise and store (bf16, the cast before o_proj)
  const float i0 = l0 > 0.f ? 1.0f / l0 : 0.f, i1 = l1 > 0.f ? 1.0f / l1 : 0.f;
  const int r0 = rbase + g, r1 = r0 + 8;
  uint16_t* o0 = a.out + (long long)(ti.row0 + r0) * kQDim + (2 * h + hh) * kHeadDim;
  uint16_t* o1 = o0 + 8LL * kQDim;
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int c = nt * 8 + tig * 2;
    if (r0 < ti.nrows)
      *reinterpret_cast<uint32_t*>(o0 + c) = pack_bf16(acc[nt][0] * i0, acc[nt][1] * i0);
    if (r1 < ti.nrows)
      *reinterpret_cast<uint32_t*>(o1 + c) = pack_bf16(acc[nt][2] * i1, acc[nt][3] * i1);
  }
}

}  // namespace

void launch_attn_prefill(const PrefillAttnArgs& a, int ntiles, const uint16_t* kv_pool,
                         long long pool_rows, cudaStream_t s) {
  if (ntiles <= 0) return;
  static std::atomic<unsigned long long> configured{0};
  once_per_device(configured, [] {
    cudaFuncSetAttribute(attn_prefill_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         PfShape<false>::kSmem);
    cudaFuncSetAttribute(attn_prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         PfShape<true>::kSmem);
  });
  CUtensorMap map;
  if (!make_tmap_2d(&map, kv_pool, pool_rows, kHeadDim, 64, kPage)) return;
  const int items = ntiles * kKvHeads;
  if (items >= 2 * tc_sms())
    launch_pdl(attn_prefill_kernel<true>, dim3(items), dim3(kPfThreads), PfShape<true>::kSmem, s, map, a);
  else
    launch_pdl(attn_prefill_kernel<false>, dim3(items), dim3(kPfThreads), PfShape<false>::kSmem, s, map, a);
}

int prefill_tile_rows() { return kPfRows; }

}  // namespace orx
