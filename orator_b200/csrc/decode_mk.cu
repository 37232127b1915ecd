// Persistent decode kernel: every phase of every layer of `steps` greedy
// tokens in ONE cooperative launch (one CTA per SM).
//
// The per-kernel decode chain (gemv.cu + attention.cu) pays a kernel boundary
// five times per layer: about 1.2 us until the dependent grid is released plus
// the ramp-up and drain of every launch. Here the phases of a token
//   per layer: qkv GEMV -> attention -> o GEMV -> gate/up GEMV -> down GEMV
//   then:      lm_head GEMV + banned argmax
// are separated by grid barriers (a monotonically growing arrival counter,
// bounded spin on the global timer, error word instead of a trap), and every
// warp streams its weight chunks continuously ACROSS the barriers: its 4-slot
// bulk-copy ring always runs ahead into the next phase's rows, so HBM keeps
// streaming while the grid synchronizes. Attention works on (kv head, split)
// items and leaves un-normalised partials; the o phase merges them in its
// prologue (no last-block combine on the critical path).
//
// Same math as the per-kernel path (and the reference,
// src/model/asr_text_decoder.cu:360-438): fp32 RMSNorm then bf16 activations
// before each projection, fp32 accumulation, bf16 KV, fp32 softmax, SwiGLU
// with expf, fp32 residual adds, tied lm_head with banned argmax.
#include <cstdlib>
#include <utility>

#include "common.cuh"
#include "engine.h"
#include "kernels.h"

namespace orx {
namespace {

constexpr int kW = 8;                  // warps per CTA
constexpr int kT = kW * 32;
constexpr int kDMax = 4;               // ring slots per warp (capacity)
constexpr int kChunkE = 2048;          // bf16 per chunk
constexpr int kChunkB = kChunkE * 2;   // 4 KiB
constexpr int kP = 8;                  // pages per attention split (one per warp)
constexpr int kKRowB = kHeadDim * 2 + 16;
constexpr int kKTileB = kPage * kKRowB;
constexpr int kVTileB = kPage * kHeadDim * 2;
constexpr int kPgB = kKTileB + kVTileB;
constexpr int kPart = kMkPart;         // floats per (kv head, split) partial
constexpr int kMaxSplit = kMkMaxSplit; // splits per kv head (4096 positions)
constexpr unsigned long long kBarrierNs = 1000ull * 1000 * 1000;

enum Phase : int { kPhQkv = 0, kPhO = 1, kPhGu = 2, kPhDown = 3, kPhLm = 4 };

struct MkSmem {
  alignas(128) uint8_t ring[kW * kDMax][kChunkB];   // 128 KiB weight rings
  alignas(128) uint8_t pages[kP][kPgB];          // 66 KiB attention staging
  alignas(16) uint16_t xs[kInter];               // activation of the phase
  uint64_t full[kW * kDMax];
  float red[kW];
  unsigned long long best[kW];
  float qs[2][kHeadDim];
  float sm_m[kW][2], sm_l[kW][2];
  float sm_acc[kW][2][kHeadDim];
  int ptab[kMkMaxSplit * kP];                    // the page table, read once per launch
  MkLayerW lw[kMkMaxLayers];                     // per-layer weight pointers (no global loads in issue)
  float xown[kMkOwnRows];  // this CTA's rows of the residual x (master copy)
};

static_assert(sizeof(MkSmem) + 128 <= 227 * 1024, "persistent decode kernel exceeds shared memory");

// Units of a phase held by CTA `b` of `G` and the warp's count of chunks.
struct PhaseGeom {
  int units, K, rpu;
  __device__ int cpr() const { return K / kChunkE; }
  __device__ int cpu() const { return rpu * cpr(); }
};

__device__ __forceinline__ PhaseGeom geom(int ph, int vocab) {
  switch (ph) {
    case kPhQkv: return {kQkvDim, kHidden, 1};
    case kPhO: return {kHidden, kQDim, 1};
    case kPhGu: return {kInter, kHidden, 2};
    case kPhDown: return {kHidden, kInter, 1};
    default: return {vocab, kHidden, 1};
  }
}

__device__ __forceinline__ void unit_range(int units, int b, int G, int& u0, int& n) {
  const long long a0 = (long long)b * units / G, a1 = (long long)(b + 1) * units / G;
  u0 = static_cast<int>(a0);
  n = static_cast<int>(a1 - a0);
}

__device__ __forceinline__ int warp_units(int n, int warp) {
  return n > warp ? (n - warp + kW - 1) / kW : 0;
}

// Grid barrier #k: every CTA adds one arrival (a release reduction: no
// round trip) and spins with acquire loads until the counter holds
// (k + 1) * G. Bounded: the shared error word is consulted only after 20 us
// of waiting (an earlier failure ends the wait then), and after the time
// limit the error word is set; no trap.
__device__ __forceinline__ void grid_barrier(unsigned int* ctr, unsigned int target, int* err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
    const unsigned long long t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
      unsigned int v;
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= target) break;
      if ((i & 63) == 0) {
        const unsigned long long dt = global_ns() - t0;
        if (dt > 20000ull && *reinterpret_cast<volatile int*>(err) != 0) break;
        if (dt > kBarrierNs) {
          atomicCAS(err, 0, 21);
          break;
        }
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ void cp_async16_mk(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ float ldcg_f(const float* p) { return __ldcg(p); }

template <int kD>
__global__ void __launch_bounds__(kT, 1) decode_mk_kernel(MkArgs a) {
  extern __shared__ uint8_t mk_raw[];
  MkSmem& sm = *reinterpret_cast<MkSmem*>((reinterpret_cast<uintptr_t>(mk_raw) + 127) &
                                          ~uintptr_t(127));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x, G = gridDim.x;
  int* err = &a.st->err;
  unsigned int bar_k = 0;  // barriers passed so far
  auto ready = [&]() {  // this CTA's inputs of the coming phase are in place
    if (a.trace_cta && tid == 0) a.trace_cta[((bar_k + 1) * G + b) * 2] = global_ns();
  };
  auto barrier_raw = [&]() {
    ++bar_k;
    if (a.trace && b == 0 && tid == 0) a.trace[2 * bar_k] = global_ns();   // arrive
    if (a.trace_cta && tid == 0) a.trace_cta[(bar_k * G + b) * 2 + 1] = global_ns();
    grid_barrier(a.bar, bar_k * static_cast<unsigned int>(G), err);
    if (a.trace && b == 0 && tid == 0) a.trace[2 * bar_k + 1] = global_ns();  // depart
  };
  if (a.trace && b == 0 && tid == 0) a.trace[1] = global_ns();

  // ---- this warp's chunk schedule ------------------------------------------
  int nph[5], u0ph[5];
  for (int ph = 0; ph < 5; ++ph) {
    const PhaseGeom g = geom(ph, a.vocab);
    int u0, n;
    unit_range(g.units, b, G, u0, n);
    u0ph[ph] = u0;
    nph[ph] = warp_units(n, warp) * g.cpu();
  }
  const int per_layer = nph[0] + nph[1] + nph[2] + nph[3];
  const long long per_token = (long long)a.L * per_layer + nph[4];
  const long long total = per_token * a.steps;
  uint64_t* full = &sm.full[warp * kD];

  // Chunk cursor (lane 0): walks (token, layer, phase, unit, row, chunk) in
  // consumption order without divisions; it feeds the ring.
  auto nu_of = [&](int ph) {
    return ph == 0 ? nph[0] : ph == 1 ? nph[1] : ph == 2 ? nph[2] / 2 : ph == 3 ? nph[3] / 3 : nph[4];
  };
  // Per phase the warp's rows are unit u0 + warp + 8k: row pointers advance
  // by a fixed stride (gate/up: +8 rows, +64 more when the unit crosses a
  // 64-unit block, since gate and up rows are interleaved in 128-row tiles).
  struct Cur {
    int l, ph, k, r, c, nu, unit;
    const uint16_t* rowp;  // row r = 0 of the current unit
    const uint16_t* p;     // the chunk the next issue copies
  };
  auto settle = [&](Cur& q) {  // enter phase q.ph at its first unit (skipping empty phases)
    while (true) {
      q.nu = nu_of(q.ph);
      if (q.k < q.nu) break;
      q.k = 0;
      if (q.ph == kPhLm) { q.ph = 0; q.l = 0; }
      else if (q.ph == kPhDown) { q.ph = (q.l + 1 < a.L) ? 0 : kPhLm; q.l = (q.l + 1 < a.L) ? q.l + 1 : q.l; }
      else ++q.ph;
    }
    const MkLayerW& Lw = sm.lw[q.l];
    const uint16_t* W = q.ph == kPhQkv ? Lw.qkv : q.ph == kPhO ? Lw.o : q.ph == kPhGu ? Lw.gu
                      : q.ph == kPhDown ? Lw.down : a.embed;
    const int K = (q.ph == kPhDown) ? kInter : kHidden;
    q.unit = (q.ph == 0 ? u0ph[0] : q.ph == 1 ? u0ph[1] : q.ph == 2 ? u0ph[2]
              : q.ph == 3 ? u0ph[3] : u0ph[4]) + warp;
    const long long row = q.ph == kPhGu ? (long long)(q.unit >> 6) * 128 + (q.unit & 63) : q.unit;
    q.rowp = W + row * K;
    q.p = q.rowp;
  };
  auto advance = [&](Cur& q) {
    if (q.ph == kPhDown) {  // three chunks per row
      if (++q.c < kInter / kChunkE) {
        q.p += kChunkE;
        return;
      }
      q.c = 0;
    } else if (q.ph == kPhGu && q.r == 0) {  // gate row -> up row of the same unit
      q.r = 1;
      q.p = q.rowp + 64 * kHidden;
      return;
    }
    q.r = 0;
    if (++q.k == q.nu) {
      q.k = 0;
      if (q.ph == kPhLm) { q.ph = 0; q.l = 0; }
      else if (q.ph == kPhDown) { q.ph = (q.l + 1 < a.L) ? 0 : kPhLm; q.l = (q.l + 1 < a.L) ? q.l + 1 : q.l; }
      else ++q.ph;
      settle(q);
      return;
    }
    const int K = (q.ph == kPhDown) ? kInter : kHidden;
    int step = kW;
    if (q.ph == kPhGu && (q.unit & 63) >= 64 - kW) step += 64;
    q.unit += kW;
    q.rowp += (long long)step * K;
    q.p = q.rowp;
  };
  Cur cur = {0, 0, 0, 0, 0, 0, 0, nullptr, nullptr};
  auto issue = [&](long long seq) {  // lane 0 only; seq selects the ring slot
    const int slot = static_cast<int>(seq % kD);
    mbar_arrive_expect_tx(&full[slot], kChunkB);
    bulk_g2s(sm.ring[warp * kD + slot], cur.p, kChunkB, &full[slot]);
    advance(cur);
  };
  for (int i = tid; i < a.L * static_cast<int>(sizeof(MkLayerW) / 8); i += kT)
    reinterpret_cast<unsigned long long*>(sm.lw)[i] = reinterpret_cast<const unsigned long long*>(a.layers)[i];
  __syncthreads();
  settle(cur);
  if (lane == 0) {
    for (int i = 0; i < kD; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
    for (long long q = 0; q < kD && q < total; ++q) issue(q);
  }
  __syncwarp();
  long long seq = 0;  // next chunk this warp consumes
  auto barrier = [&]() { barrier_raw(); };

  // Consume one phase: per unit of this warp, rpu rows of cpr chunks each.
  // A slot is refilled right after the warp's FMAs have consumed the values
  // it loaded from it (so the bulk copy cannot overwrite unread data and no
  // proxy fence is needed). Row sums are reduced two at a time: lanes 0-15
  // finish row A and lanes 16-31 row B in one 5-step butterfly (the same
  // addition tree as a full-warp reduction, so the sums are unchanged), and
  // lanes 0 and 16 run the two epilogues side by side. In the gate/up phase
  // the pair is (gate, up) of one unit.
  auto run_phase = [&](int ph, auto&& epi) {
    const PhaseGeom g = geom(ph, a.vocab);
    const int nu = nph[ph] / g.cpu();
    float held = 0.f;      // partial of a row waiting for its partner (rpu == 1)
    int held_unit = -1;
    // With one chunk per row (K = 2048) every row meets the same activation
    // slice: keep it in registers for the whole phase.
    const bool one = g.cpr() == 1;
    uint4 xr[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) xr[j] = reinterpret_cast<const uint4*>(sm.xs)[j * 32 + lane];
    for (int k = 0; k < nu; ++k) {
      const int unit = u0ph[ph] + warp + k * kW;
      float part[2] = {0.f, 0.f};
      for (int r = 0; r < g.rpu; ++r) {
        float acc4[4] = {0.f, 0.f, 0.f, 0.f};
        for (int c = 0; c < g.cpr(); ++c) {
          const int slot = static_cast<int>(seq % kD);
          mbar_wait(&full[slot], static_cast<uint32_t>((seq / kD) & 1), err, 23);
          const uint4* wp = reinterpret_cast<const uint4*>(sm.ring[warp * kD + slot]);
          const uint4* xp = reinterpret_cast<const uint4*>(sm.xs + c * kChunkE);
          uint4 wv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) wv[j] = wp[j * 32 + lane];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint4 w = wv[j];
            const uint4 xv = one ? xr[j] : xp[j * 32 + lane];
            float& acc = acc4[j & 3];
            acc = fma2_bf16(w.x, xv.x, acc);
            acc = fma2_bf16(w.y, xv.y, acc);
            acc = fma2_bf16(w.z, xv.z, acc);
            acc = fma2_bf16(w.w, xv.w, acc);
          }
          __syncwarp();
          if (lane == 0 && seq + kD < total) issue(seq + kD);
          ++seq;
        }
        part[r] = (acc4[0] + acc4[1]) + (acc4[2] + acc4[3]);
      }
      if (g.rpu == 2) {
        const float s = reduce_pair(part[0], part[1], lane);  // lane 0: gate, lane 16: up
        const float up = __shfl_sync(0xffffffffu, s, 16);
        if (lane == 0) epi(unit, s, up);
      } else if (held_unit >= 0) {
        const float s = reduce_pair(held, part[0], lane);
        if (lane == 0) epi(held_unit, s, 0.f);
        if (lane == 16) epi(unit, s, 0.f);
        held_unit = -1;
      } else {
        held = part[0];
        held_unit = unit;
      }
    }
    if (held_unit >= 0) {
      const float s = warp_sum(held);
      if (lane == 0) epi(held_unit, s, 0.f);
    }
  };

  // RMSNorm of a fp32 row of 2048 (global, or given values) into sm.xs as bf16.
  auto load_w8 = [&](const float* w, float* wv) {
    const float4 w0 = reinterpret_cast<const float4*>(w)[tid * 2];
    const float4 w1 = reinterpret_cast<const float4*>(w)[tid * 2 + 1];
    wv[0] = w0.x; wv[1] = w0.y; wv[2] = w0.z; wv[3] = w0.w;
    wv[4] = w1.x; wv[5] = w1.y; wv[6] = w1.z; wv[7] = w1.w;
  };
  // `wv`: this thread's 8 norm weights, loaded ahead (before the barrier).
  auto norm_to_xs = [&](const float* v8, const float* wv) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v8[j] * v8[j];
    ss = warp_sum(ss);
    if (lane == 0) sm.red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < kW; ++w2) tot += sm.red[w2];
    const float inv = rsqrtf(tot / kHidden + a.eps);
    uint32_t pk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      pk[j] = static_cast<uint32_t>(f2bf(v8[2 * j] * inv * wv[2 * j])) |
              (static_cast<uint32_t>(f2bf(v8[2 * j + 1] * inv * wv[2 * j + 1])) << 16);
    reinterpret_cast<uint4*>(sm.xs)[tid] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    __syncthreads();
  };
  auto load_x8 = [&](float* v8) {
    const float4 p0 = __ldcg(reinterpret_cast<const float4*>(a.x) + tid * 2);
    const float4 p1 = __ldcg(reinterpret_cast<const float4*>(a.x) + tid * 2 + 1);
    v8[0] = p0.x; v8[1] = p0.y; v8[2] = p0.z; v8[3] = p0.w;
    v8[4] = p1.x; v8[5] = p1.y; v8[6] = p1.z; v8[7] = p1.w;
  };

  const float scale = 0.08838834764831845f;  // 1/sqrt(128) as float
  // rows of x this CTA owns in the o and down phases (same split of 2048)
  const int u_own = u0ph[kPhO];
  int n_own;
  {
    int u0;
    unit_range(kHidden, b, G, u0, n_own);
  }
  float wn[8];  // norm weights of the coming phase
  // Stage this CTA's first attention item of `layer` at position p into
  // sm.pages (cache entries older than p are final; the owner of the last
  // page patches row p itself). Issued one layer ahead, right after the
  // previous attention phase, so the copies run under the o/gate-up/down
  // phases instead of delaying the next qkv phase.
  auto stage_first = [&](int layer, int p) {
    const int np = (p + kPage) / kPage, ns = (np + kP - 1) / kP;
    if (b >= kKvHeads * ns) return;
    const int h0 = b / ns, s0 = b % ns;
    const uint16_t* kvl = a.kv + (long long)layer * a.kv_layer_stride;
    const int pb = s0 * kP, pe = pb + kP < np ? pb + kP : np;
    const int n16 = (pe - pb) * 2 * kPage * 16;
    for (int i = tid; i < n16; i += kT) {
      const int pg = i / (2 * kPage * 16), rem = i % (2 * kPage * 16);
      const int isv = rem / (kPage * 16), r = (rem / 16) % kPage, c = rem % 16;
      const uint16_t* src = kvl + (long long)sm.ptab[pb + pg] * kPageElems +
                            (isv ? kHalfPageElems : 0) + (h0 * kPage + r) * kHeadDim + c * 8;
      uint8_t* base = sm.pages[pg];
      cp_async16_mk(smem_u32(isv ? base + kKTileB + r * kHeadDim * 2 + c * 16
                                 : base + r * kKRowB + c * 16), src);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int i = tid; i < kMkMaxSplit * kP; i += kT) sm.ptab[i] = i < a.max_pages ? a.page_table[i] : 0;
  __syncthreads();
  stage_first(0, a.pos0);

  for (int t = 0; t < a.steps; ++t) {
    const int pos = a.pos0 + t;
    int tok;
    if (t == 0) {
      tok = *a.tok_ptr;
    } else {
      tok = argmax_key_index(__ldcg(&a.best2[(t - 1) & 1]));
    }
    if (b == 0 && tid == 0 && a.record) {
      const int k = a.count0 + t;
      if (k < a.st->out_cap) a.st->out[k] = tok;
    }
    const int npages = (pos + kPage) / kPage;
    const int nsplit = (npages + kP - 1) / kP;
    const int items = kKvHeads * nsplit;

    for (int l = 0; l < a.L; ++l) {
      const MkLayerW& Lw = sm.lw[l];
      uint16_t* kvl = a.kv + (long long)l * a.kv_layer_stride;
      // ---------------- qkv ----------------
      {
        float v8[8];
        if (l == 0) {
          const uint4 w = reinterpret_cast<const uint4*>(a.embed + (long long)tok * kHidden)[tid];
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) { v8[2 * j] = bf_lo(ww[j]); v8[2 * j + 1] = bf_hi(ww[j]); }
          if (tid < n_own) sm.xown[tid] = bf2f(a.embed[(long long)tok * kHidden + u_own + tid]);
          load_w8(Lw.in_ln, wn);
        } else {
          load_x8(v8);
        }
        norm_to_xs(v8, wn);
        ready();
        run_phase(kPhQkv, [&](int u, float acc, float) { a.qkv[u] = acc; });
      }
      barrier();
      if (l == 0 && b == 0 && tid == 0) a.best2[(t + 1) & 1] = 0ull;

      // ---------------- attention ----------------
      for (int it = b; it < items; it += G) {
        const int h = it / nsplit, sp = it % nsplit;
        const int pb = sp * kP, pe = pb + kP < npages ? pb + kP : npages;
        if (it != b) {  // further items (very long contexts): stage now
          __syncthreads();
          const int n16 = (pe - pb) * 2 * kPage * 16;
          for (int i = tid; i < n16; i += kT) {
            const int pg = i / (2 * kPage * 16), rem = i % (2 * kPage * 16);
            const int isv = rem / (kPage * 16), r = (rem / 16) % kPage, c = rem % 16;
            const uint16_t* src = kvl + (long long)sm.ptab[pb + pg] * kPageElems +
                                  (isv ? kHalfPageElems : 0) + (h * kPage + r) * kHeadDim + c * 8;
            uint8_t* base = sm.pages[pg];
            cp_async16_mk(smem_u32(isv ? base + kKTileB + r * kHeadDim * 2 + c * 16
                                       : base + r * kKRowB + c * 16), src);
          }
          asm volatile("cp.async.commit_group;" ::: "memory");
        }
        const bool owner = (pe == npages);
        float knew[4], vnew[4];
        if (warp < 2) {
          float v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = __ldcg(a.qkv + (2 * h + warp) * kHeadDim + lane + 32 * i);
          const float* w = Lw.qn;
          const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
          const float inv = rsqrtf(ss / kHeadDim + 1e-6f);
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = v[i] * inv * w[lane + 32 * i];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int j = lane + 32 * i;
            const float c = a.rope_cos[pos * 64 + j], sn = a.rope_sin[pos * 64 + j];
            const float lo = v[i], hi = v[i + 2];
            v[i] = lo * c - hi * sn;
            v[i + 2] = hi * c + lo * sn;
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) sm.qs[warp][lane + 32 * i] = v[i];
        } else if (warp == 2 && owner) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            knew[i] = __ldcg(a.qkv + kQDim + h * kHeadDim + lane + 32 * i);
            vnew[i] = __ldcg(a.qkv + kQDim + kKvDim + h * kHeadDim + lane + 32 * i);
          }
          const float ss = warp_sum(knew[0] * knew[0] + knew[1] * knew[1] + knew[2] * knew[2] +
                                    knew[3] * knew[3]);
          const float inv = rsqrtf(ss / kHeadDim + 1e-6f);
#pragma unroll
          for (int i = 0; i < 4; ++i) knew[i] = knew[i] * inv * Lw.kn[lane + 32 * i];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int j = lane + 32 * i;
            const float c = a.rope_cos[pos * 64 + j], sn = a.rope_sin[pos * 64 + j];
            const float lo = knew[i], hi = knew[i + 2];
            knew[i] = lo * c - hi * sn;
            knew[i + 2] = hi * c + lo * sn;
          }
          uint16_t* dst = kvl + (long long)sm.ptab[pos / kPage] * kPageElems +
                          (h * kPage + pos % kPage) * kHeadDim;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dst[lane + 32 * i] = f2bf(knew[i]);
            dst[kHalfPageElems + lane + 32 * i] = f2bf(vnew[i]);
          }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
        __syncthreads();
        if (it == b) ready();
        if (owner && warp == 2) {
          uint8_t* base = sm.pages[pos / kPage - pb];
          uint16_t* kd = reinterpret_cast<uint16_t*>(base + (pos % kPage) * kKRowB);
          uint16_t* vd = reinterpret_cast<uint16_t*>(base + kKTileB + (pos % kPage) * kHeadDim * 2);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            kd[lane + 32 * i] = f2bf(knew[i]);
            vd[lane + 32 * i] = f2bf(vnew[i]);
          }
        }
        __syncthreads();
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
        float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
        const int p = pb + warp;
        if (p < pe) {
          const int r = lane & 15, hh = lane >> 4;
          const uint8_t* base = sm.pages[warp];
          const uint4* krow = reinterpret_cast<const uint4*>(base + r * kKRowB);
          const uint16_t* V = reinterpret_cast<const uint16_t*>(base + kKTileB);
          float d4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const uint4 w = krow[i];
            const float* q = &sm.qs[hh][i * 8];
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
          const float sc = valid ? dot * scale : -INFINITY;
          float mx = sc;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
          const float mxo = __shfl_xor_sync(0xffffffffu, mx, 16);
          m0 = hh ? mxo : mx;
          m1 = hh ? mx : mxo;
          const float pl = valid ? expf(sc - (hh ? m1 : m0)) : 0.f;
          float ps = pl;
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
          const float pso = __shfl_xor_sync(0xffffffffu, ps, 16);
          l0 = hh ? pso : ps;
          l1 = hh ? ps : pso;
#pragma unroll
          for (int r2 = 0; r2 < kPage; ++r2) {
            const uint2 vv = reinterpret_cast<const uint2*>(V + r2 * kHeadDim)[lane];
            const float p0 = __shfl_sync(0xffffffffu, pl, r2);
            const float p1 = __shfl_sync(0xffffffffu, pl, 16 + r2);
            const float v4[4] = {bf_lo(vv.x), bf_hi(vv.x), bf_lo(vv.y), bf_hi(vv.y)};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              acc0[i] = fmaf(p0, v4[i], acc0[i]);
              acc1[i] = fmaf(p1, v4[i], acc1[i]);
            }
          }
        }
        if (lane == 0) {
          sm.sm_m[warp][0] = m0; sm.sm_m[warp][1] = m1;
          sm.sm_l[warp][0] = l0; sm.sm_l[warp][1] = l1;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          sm.sm_acc[warp][0][lane * 4 + i] = acc0[i];
          sm.sm_acc[warp][1][lane * 4 + i] = acc1[i];
        }
        __syncthreads();
        {  // CTA combine -> partial (m, l, unnormalised acc) of both q heads
          const int kk = tid >> 7, d = tid & 127;
          float mm = -INFINITY;
          for (int w2 = 0; w2 < kW; ++w2) mm = fmaxf(mm, sm.sm_m[w2][kk]);
          float ll = 0.f, aa = 0.f;
          for (int w2 = 0; w2 < kW; ++w2) {
            const float e = sm.sm_l[w2][kk] > 0.f ? expf(sm.sm_m[w2][kk] - mm) : 0.f;
            ll += sm.sm_l[w2][kk] * e;
            aa += sm.sm_acc[w2][kk][d] * e;
          }
          float* part = a.part + ((long long)h * kMaxSplit + sp) * kPart + kk * 132;
          part[d] = aa;
          if (d == 0) { part[128] = mm; part[129] = ll; }
        }
      }
      // pages are free again (the last item's reads precede its final sync)
      if (l + 1 < a.L) stage_first(l + 1, pos);
      else if (t + 1 < a.steps) stage_first(0, pos + 1);
      barrier();

      // ---------------- o (merges the attention splits) ----------------
      {
        // Every thread merges the splits of its 8 output dims in one pass of
        // independent loads (running max, rescaled sums): one L2 round trip.
        const int d0 = tid * 8, qh = d0 / kHeadDim, h = qh >> 1, kk = qh & 1;
        const float* pbase = a.part + (long long)h * kMaxSplit * kPart + kk * 132;
        const int dd = d0 % kHeadDim;
        float o8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float mm = -INFINITY, ll = 0.f;
#pragma unroll 4
        for (int sp = 0; sp < nsplit; ++sp) {
          const float* ps = pbase + sp * kPart;
          const float2 ml = __ldcg(reinterpret_cast<const float2*>(ps + 128));
          const float4 q0 = __ldcg(reinterpret_cast<const float4*>(ps + dd));
          const float4 q1 = __ldcg(reinterpret_cast<const float4*>(ps + dd + 4));
          const float mn = fmaxf(mm, ml.x);
          const float co = expf(mm - mn), cs = expf(ml.x - mn);
          ll = ll * co + ml.y * cs;
          o8[0] = o8[0] * co + q0.x * cs; o8[1] = o8[1] * co + q0.y * cs;
          o8[2] = o8[2] * co + q0.z * cs; o8[3] = o8[3] * co + q0.w * cs;
          o8[4] = o8[4] * co + q1.x * cs; o8[5] = o8[5] * co + q1.y * cs;
          o8[6] = o8[6] * co + q1.z * cs; o8[7] = o8[7] * co + q1.w * cs;
          mm = mn;
        }
        const float inv = 1.0f / ll;
        uint32_t pk[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          pk[j] = static_cast<uint32_t>(f2bf(o8[2 * j] * inv)) |
                  (static_cast<uint32_t>(f2bf(o8[2 * j + 1] * inv)) << 16);
        reinterpret_cast<uint4*>(sm.xs)[tid] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        __syncthreads();
        ready();
        run_phase(kPhO, [&](int u, float acc, float) {
          const float xn = sm.xown[u - u_own] + acc;  // this lane wrote it last (down phase)
          sm.xown[u - u_own] = xn;
          a.x[u] = xn;
        });
      }
      load_w8(Lw.post_ln, wn);
      barrier();

      // ---------------- gate/up + SwiGLU ----------------
      {
        float v8[8];
        load_x8(v8);
        norm_to_xs(v8, wn);
        ready();
        run_phase(kPhGu, [&](int u, float g, float up) {
          a.act_g[u] = f2bf((g / (1.0f + expf(-g))) * up);
        });
      }
      barrier();

      // ---------------- down ----------------
      {
        const uint4* src = reinterpret_cast<const uint4*>(a.act_g);
        for (int i = tid; i < kInter / 8; i += kT) reinterpret_cast<uint4*>(sm.xs)[i] = __ldcg(src + i);
        __syncthreads();
        ready();
        run_phase(kPhDown, [&](int u, float acc, float) {
          const float xn = sm.xown[u - u_own] + acc;
          sm.xown[u - u_own] = xn;
          a.x[u] = xn;
        });
      }
      load_w8(l + 1 < a.L ? sm.lw[l + 1].in_ln : a.final_norm, wn);
      barrier();
    }

    // ---------------- final norm + lm_head + banned argmax ----------------
    {
      float v8[8];
      load_x8(v8);
      norm_to_xs(v8, wn);
      const int count_after = a.record ? a.count0 + t + 1 : a.count0;
      const bool ban = count_after < a.ban_steps;
      const int bn0 = ban ? a.ban0 : -1, bn1 = ban ? a.ban1 : -1;
      unsigned long long best = 0ull;
      ready();
      run_phase(kPhLm, [&](int u, float acc, float) {
        a.logits[u] = acc;
        if (u != bn0 && u != bn1 && !(acc != acc)) {
          const unsigned long long k = argmax_key(acc, u);
          best = k > best ? k : best;
        }
      });
      {
        const unsigned long long ob = __shfl_sync(0xffffffffu, best, 16);
        if (lane == 0) sm.best[warp] = ob > best ? ob : best;
      }
      __syncthreads();
      if (tid == 0) {
        unsigned long long bb = 0;
        for (int w2 = 0; w2 < kW; ++w2) bb = sm.best[w2] > bb ? sm.best[w2] : bb;
        if (bb) atomicMax(&a.best2[t & 1], bb);
      }
    }
    barrier();
  }
  if (b == 0 && tid == 0) {
    StepState* st = a.st;
    if (a.finalize) {
      st->tok = argmax_key_index(__ldcg(&a.best2[(a.steps - 1) & 1]));
      st->pos = a.pos0 + a.steps;
    }
    if (a.record) st->count = a.count0 + a.steps;
  }
}

}  // namespace

size_t decode_mk_smem() { return sizeof(MkSmem) + 128; }

void launch_decode_mk_config() {
  static std::atomic<unsigned long long> done{0};
  once_per_device(done, [] {
    cudaFuncSetAttribute(decode_mk_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(decode_mk_smem()));
    cudaFuncSetAttribute(decode_mk_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(decode_mk_smem()));
    cudaFuncSetAttribute(decode_mk_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(decode_mk_smem()));
  });
}

cudaError_t launch_decode_mk(const MkArgs& a, int grid, cudaStream_t s) {
  launch_decode_mk_config();
  const size_t smem = decode_mk_smem();
  MkArgs copy = a;
  void* params[] = {&copy};
  static const int depth = [] {
    const char* e = std::getenv("ORX_MK_D");
    return e ? std::atoi(e) : 4;
  }();
  const void* fn = depth == 2 ? reinterpret_cast<const void*>(decode_mk_kernel<2>)
                 : depth == 3 ? reinterpret_cast<const void*>(decode_mk_kernel<3>)
                              : reinterpret_cast<const void*>(decode_mk_kernel<4>);
  return cudaLaunchCooperativeKernel(fn, dim3(grid),
                                     dim3(kT), params, smem, s);
}

int decode_mk_max_grid() {
  int dev = 0, sms = 0, per = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  launch_decode_mk_config();
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, decode_mk_kernel<4>, kT, decode_mk_smem());
  return (per >= 1 && sms * kMkOwnRows >= kHidden) ? sms : 0;
}

}  // namespace orx
