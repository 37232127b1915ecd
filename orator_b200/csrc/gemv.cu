// Weight-streaming GEMV for batch-1 decode on sm_100a.
//
// Replaces the reference's F32ToBf16 -> GemvBf16Vec4Kernel -> (SwiGLU |
// AddResidual | ArgmaxBanned) launch chains (src/model/asr_gemm.cu:109-215,
// src/model/asr_text_decoder.cu:404-438, src/model/asr_ops.cu:199-333) with a
// single kernel per projection:
//
//  * one CTA per SM, 8 warps; every warp streams its own 4 KiB weight chunks
//    (2048 bf16 of one row) with 1-D bulk async copies (TMA engine) into its
//    own kDepth-slot shared ring guarded by mbarriers, so no warp waits on
//    another's progress;
//  * the first kDepth chunks of every warp are issued BEFORE
//    griddepcontrol.wait: weights never depend on the previous kernel, so
//    under programmatic dependent launch the next projection's weights are in
//    flight while the previous kernel finishes;
//  * the warps then build the bf16 activation in shared memory (fused RMSNorm
//    or embedding gather + RMSNorm, with the reference's bf16 rounding point)
//    and reduce whole rows: fp32 FMA over bf16 operands, warp shuffle
//    reduction;
//  * fused epilogues: fp32 store, residual add, SwiGLU + bf16 cast, or logits
//    with a fused banned argmax (per-CTA best -> 64-bit atomicMax -> last CTA
//    publishes the token and advances the position).
#include <cstdlib>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace orx {
namespace {

constexpr int kChunk = 2048;             // bf16 elements per ring slot
constexpr int kChunkBytes = kChunk * 2;  // 4 KiB
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreadsGemv = kConsumers;
constexpr int kMaxK = kInter;  // 6144

template <int kDepth>
struct GemvSmem {
  static constexpr int kSlots = kConsumerWarps * kDepth;
  alignas(128) uint8_t ring[kSlots][kChunkBytes];
  alignas(16) uint16_t xs[kMaxK];
  uint64_t full[kSlots];
  float red[kConsumerWarps];
  unsigned long long best[kConsumerWarps];
  int last;
};

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

// Row of weight matrix holding output `r` of unit `u` (SwiGLU units pair the
// gate and up rows of a 128-row tile: [64 gate | 64 up]).
__device__ __forceinline__ long long unit_row(int epi, int u, int r) {
  if (epi == kEpiSwiglu) return (long long)(u >> 6) * 128 + (u & 63) + r * 64;
  return u;
}

template <int kDepth>
__global__ void __launch_bounds__(kThreadsGemv, 2) gemv_kernel(GemvArgs a) {
  extern __shared__ uint8_t smem_raw[];
  GemvSmem<kDepth>& sm = *reinterpret_cast<GemvSmem<kDepth>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int G = gridDim.x;
  trace_mark(a.trace, 0);
  const long long u0 = (long long)blockIdx.x * a.units / G;
  const long long u1 = (long long)(blockIdx.x + 1) * a.units / G;
  const int my_units = static_cast<int>(u1 - u0);
  const int rpu = (a.epi == kEpiSwiglu) ? 2 : 1;
  const int cpr = a.K / kChunk;
  const int cpu = rpu * cpr;
  int* err = a.st ? &a.st->err : nullptr;
  // This warp's chunk sequence: units warp, warp+8, ...; per unit its rows
  // and K-chunks in order.
  const int my_w_units = my_units > warp ? (my_units - warp + kConsumerWarps - 1) / kConsumerWarps : 0;
  const int n_w = my_w_units * cpu;
  uint64_t* full = &sm.full[warp * kDepth];
  uint8_t(*ring)[kChunkBytes] = &sm.ring[warp * kDepth];
  auto issue = [&](int j) {
    const int lu = warp + (j / cpu) * kConsumerWarps, rem = j % cpu;
    const int r = rem / cpr, c = rem % cpr;
    const long long row = unit_row(a.epi, static_cast<int>(u0) + lu, r);
    const int slot = j % kDepth;
    mbar_arrive_expect_tx(&full[slot], kChunkBytes);
    bulk_g2s(ring[slot], a.W + row * a.K + (long long)c * kChunk, kChunkBytes, &full[slot]);
  };

  if (lane == 0) {
    for (int i = 0; i < kDepth; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
    for (int j = 0; j < kDepth && j < n_w; ++j) issue(j);
  }
  __syncwarp();
  pdl_trigger();

  pdl_wait();
  trace_mark(a.trace, 1);
  if (a.act_mode == kActBf16) {
    const uint4* src = reinterpret_cast<const uint4*>(a.act);
    uint4* dst = reinterpret_cast<uint4*>(sm.xs);
    for (int i = tid; i < a.K / 8; i += kConsumers) dst[i] = src[i];
  } else {
    // RMSNorm of one fp32 row of 2048 (8 elements per thread).
    float v[8];
    if (a.act_mode == kActEmbedNorm) {
      const int tok = *a.tok_ptr;
      const uint4 w = reinterpret_cast<const uint4*>(a.embed + (long long)tok * kHidden)[tid];
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = bf_lo(ww[j]);
        v[2 * j + 1] = bf_hi(ww[j]);
      }
      if (blockIdx.x == 0) {
        float4* xo = reinterpret_cast<float4*>(a.x_init) + tid * 2;
        xo[0] = make_float4(v[0], v[1], v[2], v[3]);
        xo[1] = make_float4(v[4], v[5], v[6], v[7]);
        if (tid == 0 && a.record && a.st) {
          StepState* st = a.st;
          if (st->count < st->out_cap) st->out[st->count] = tok;
          st->count = st->count + 1;
        }
      }
    } else {
      const float4* xi = reinterpret_cast<const float4*>(a.x) + tid * 2;
      const float4 p0 = xi[0], p1 = xi[1];
      v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w;
      v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
    ss = warp_sum(ss);
    if (lane == 0) sm.red[warp] = ss;
    consumer_sync();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) tot += sm.red[w];
    const float inv = rsqrtf(tot / kHidden + a.eps);
    const float4* nw = reinterpret_cast<const float4*>(a.norm_w) + tid * 2;
    const float4 w0 = nw[0], w1 = nw[1];
    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    uint32_t packed[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = f2bf(v[2 * j] * inv * wv[2 * j]);
      const uint32_t hi = f2bf(v[2 * j + 1] * inv * wv[2 * j + 1]);
      packed[j] = lo | (hi << 16);
    }
    reinterpret_cast<uint4*>(sm.xs)[tid] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
  }
  consumer_sync();

  bool ban = false;
  int ban0 = -1, ban1 = -1;
  if (a.epi == kEpiLogits && a.st) {
    ban = a.st->count < a.st->ban_steps;
    ban0 = ban ? a.st->ban0 : -1;
    ban1 = ban ? a.st->ban1 : -1;
  }
  unsigned long long best = 0ull;

  int jw = 0;  // chunks this warp has consumed
  for (int lu = warp; lu < my_units; lu += kConsumerWarps) {
    float accs[2] = {0.f, 0.f};
    for (int r = 0; r < rpu; ++r) {
      float acc4[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = 0; c < cpr; ++c) {
        const int slot = jw % kDepth;
        mbar_wait(&full[slot], (jw / kDepth) & 1, err, 13);
        const uint4* wp = reinterpret_cast<const uint4*>(ring[slot]);
        const uint4* xp = reinterpret_cast<const uint4*>(sm.xs + c * kChunk);
        uint4 wv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) wv[j] = wp[j * 32 + lane];
        __syncwarp();
        // the slot is free again: refill it with this warp's chunk jw + kDepth
        if (lane == 0 && jw + kDepth < n_w) {
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          issue(jw + kDepth);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 w = wv[j];
          const uint4 x = xp[j * 32 + lane];
          float& acc = acc4[j & 3];
          acc = fma2_bf16(w.x, x.x, acc);
          acc = fma2_bf16(w.y, x.y, acc);
          acc = fma2_bf16(w.z, x.z, acc);
          acc = fma2_bf16(w.w, x.w, acc);
        }
        ++jw;
      }
      const float acc = (acc4[0] + acc4[1]) + (acc4[2] + acc4[3]);
      accs[r] = warp_sum(acc);
    }
    if (lane == 0) {
      const int u = static_cast<int>(u0) + lu;
      switch (a.epi) {
        case kEpiStore: a.out_f32[u] = accs[0]; break;
        case kEpiResid: a.out_f32[u] += accs[0]; break;
        case kEpiSwiglu: {
          const float g = accs[0], up = accs[1];
          a.out_bf16[u] = f2bf((g / (1.0f + expf(-g))) * up);
          break;
        }
        case kEpiLogits: {
          a.out_f32[u] = accs[0];
          if (u != ban0 && u != ban1 && !(accs[0] != accs[0])) {
            const unsigned long long k = argmax_key(accs[0], u);
            best = k > best ? k : best;
          }
          break;
        }
      }
    }
  }

  if (a.trace) {
    __syncthreads();
    trace_mark(a.trace, 2);
  }
  if (a.epi == kEpiLogits && a.st) {
    if (lane == 0) sm.best[warp] = best;
    consumer_sync();
    if (tid == 0) {
      unsigned long long b = 0;
      for (int w = 0; w < kConsumerWarps; ++w) b = sm.best[w] > b ? sm.best[w] : b;
      if (b) atomicMax(&a.st->best, b);
      __threadfence();
      const int ticket = atomicAdd(&a.st->done, 1);
      if (ticket == G - 1) {
        __threadfence();
        StepState* st = a.st;
        const unsigned long long fin = atomicExch(&st->best, 0ull);
        st->done = 0;
        if (a.finalize) {
          st->tok = argmax_key_index(fin);
          st->pos = st->pos + 1;
        }
      }
    }
  }
}


template <int D>
void launch_depth(const GemvArgs& a, int grid, cudaStream_t s) {
  static std::atomic<unsigned long long> configured{0};
  const size_t smem = sizeof(GemvSmem<D>) + 128;
  once_per_device(configured, [&] {
    cudaFuncSetAttribute(gemv_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
  });
  launch_pdl(gemv_kernel<D>, dim3(grid), dim3(kThreadsGemv), smem, s, a);
}

// Ring depth per warp: deeper rings keep more bytes in flight per SM (better
// for long streams) but stop two GEMV CTAs from sharing an SM (less
// prologue overlap under programmatic dependent launch).
int depth_for(const GemvArgs& a) {
  static const int layer_depth = [] {
    const char* v = std::getenv("ORX_GEMV_DEPTH");
    return v ? std::atoi(v) : 3;
  }();
  static const int head_depth = [] {
    const char* v = std::getenv("ORX_GEMV_HEAD_DEPTH");
    return v ? std::atoi(v) : 6;
  }();
  return a.epi == kEpiLogits ? head_depth : layer_depth;
}

}  // namespace

void launch_gemv(const GemvArgs& a, int num_sms, cudaStream_t s) {
  const int grid = a.units < num_sms ? a.units : num_sms;
  switch (depth_for(a)) {
    case 2: launch_depth<2>(a, grid, s); break;
    case 4: launch_depth<4>(a, grid, s); break;
    case 5: launch_depth<5>(a, grid, s); break;
    case 6: launch_depth<6>(a, grid, s); break;
    default: launch_depth<3>(a, grid, s); break;
  }
}

}  // namespace orx
