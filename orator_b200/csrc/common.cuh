// Shared constants and sm_100a device helpers for the Qwen3-ASR decoder path.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace orx {

// Qwen3-ASR-1.7B text decoder dimensions (AsrTextConfig defaults,
// include/model/asr_text_decoder.h:30-43 of the reference). The layer count,
// vocabulary and maximum sequence length stay runtime parameters.
constexpr int kHidden = 2048;
constexpr int kQHeads = 16;
constexpr int kKvHeads = 8;
constexpr int kHeadDim = 128;
constexpr int kQDim = kQHeads * kHeadDim;    // 2048
constexpr int kKvDim = kKvHeads * kHeadDim;  // 1024
constexpr int kQkvDim = kQDim + 2 * kKvDim;  // 4096
constexpr int kInter = 6144;
constexpr int kPage = 16;                    // tokens per KV page
constexpr int kGroup = kQHeads / kKvHeads;   // q heads per kv head
// One KV page of one layer: [K|V][kv head][16 tokens][128] bf16 = 64 KiB.
constexpr int kPageElems = 2 * kKvHeads * kPage * kHeadDim;
constexpr int kHalfPageElems = kKvHeads * kPage * kHeadDim;

// Error codes written to the device status word (never a trap).
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitTimeout = 1,
  kErrBadIndex = 2,
};

// Bounded waits: give up after this many nanoseconds of the global timer.
constexpr unsigned long long kWaitLimitNs = 200ull * 1000 * 1000;

__device__ __forceinline__ float bf2f(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// acc += lo(a)*lo(b) + hi(a)*hi(b) for packed bf16 pairs, with the mixed
// precision FMA (bf16 operands, fp32 accumulate; each product exact in fp32,
// one rounding per FMA, the same arithmetic as fmaf on upcast operands).
__device__ __forceinline__ float fma2_bf16(uint32_t a, uint32_t b, float acc) {
  asm("{\n .reg .b16 al, ah, bl, bh;\n mov.b32 {al, ah}, %1;\n mov.b32 {bl, bh}, %2;\n"
      " fma.rn.f32.bf16 %0, al, bl, %0;\n fma.rn.f32.bf16 %0, ah, bh, %0;\n}"
      : "+f"(acc)
      : "r"(a), "r"(b));
  return acc;
}

// Banned argmax with the tie rule of the reference's single-block
// ArgmaxBannedKernel (src/model/asr_ops.cu:300-325), packed into one monotone
// 64-bit key so that any reduction order (warp shuffles, CTA partials,
// atomicMax across CTAs) yields the same winner as that kernel:
//  * thread t of its 256 scans i = t, t + 256, ... and keeps the first strict
//    maximum above its -1e30 start, so values <= -1e30 (and NaN) never win and
//    an all-excluded input returns index 0 (key 0 here);
//  * its shared-memory tree pairs slot t with t + s for s = 128, 64, ..., 1 and
//    takes the upper slot only when strictly greater, so among equal maxima
//    the slot whose bit-reversed 8-bit number is smallest wins (bit 0 of the
//    slot decides first, then bit 1, ...), and inside a slot the lowest i.
// Key: orderable(value) << 32 | (255 - brev8(i & 255)) << 24 | (2^24 - 1 - (i >> 8)).
// -0.0 is folded into +0.0 (the reference's `>` treats them as equal).
__host__ __device__ __forceinline__ uint32_t brev8(uint32_t x) {
  x = ((x & 0xF0u) >> 4) | ((x & 0x0Fu) << 4);
  x = ((x & 0xCCu) >> 2) | ((x & 0x33u) << 2);
  x = ((x & 0xAAu) >> 1) | ((x & 0x55u) << 1);
  return x;
}
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  if (!(v > -1e30f)) return 0ull;
  uint32_t u = v == 0.0f ? 0u : __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  const uint32_t i = static_cast<uint32_t>(idx);
  const uint32_t lo = ((255u - brev8(i & 255u)) << 24) | (0xFFFFFFu - (i >> 8));
  return (static_cast<unsigned long long>(u) << 32) | lo;
}
// Index of a key; key 0 (nothing eligible) is index 0, as in the reference.
__host__ __device__ __forceinline__ int argmax_key_index(unsigned long long k) {
  if (k == 0ull) return 0;
  const uint32_t lo = static_cast<uint32_t>(k & 0xFFFFFFFFull);
  const uint32_t slot = brev8(255u - (lo >> 24));
  const uint32_t hi = 0xFFFFFFu - (lo & 0xFFFFFFu);
  return static_cast<int>(hi * 256u + slot);
}

// ---- programmatic dependent launch ---------------------------------------
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- mbarrier + bulk async copy (TMA engine, no tensor map) ---------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Debug timeline: slot[0] = earliest CTA start, slot[1] = latest CTA past
// griddepcontrol.wait, slot[2] = latest CTA end (global timer, ns).
__device__ __forceinline__ void trace_mark(unsigned long long* slot, int k) {
  if (slot && threadIdx.x == 0) {
    const unsigned long long t = global_ns();
    if (k == 0) atomicMin(slot, t); else atomicMax(slot + k, t);
  }
}

// Bounded wait: returns false after kWaitLimitNs, or at once when another
// wait already failed (*err != 0), recording `site` in *err. No trap.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err,
                                          int site = kErrWaitTimeout) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 0) {
      if (err && *reinterpret_cast<volatile int*>(err) != 0) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        if (err) atomicExch(err, site);
        return false;
      }
    }
  }
}
// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v += __shfl_xor_sync(0xffffffffu, v, m);
  return v;
}
// Sums two per-lane values over the warp at once: lanes 0-15 end with the
// sum of `a`, lanes 16-31 with the sum of `b`. Lane 0's addition tree is the
// one warp_sum uses (xor 16, 8, 4, 2, 1).
__device__ __forceinline__ float reduce_pair(float a, float b, int lane) {
  const bool hi = (lane & 16) != 0;
  float keep = hi ? b : a;
  keep += __shfl_xor_sync(0xffffffffu, hi ? a : b, 16);
#pragma unroll
  for (int m = 8; m > 0; m >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, m);
  return keep;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// ---- tensor-core and TMA helpers shared by the attention kernels ----------
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

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y,
                                       uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Byte offset of element (r, c) of a staged 16 x 128 bf16 tile: two 16 x 64
// halves, each in the 128-byte TMA swizzle (16-byte chunk ^ row % 8).
__device__ __forceinline__ int sw_off(int r, int c) {
  return (c >> 6) * 2048 + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2;
}

}  // namespace orx
