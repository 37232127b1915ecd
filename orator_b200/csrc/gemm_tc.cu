// tcgen05 / TMEM projection GEMM for prefill and batched decode (sm_100a).
//
//   out[t, n] (op)= sum_k X[t, k] * W[n, k]       X: [T, K] bf16, W: [N, K] bf16
//
// "Weight-stationary" orientation: the MMA's M side is 128 weight rows and its
// N side is a tile of BN tokens (16..256), so a batch of 64 decode tokens or
// a 400-row prefill both map onto full 128-row tcgen05 tiles. Each CTA owns
// one 128-row weight tile, one token tile and one K range (split-K for the
// short projections):
//   * warp 0 / one lane: TMA producer — 128x64 weight box and BNx64
//     activation box per stage (128-byte swizzle), mbarrier complete_tx;
//   * warp 1 / one lane: MMA issuer — 4 x tcgen05.mma (K = 16 each) per stage
//     into a TMEM accumulator of BN fp32 columns, tcgen05.commit releases the
//     stage;
//   * 8 epilogue warps (two per 32-lane TMEM quarter, one for the even and
//     one for the odd 32-column chunks): tcgen05.ld of their 32 TMEM lanes
//     (= 32 weight rows), then fp32 store, residual add, SwiGLU on
//     [64 gate | 64 up] tiles with the bf16 cast of the reference, or bias +
//     GELU / ReLU (Linear); with split K they write fp32 partials, summed in
//     split order by a reduction kernel (deterministic).
// Replaces Bf16WmmaKernel2 (include/model/gemm.cuh:394-459) and the
// F32ToBf16 / AddResidual / SwiGLU launches around it.
// No TMA multicast anywhere: every CTA loads its own tiles.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace orx {
namespace {

constexpr int kTcThreads = 128;
constexpr int kBK = 64;                  // K per stage (128 bytes of bf16)
constexpr int kATileB = 128 * kBK * 2;   // 16 KiB

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>(1) << 16;            // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;    // SBO: 8 rows x 128 B
  d |= static_cast<uint64_t>(1) << 46;            // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <int BN, int STAGES>
struct TcSmem {
  alignas(1024) uint8_t a[STAGES][kATileB];
  alignas(1024) uint8_t b[STAGES][BN * kBK * 2];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];   // MMA -> epilogue: accumulator buffer ready
  uint64_t acc_empty[2];  // epilogue -> MMA: accumulator buffer drained
  uint32_t tmem_base;
  // SwiGLU, per column half of the epilogue: up rows handed to the gate-row
  // threads, gate rows of columns 16-31 handed to the up-row threads
  float swap_up[2][64][33];
  float swap_gate[2][64][17];
};

// Persistent, warp-specialised GEMM. Work items (m tile, n tile, k split) are
// strided over the CTAs; warp 0 streams TMA stages continuously across items,
// warp 1 issues the MMAs into one of two TMEM accumulators, and warps 2-5 run
// the epilogue of item i while the MMAs of item i + 1 proceed.
constexpr int kTcWarps = 10;  // producer, MMA, 8 epilogue warps (two per TMEM lane quarter)
constexpr int kTcThreadsP = kTcWarps * 32;

template <int BN, int STAGES>
__global__ void __launch_bounds__(kTcThreadsP, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                   TcArgs g, int splits) {
  extern __shared__ uint8_t tc_raw[];
  TcSmem<BN, STAGES>& sm = *reinterpret_cast<TcSmem<BN, STAGES>*>(
      (reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (g.N + 127) / 128, nt = (g.T + BN - 1) / BN;
  const int items = mt * nt * splits;
  const int kper = g.K / splits, KT = (kper + kBK - 1) / kBK;
  // two accumulators of BN columns; the allocation is a power of two >= 32
  constexpr int kAccCols = BN < 32 ? 32 : BN;
  constexpr int kTmemCols = 2 * kAccCols <= 64 ? 64 : 2 * kAccCols <= 128 ? 128
                          : 2 * kAccCols <= 256 ? 256 : 512;
  int* err = g.err;

  if (warp == 0) {
    if (lane == 0) {
      for (int s = 0; s < STAGES; ++s) {
        mbar_init(&sm.full[s], 1);
        mbar_init(&sm.empty[s], 1);
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(&sm.acc_full[b], 1);
        mbar_init(&sm.acc_empty[b], 8);  // one arrival per epilogue warp
      }
      fence_mbar_init();
    }
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = sm.tmem_base;
  pdl_trigger();

  auto decode_item = [&](int it, int& m0, int& n0, int& kz) {
    kz = it % splits;
    const int r = it / splits;
    m0 = (r % mt) * 128;
    n0 = (r / mt) * BN;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer: stages of all of this CTA's items back to back ----
      // Weight tiles do not depend on the previous kernel, so the first
      // STAGES of them are issued before griddepcontrol.wait; the matching
      // activation tiles follow once the producer of X has finished.
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      const int my_items = blockIdx.x < items ? (items - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
      const int total = my_items * KT;
      const int pre = total < STAGES ? total : STAGES;
      auto coords = [&](int q, int& k, int& m0, int& n0) {
        const int j = q / KT, kt = q - j * KT;
        int kz;
        decode_item(blockIdx.x + j * gridDim.x, m0, n0, kz);
        k = kz * kper + kt * kBK;
      };
      for (int q = 0; q < pre; ++q) {
        int k, m0, n0;
        coords(q, k, m0, n0);
        mbar_arrive_expect_tx(&sm.full[q], kATileB + BN * kBK * 2);
        tma_load_2d(sm.a[q], &tmW, k, m0, &sm.full[q]);
      }
      pdl_wait();  // activations come from the previous kernel
      for (int q = 0; q < pre; ++q) {
        int k, m0, n0;
        coords(q, k, m0, n0);
        tma_load_2d(sm.b[q], &tmX, k, n0, &sm.full[q]);
      }
      for (int q = pre; q < total; ++q) {
        const int s = q % STAGES;
        if (!mbar_wait(&sm.empty[s], ((q / STAGES) - 1) & 1, err, 31)) break;
        int k, m0, n0;
        coords(q, k, m0, n0);
        mbar_arrive_expect_tx(&sm.full[s], kATileB + BN * kBK * 2);
        tma_load_2d(sm.a[s], &tmW, k, m0, &sm.full[s]);
        tma_load_2d(sm.b[s], &tmX, k, n0, &sm.full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) |
                                 (static_cast<uint32_t>(BN >> 3) << 17) | (8u << 24);
      int q = 0, j = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++j) {
        const int b = j & 1;
        if (j >= 2 && !mbar_wait(&sm.acc_empty[b], ((j >> 1) - 1) & 1, err, 34)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + b * kAccCols;
        for (int kt = 0; kt < KT; ++kt, ++q) {
          const int s = q % STAGES;
          if (!mbar_wait(&sm.full[s], (q / STAGES) & 1, err, 32)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t ad = umma_desc_sw128(smem_u32(sm.a[s]));
          const uint64_t bd = umma_desc_sw128(smem_u32(sm.b[s]));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)  // +32 bytes per K=16 step inside the atom
            umma_f16(acc, ad + 2 * kk, bd + 2 * kk, idesc, (kt | kk) != 0);
          umma_commit(&sm.empty[s]);
        }
        umma_commit(&sm.acc_full[b]);
      }
    }
  } else {
    // ---- epilogue warps 2..9: TMEM lane quarter = warp % 4; warps 2-5
    // drain the even 32-column chunks, warps 6-9 the odd ones ----
    pdl_wait();
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int bar_id = 1 + half;  // named barrier of this half's 128 threads
    int j = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x, ++j) {
      int m0, n0, kz;
      decode_item(it, m0, n0, kz);
      const int b = j & 1;
      mbar_wait(&sm.acc_full[b], (j >> 1) & 1, err, 33);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int rloc = quarter * 32 + lane;  // row within the 128-row tile
      const int row = m0 + rloc;
      const uint32_t tbase = tmem + b * kAccCols + (static_cast<uint32_t>(quarter * 32) << 16);
      // Output stage of 32 finished accumulator columns (tokens n0 + c0 ..).
      auto finish = [&](float* v, int c0) {
        if (g.epi == kEpiSwiglu) {
          // gate row j pairs with up row j + 64; the gate-row threads finish
          // columns 0-15 of the chunk, the up-row threads columns 16-31
          asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
          if (rloc >= 64) {
#pragma unroll
            for (int i = 0; i < 32; ++i) sm.swap_up[half][rloc - 64][i] = v[i];
          } else {
#pragma unroll
            for (int i = 16; i < 32; ++i) sm.swap_gate[half][rloc][i - 16] = v[i];
          }
          asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
          const int lim = min(min(32, BN - c0), g.T - (n0 + c0));
          const int jr = rloc & 63;
          uint16_t* po = g.out_bf16 + (long long)(n0 + c0) * g.ldo + (m0 >> 1) + jr;
          if (rloc < 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (i < lim) {
                const float gt = v[i], up = sm.swap_up[half][jr][i];
                po[(long long)i * g.ldo] = f2bf((gt / (1.0f + expf(-gt))) * up);
              }
          } else {
#pragma unroll
            for (int i = 16; i < 32; ++i)
              if (i < lim) {
                const float gt = sm.swap_gate[half][jr][i - 16], up = v[i];
                po[(long long)i * g.ldo] = f2bf((gt / (1.0f + expf(-gt))) * up);
              }
          }
        } else if (g.epi == kEpiLinear) {
          // Straight-line per mode: the activation and the output kind are
          // chosen once per 32-column chunk, stores are predicated.
          const int lim = min(min(32, BN - c0), g.T - (n0 + c0));
          if (row < g.N && lim > 0) {
            const float bv = g.bias ? g.bias[row] : 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] += bv;
            switch (g.act) {
              case 1:
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  v[i] = 0.5f * v[i] * (1.0f + erff(v[i] * 0.70710678118654752440f));
                break;
              case 2:
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.0f);
                break;
              case 3:
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = v[i] / (1.0f + expf(-v[i]));
                break;
              case 4:
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = 1.0f / (1.0f + expf(-v[i]));
                break;
              default:
                break;
            }
            const long long base = (long long)(n0 + c0) * g.ldo + row;
            if (g.out_bf16) {
              uint16_t* po = g.out_bf16 + base;
              if (g.split3) {  // [hi | hi | lo] operand of the next fp32-grade GEMM
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (i < lim) {
                    const uint16_t hi = f2bf(v[i]);
                    uint16_t* q = po + (long long)i * g.ldo;
                    q[0] = hi;
                    q[g.N] = hi;
                    q[2 * g.N] = f2bf(v[i] - bf2f(hi));
                  }
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (i < lim) po[(long long)i * g.ldo] = f2bf(v[i]);
              }
            } else {
              float* po = g.out_f32 + base;
              if (g.resid) {
                const float sc = g.resid == 2 ? 0.5f : 1.0f;
                float r[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) r[i] = i < lim ? po[(long long)i * g.ldo] : 0.f;
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (i < lim) po[(long long)i * g.ldo] = r[i] + sc * v[i];
              } else {
#pragma unroll
                for (int i = 0; i < 32; ++i)
                  if (i < lim) po[(long long)i * g.ldo] = v[i];
              }
            }
          }
        } else {
          float r[32];
          const int lim = min(min(32, BN - c0), g.T - (n0 + c0));
          float* po = g.out_f32 + (long long)(n0 + c0) * g.ldo + row;
          const bool rd = g.epi == kEpiResid;
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = (rd && i < lim) ? po[(long long)i * g.ldo] : 0.f;
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (i < lim) po[(long long)i * g.ldo] = r[i] + v[i];
        }
      };
      for (int c0 = half * 32; c0 < BN; c0 += 64) {
        float v[32];
        tmem_ld32(tbase + c0, v);
        if (splits > 1) {
          const int lim = min(min(32, BN - c0), g.T - (n0 + c0));
          float* pw = g.ws + ((long long)kz * g.T + n0 + c0) * g.N + row;
          if (row < g.N) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i < lim) pw[(long long)i * g.N] = v[i];
          }
        } else {
          finish(v, c0);
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                              CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                              CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeFn>(nullptr);
    return reinterpret_cast<EncodeFn>(p);
  }();
  return fn;
}

// 2-D bf16 map over a row-major [rows, K] matrix; box = 64 elements x box_rows,
// 128-byte swizzle (the canonical K-major layout of tcgen05 operands).
bool make_map(CUtensorMap* m, const void* base, long long rows, int K, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

__global__ void splitk_reduce_kernel(TcArgs g, int splits) {
  pdl_trigger();
  pdl_wait();
  const long long n = (long long)g.T * g.N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int z = 0; z < splits; ++z) acc += g.ws[z * n + i];
    const long long t = i / g.N, row = i % g.N;
    float* o = g.out_f32 + t * g.ldo + row;
    if (g.epi == kEpiResid) *o += acc; else *o = acc;
  }
}

// Split-K reduction of residual rows of 2048 fused with the RMSNorm that
// follows (one CTA per token row, 8 columns per thread): x += sum of the
// partials in split order, then xn = bf16(x * rsqrtf(mean(x^2) + eps) * w),
// the same operations in the same order as splitk_reduce_kernel followed by
// rmsnorm_bf16_kernel.
__global__ void __launch_bounds__(256) splitk_reduce_norm_kernel(TcArgs g, int splits) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  const int t = blockIdx.x, tid = threadIdx.x;
  const long long n = (long long)g.T * g.N;
  const long long off = (long long)t * g.N + tid * 8;
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int z = 0; z < splits; ++z) {
    const float4* p = reinterpret_cast<const float4*>(g.ws + z * n + off);
    const float4 p0 = p[0], p1 = p[1];
    a[0] += p0.x; a[1] += p0.y; a[2] += p0.z; a[3] += p0.w;
    a[4] += p1.x; a[5] += p1.y; a[6] += p1.z; a[7] += p1.w;
  }
  float4* xo = reinterpret_cast<float4*>(g.out_f32 + (long long)t * g.ldo + tid * 8);
  const float4 x0 = xo[0], x1 = xo[1];
  const float v[8] = {x0.x + a[0], x0.y + a[1], x0.z + a[2], x0.w + a[3],
                      x1.x + a[4], x1.y + a[5], x1.z + a[6], x1.w + a[7]};
  xo[0] = make_float4(v[0], v[1], v[2], v[3]);
  xo[1] = make_float4(v[4], v[5], v[6], v[7]);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float inv = rsqrtf(tot / kHidden + g.eps);
  const float4* wi = reinterpret_cast<const float4*>(g.norm_w) + tid * 2;
  const float4 w0 = wi[0], w1 = wi[1];
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  uint32_t pk[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    pk[j] = static_cast<uint32_t>(f2bf(v[2 * j] * inv * wv[2 * j])) |
            (static_cast<uint32_t>(f2bf(v[2 * j + 1] * inv * wv[2 * j + 1])) << 16);
  reinterpret_cast<uint4*>(g.norm_out + (long long)t * kHidden)[tid] =
      make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// Linear epilogue after split-K: y = act(sum of the partials in split order
// + bias), stored as in the GEMM epilogue (bf16, the split3 operand form, or
// fp32 with an optional residual add).
__global__ void splitk_linear_kernel(TcArgs g, int splits) {
  pdl_trigger();
  pdl_wait();
  const long long n = (long long)g.T * g.N;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int z = 0; z < splits; ++z) v += g.ws[z * n + i];
    const long long t = i / g.N;
    const int row = static_cast<int>(i % g.N);
    if (g.bias) v += g.bias[row];
    switch (g.act) {
      case 1: v = 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f)); break;
      case 2: v = fmaxf(v, 0.0f); break;
      case 3: v = v / (1.0f + expf(-v)); break;
      case 4: v = 1.0f / (1.0f + expf(-v)); break;
      default: break;
    }
    const long long o = t * g.ldo + row;
    if (g.out_bf16) {
      const uint16_t hi = f2bf(v);
      if (g.split3) {
        g.out_bf16[o] = hi;
        g.out_bf16[o + g.N] = hi;
        g.out_bf16[o + 2 * g.N] = f2bf(v - bf2f(hi));
      } else {
        g.out_bf16[o] = hi;
      }
    } else if (g.resid) {
      g.out_f32[o] += (g.resid == 2 ? 0.5f : 1.0f) * v;
    } else {
      g.out_f32[o] = v;
    }
  }
}

// SwiGLU after split-K: output j of token t pairs gate row (j/64)*128 + j%64
// with the up row 64 further in the same 128-row tile.
__global__ void splitk_swiglu_kernel(TcArgs g, int splits) {
  pdl_trigger();
  pdl_wait();
  const long long n = (long long)g.T * g.N, half = (long long)g.T * (g.N / 2);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < half;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / (g.N / 2);
    const int j = static_cast<int>(i % (g.N / 2));
    const long long gr = t * g.N + (j >> 6) * 128 + (j & 63);
    float gt = 0.f, up = 0.f;
    for (int z = 0; z < splits; ++z) {
      gt += g.ws[z * n + gr];
      up += g.ws[z * n + gr + 64];
    }
    g.out_bf16[t * g.ldo + j] = f2bf((gt / (1.0f + expf(-gt))) * up);
  }
}

template <int BN, int STAGES>
void launch_bn(const CUtensorMap& mw, const CUtensorMap& mx, const TcArgs& g, int splits,
               cudaStream_t s) {
  static std::atomic<unsigned long long> configured{0};
  static int sms_of[64];
  const size_t smem = sizeof(TcSmem<BN, STAGES>) + 1024;
  int dev = 0;
  cudaGetDevice(&dev);
  once_per_device(configured, [&] {
    cudaFuncSetAttribute(tc_gemm_kernel<BN, STAGES>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    cudaDeviceGetAttribute(&sms_of[dev & 63], cudaDevAttrMultiProcessorCount, dev);
  });
  const int sms = sms_of[dev & 63] > 0 ? sms_of[dev & 63] : 148;
  const int items = ((g.N + 127) / 128) * ((g.T + BN - 1) / BN) * splits;
  const int grid = items < sms ? items : sms;
  launch_pdl(tc_gemm_kernel<BN, STAGES>, dim3(grid), dim3(kTcThreadsP), smem, s, mw, mx, g,
             splits);
}

}  // namespace

bool tc_available() { return encode_fn() != nullptr; }

bool make_tmap_2d(void* map, const void* base, long long rows, int cols, int box_cols, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return fn(static_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
            const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int tc_sms() {
  static std::atomic<int> sms_of[64];  // per device, filled on first use
  int dev = 0;
  cudaGetDevice(&dev);
  int v = sms_of[dev & 63].load(std::memory_order_relaxed);
  if (v <= 0) {
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    sms_of[dev & 63].store(v, std::memory_order_relaxed);
  }
  return v > 0 ? v : 148;
}

// Token columns per tile. Up to 128 rows: the next power of two. Above, 144
// or 256, whichever finishes sooner on `sms` CTAs: rounds of (weight tile x
// token tile x split) items times the time of one k-block, the larger of the
// boxes at about 120 GB/s of L2-to-SM bandwidth and the tensor time (144
// balances 400-row prefills: 3 tiles of 144 instead of 256 + 144).
int tc_token_tile(int N, int T, int splits, int sms) {
  if (T <= 128 || sms <= 0) return T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : T <= 128 ? 128 : 256;
  auto cost = [&](int bn) {
    const long long items = (long long)((N + 127) / 128) * ((T + bn - 1) / bn) * splits;
    const double rounds = (double)((items + sms - 1) / sms);
    const double kb = std::max((16384.0 + bn * 128.0) / 120e9, 2.0 * 128 * bn * 64 / 10.8e12);
    return rounds * kb;
  };
  return cost(144) < cost(256) ? 144 : 256;
}

// Cost model as for the decoder projections (rounds x k-blocks x time per
// k-block + the reduction), with a floor of 0.45 us per k-block: the latency
// of one stage of a CTA's ring, measured on B200 for these small tiles.
int linear_plan(int N, int K, int T, int sms, int* bn_out) {
  int best_bn = 32, best_sp = 1;
  double best = 1e30;
  const int mt = (N + 127) / 128;
  for (int bn : {32, 64, 128, 256}) {
    if (bn > 32 && (bn >> 1) >= T) break;
    for (int sp : {1, 2, 3, 4, 6, 8}) {
      if (K % (64 * sp) != 0 || (sp > 1 && K / sp < 128)) continue;
      const long long items = (long long)mt * ((T + bn - 1) / bn) * sp;
      const int active = static_cast<int>(std::min<long long>(items, sms));
      const double rounds = (double)((items + sms - 1) / sms);
      const double kb = K / 64.0 / sp;
      const double w_bytes = 128.0 * 64 * 2, x_bytes = bn * 64 * 2.0;
      const double per_sm_hbm = std::min(6.4e12 / active, 55e9);
      const double t_unit = std::max({0.45e-6, w_bytes / per_sm_hbm, (w_bytes + x_bytes) / 120e9,
                                      2.0 * 128 * bn * 64 / 10.8e12});
      const double red = sp > 1 ? (sp * 8.0 * T * N) / 3e12 + 4e-6 : 0.0;
      const double c = rounds * kb * t_unit + red;
      if (c < best * 0.97) {  // prefer the earlier (simpler) plan on near ties
        best = c;
        best_bn = bn;
        best_sp = sp;
      }
    }
  }
  *bn_out = best_bn;
  return best_sp;
}

void launch_gemm_tc(const uint16_t* X, const uint16_t* W, const TcArgs& g, int splits,
                    cudaStream_t s) {
  if (g.T <= 0) return;
  int bn = g.epi == kEpiLinear ? tc_token_tile(g.N, g.T, splits, 0) : tc_token_tile(g.N, g.T, splits, tc_sms());
  if (g.bn_hint > 0) {
    bn = g.bn_hint;
  } else if (g.epi == kEpiLinear && splits == 1) {
    // No split-K here: narrower token tiles until the tiles cover most SMs
    // (the weight tile is then re-read from L2 by more CTAs).
    const int mt = (g.N + 127) / 128;
    while (bn > 32 && mt * ((g.T + bn - 1) / bn) < 111) bn >>= 1;
  }
  CUtensorMap mw, mx;
  if (!make_map(&mw, W, g.N, g.K, 128) || !make_map(&mx, X, g.T, g.K, bn)) {
    fprintf(stderr, "orx: tensor map encoding failed\n");
    return;
  }
  switch (bn) {
    case 16: launch_bn<16, 8>(mw, mx, g, splits, s); break;
    case 32: launch_bn<32, 8>(mw, mx, g, splits, s); break;
    case 64: launch_bn<64, 8>(mw, mx, g, splits, s); break;
    case 128: launch_bn<128, 6>(mw, mx, g, splits, s); break;
    case 144: launch_bn<144, 5>(mw, mx, g, splits, s); break;
    default: launch_bn<256, 4>(mw, mx, g, splits, s); break;
  }
  const bool norm = g.norm_w != nullptr;
  if (norm && (g.N != kHidden || g.ldo != kHidden || g.epi != kEpiResid)) {
    fprintf(stderr, "orx: fused RMSNorm needs residual rows of 2048\n");
    return;
  }
  if (splits > 1) {
    const long long n = (long long)g.T * g.N;
    const int grid = static_cast<int>(std::min<long long>((n + 255) / 256, 148 * 16));
    if (g.epi == kEpiSwiglu)
      launch_pdl(splitk_swiglu_kernel, dim3(grid), dim3(256), 0, s, g, splits);
    else if (g.epi == kEpiLinear)
      launch_pdl(splitk_linear_kernel, dim3(grid), dim3(256), 0, s, g, splits);
    else if (norm)
      launch_pdl(splitk_reduce_norm_kernel, dim3(g.T), dim3(256), 0, s, g, splits);
    else
      launch_pdl(splitk_reduce_kernel, dim3(grid), dim3(256), 0, s, g, splits);
  } else if (norm) {
    launch_rmsnorm_bf16(g.out_f32, g.norm_w, g.norm_out, g.T, g.eps, s);
  }
}

}  // namespace orx
