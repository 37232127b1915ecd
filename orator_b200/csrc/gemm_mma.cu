// Prefill / batched projection GEMM, out = A[M,K] * W[N,K]^T, bf16 operands
// with fp32 accumulation and fused epilogues (store, residual add, SwiGLU +
// bf16 cast).  Replaces the reference's Bf16WmmaKernel2 + F32ToBf16 /
// AddResidual / SwiGLU chain (include/model/gemm.cuh:394-459,
// src/model/asr_text_decoder.cu:518-555).
//
// Baseline tensor-core path (mma.sync m16n8k16 + ldmatrix + 3-stage cp.async);
// the tcgen05 path in gemm_tc.cu is preferred where it applies.
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace orx {
namespace {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
constexpr int kGemmThreads = 256;
constexpr int kTileBytes = BM * BK * 2;  // 8 KiB per operand per stage
constexpr int kCPad = BN + 4;
constexpr int kGemmSmem =
    (STAGES * 2 * kTileBytes > BM * kCPad * 4) ? STAGES * 2 * kTileBytes : BM * kCPad * 4;

__device__ __forceinline__ int swz(int row, int chunk) {
  return row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(kGemmThreads) gemm_mma_kernel(GemmArgs g) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int wm = warp >> 2, wn = warp & 3;  // 2 x 4 warps, warp tile 64 x 32
  const uint32_t sbase = smem_u32(smem);
  pdl_trigger();
  pdl_wait();

  auto load_stage = [&](int st, int k0) {
    const uint32_t sa = sbase + st * 2 * kTileBytes, sb = sa + kTileBytes;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = tid + i * kGemmThreads;  // 0..511
      const int row = c >> 2, ch = c & 3;
      const bool pa = (m0 + row) < g.M;
      const uint16_t* srcA = g.A + (long long)(pa ? m0 + row : 0) * g.K + k0 + ch * 8;
      cp_async16(sa + swz(row, ch), srcA, pa);
      const uint16_t* srcB = g.W + (long long)(n0 + row) * g.K + k0 + ch * 8;
      cp_async16(sb + swz(row, ch), srcB, true);
    }
  };

  float acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[i][j][k] = 0.f;

  const int KT = g.K / BK;
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < KT) load_stage(s, s * BK);
    cp_commit();
  }
  for (int kt = 0; kt < KT; ++kt) {
    cp_wait<STAGES - 2>();
    __syncthreads();
    const int nk = kt + STAGES - 1;
    if (nk < KT) load_stage(nk % STAGES, nk * BK);
    cp_commit();
    const int st = kt % STAGES;
    const uint32_t sa = sbase + st * 2 * kTileBytes, sb = sa + kTileBytes;
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t af[4][4], bfr[4][2];
#pragma unroll
      for (int mi = 0; mi < 4; ++mi) {
        const int row = wm * 64 + mi * 16 + (lane & 15);
        const int ch = kk * 2 + (lane >> 4);
        ldsm_x4(sa + swz(row, ch), af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
      }
#pragma unroll
      for (int nj = 0; nj < 2; ++nj) {
        const int row = wn * 32 + nj * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int ch = kk * 2 + ((lane >> 3) & 1);
        ldsm_x4(sb + swz(row, ch), bfr[2 * nj][0], bfr[2 * nj][1], bfr[2 * nj + 1][0],
                bfr[2 * nj + 1][1]);
      }
#pragma unroll
      for (int mi = 0; mi < 4; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) mma16816(acc[mi][ni], af[mi], bfr[ni][0], bfr[ni][1]);
    }
  }
  cp_wait<0>();
  __syncthreads();

  float* cs = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int mi = 0; mi < 4; ++mi)
#pragma unroll
    for (int ni = 0; ni < 4; ++ni) {
      const int r = wm * 64 + mi * 16 + (lane >> 2);
      const int c = wn * 32 + ni * 8 + (lane & 3) * 2;
      cs[r * kCPad + c] = acc[mi][ni][0];
      cs[r * kCPad + c + 1] = acc[mi][ni][1];
      cs[(r + 8) * kCPad + c] = acc[mi][ni][2];
      cs[(r + 8) * kCPad + c + 1] = acc[mi][ni][3];
    }
  __syncthreads();
  if (g.epi == kEpiSwiglu) {
    for (int i = tid; i < BM * 64; i += kGemmThreads) {
      const int r = i >> 6, c = i & 63;
      if (m0 + r >= g.M) continue;
      const float gt = cs[r * kCPad + c], up = cs[r * kCPad + c + 64];
      g.out_bf16[(long long)(m0 + r) * g.ldo + (n0 >> 1) + c] =
          f2bf((gt / (1.0f + expf(-gt))) * up);
    }
  } else {
    for (int i = tid; i < BM * BN; i += kGemmThreads) {
      const int r = i >> 7, c = i & 127;
      if (m0 + r >= g.M) continue;
      float* o = g.out_f32 + (long long)(m0 + r) * g.ldo + n0 + c;
      if (g.epi == kEpiResid)
        *o += cs[r * kCPad + c];
      else
        *o = cs[r * kCPad + c];
    }
  }
}

}  // namespace

void launch_gemm(const GemmArgs& a, cudaStream_t s) {
  if (a.M <= 0) return;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(gemm_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kGemmSmem);
    configured = true;
  }
  launch_pdl(gemm_mma_kernel, dim3(a.N / BN, (a.M + BM - 1) / BM), dim3(kGemmThreads),
             kGemmSmem, s, a);
}

}  // namespace orx
