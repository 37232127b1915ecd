// C++ free operators of the B200 library with the reference's names and
// signatures: orator::model::asr_ops (include/model/asr_ops.cuh:22-62) and
// orator::model::asr_gemm (include/model/asr_gemm.h:22-41). Header-only over
// the C ABI in orx.h; device pointers, row-major, launched on `stream`
// (the reference's RopeInterleaved and GqaAttention take no stream and run on
// the legacy default stream; so do these). Errors become exceptions as in the
// reference: bad arguments -> std::runtime_error, CUDA failures ->
// orator::model::GpuError.
#pragma once

#include <cuda_runtime_api.h>

#include <cstdint>
#include <stdexcept>

#include "orx.h"

namespace orator {
namespace model {

#ifndef ORATOR_B200_GPU_ERROR_DEFINED
#define ORATOR_B200_GPU_ERROR_DEFINED
class GpuError : public std::runtime_error {
 public:
  using std::runtime_error::runtime_error;
};
#endif

namespace detail {
inline void OpCheck(int rc) {
  if (rc == ORX_OK) return;
  if (rc == ORX_ECUDA) throw GpuError(orx_last_error());
  throw std::runtime_error(orx_last_error());
}
}  // namespace detail

namespace asr_ops {

inline void RmsNorm(const float* x, const float* weight, float* out, int rows, int dim, float eps,
                    cudaStream_t stream = 0) {
  detail::OpCheck(orx_rms_norm(x, weight, out, rows, dim, eps, stream));
}
inline void RopeInterleaved(float* x, const int* positions, int n_tokens, int n_heads,
                            int head_dim, float theta_base) {
  detail::OpCheck(orx_rope_interleaved(x, positions, n_tokens, n_heads, head_dim, theta_base,
                                       nullptr));
}
inline void SwiGLU(const float* gate, const float* up, float* out, int n, cudaStream_t stream = 0) {
  detail::OpCheck(orx_swiglu(gate, up, out, n, stream));
}
inline void RopeHalf(float* x, const int* positions, int n_tokens, int n_heads, int head_dim,
                     float theta_base, cudaStream_t stream = 0) {
  detail::OpCheck(orx_rope_half(x, positions, n_tokens, n_heads, head_dim, theta_base, stream));
}
inline void GqaAttention(const float* q, const float* k, const float* v, float* out, int T, int Hq,
                         int Hkv, int Dh, float scale, bool causal) {
  detail::OpCheck(orx_gqa_attention(q, k, v, out, T, Hq, Hkv, Dh, scale, causal ? 1 : 0, nullptr));
}
inline void ArgmaxBanned(const float* logits, int n, int ban0, int ban1, int* out_idx,
                         cudaStream_t stream = 0) {
  detail::OpCheck(orx_argmax_banned(logits, n, ban0, ban1, out_idx, stream));
}

}  // namespace asr_ops

namespace asr_gemm {

inline void F32ToBf16(const float* in, uint16_t* out, long n, cudaStream_t stream = 0) {
  detail::OpCheck(orx_f32_to_bf16(in, out, n, stream));
}
inline void Bf16ToF32(const uint16_t* in, float* out, long n, cudaStream_t stream = 0) {
  detail::OpCheck(orx_bf16_to_f32(in, out, n, stream));
}
inline void Linear(const float* in_f32, const uint16_t* W_bf16, const float* bias_f32,
                   float* out_f32, int M, int K, int N, int act, cudaStream_t stream = 0) {
  detail::OpCheck(orx_linear(in_f32, W_bf16, bias_f32, out_f32, M, K, N, act, stream));
}
inline void LinearPre(const uint16_t* in_bf16, const uint16_t* W_bf16, const float* bias_f32,
                      float* out_f32, int M, int K, int N, int act, cudaStream_t stream = 0) {
  detail::OpCheck(orx_linear_pre(in_bf16, W_bf16, bias_f32, out_f32, M, K, N, act, stream));
}
// The reference frees its cuBLAS handle and cast scratch here; this library
// keeps a per-thread cast buffer that is released at thread exit.
inline void Shutdown() {}

}  // namespace asr_gemm
}  // namespace model
}  // namespace orator
