// Allocation-free banned argmax over fp32 logits.
//
// Some callers cannot call cudaMalloc at all: code running inside a CUDA
// stream capture they do not own, real-time audio threads that must not take
// the driver's allocation locks, or hosts whose memory is fully reserved by
// another framework's caching allocator. For them this file provides one entry
// point that needs no device memory beyond the caller's inputs and outputs:
// its scratch lives in a fixed file-scope __device__ array that every GPU
// loading this library holds until process exit.
//
// The scratch holds one 64-bit partial result per CTA plus a CTA ticket, so
// the logits count is bounded by kNoAllocMaxCtas * kNoAllocPerCta.
#include <cstdint>
#include <mutex>

#include "../../include/orx.h"
#include "common.cuh"

namespace orx {
void set_last_error(const char* msg);
namespace {

constexpr int kNoAllocThreads = 256;
constexpr int kNoAllocPerCta = 8192;   // logits scanned per CTA
constexpr int kNoAllocMaxCtas = 1024;  // => at most 8,388,608 logits
constexpr int kNoAllocMaxDevices = 64;

// [0, kNoAllocMaxCtas): per-CTA packed (value, index) maxima; [kNoAllocMaxCtas]:
// CTA ticket. 8,200 bytes. Host code must not take this symbol's address as a
// device pointer: it is a host-side stand-in; the device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned long long g_noalloc_scratch[kNoAllocMaxCtas + 1];

__global__ void __launch_bounds__(kNoAllocThreads) argmax_noalloc_kernel(
    const float* __restrict__ x, int n, int ban0, int ban1, unsigned long long* scratch,
    int* out) {
  __shared__ unsigned long long sb[kNoAllocThreads / 32];
  __shared__ bool last;
  const int base = blockIdx.x * kNoAllocPerCta;
  const int end = base + kNoAllocPerCta < n ? base + kNoAllocPerCta : n;
  unsigned long long best = 0ull;
  for (int i = base + threadIdx.x; i < end; i += kNoAllocThreads) {
    if (i == ban0 || i == ban1) continue;
    const float v = x[i];
    if (v != v) continue;
    const unsigned long long k = argmax_key(v, i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, best, o);
    best = ob > best ? ob : best;
  }
  if ((threadIdx.x & 31) == 0) sb[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0;
    for (int w = 0; w < kNoAllocThreads / 32; ++w) b = sb[w] > b ? sb[w] : b;
    scratch[blockIdx.x] = b;
    __threadfence();
    last = atomicAdd(&scratch[kNoAllocMaxCtas], 1ull) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // The last CTA reduces the partials: each thread a strided subset, then the
  // same shuffle / shared-memory tree.
  unsigned long long b = 0;
  for (int i = threadIdx.x; i < static_cast<int>(gridDim.x); i += kNoAllocThreads) {
    const unsigned long long k = __ldcg(&scratch[i]);
    b = k > b ? k : b;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long ob = __shfl_xor_sync(0xffffffffu, b, o);
    b = ob > b ? ob : b;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) sb[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long fin = 0;
    for (int w = 0; w < kNoAllocThreads / 32; ++w) fin = sb[w] > fin ? sb[w] : fin;
    *out = fin ? argmax_key_index(fin) : 0;
    scratch[kNoAllocMaxCtas] = 0ull;  // ticket back to zero for the next call
  }
}

std::mutex g_mu;
unsigned long long* g_dev_ptr[kNoAllocMaxDevices] = {};

}  // namespace
}  // namespace orx

extern "C" int orx_argmax_banned_noalloc(const float* d_logits, int n, int ban0, int ban1,
                                         int* d_out, void* stream) {
  using namespace orx;
  if (!d_logits || !d_out) {
    set_last_error("orx_argmax_banned_noalloc: null logits or output pointer");
    return ORX_EINVAL;
  }
  if (n <= 0 || n > kNoAllocMaxCtas * kNoAllocPerCta) {
    set_last_error("orx_argmax_banned_noalloc: n must be in [1, 8388608] (fixed scratch size)");
    return ORX_EINVAL;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) {
    set_last_error("orx_argmax_banned_noalloc: no usable current device");
    return ORX_ECUDA;
  }
  unsigned long long* scratch;
  {
    // First call on this device (with it current): resolve the array's
    // device address. The host-side name is not usable as a device pointer.
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_dev_ptr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
        set_last_error("orx_argmax_banned_noalloc: cudaGetSymbolAddress failed");
        return ORX_ECUDA;
      }
      g_dev_ptr[dev] = static_cast<unsigned long long*>(p);
    }
    scratch = g_dev_ptr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Only the ticket must start at zero; partials are overwritten every call.
  if (cudaMemsetAsync(scratch + kNoAllocMaxCtas, 0, sizeof(unsigned long long), s) != cudaSuccess) {
    set_last_error("orx_argmax_banned_noalloc: clearing the scratch ticket failed");
    return ORX_ECUDA;
  }
  const int grid = (n + kNoAllocPerCta - 1) / kNoAllocPerCta;
  argmax_noalloc_kernel<<<grid, kNoAllocThreads, 0, s>>>(d_logits, n, ban0, ban1, scratch, d_out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_error(cudaGetErrorString(e));
    return ORX_ECUDA;
  }
  return ORX_OK;
}
