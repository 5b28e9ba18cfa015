// Allocation-free sum of squares (see noalloc.h for the contract, the limit and
// who it is for).  This entry point has no counterpart in the TempName-5090
// reference.
#include "noalloc.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <mutex>

namespace {
constexpr int kThreads = 256;
constexpr int kVecPerThread = 8;                                  // 8 x 8 elements per thread
constexpr int64_t kChunk = int64_t(kThreads) * kVecPerThread * 8;  // 16384 elements per partial
constexpr int kMaxParts = 16384;                                  // 128 KiB of doubles
constexpr int kMaxDevices = 64;

// The scratch: one partial per 16384-element chunk, shared by all calls.
static __device__ __align__(256) double g_sqsum_scratch[kMaxParts];

std::mutex g_setup_mutex;
double* g_scratch_addr[kMaxDevices] = {nullptr};

template <typename T>
__device__ __forceinline__ void load8(const T* p, float* v);
template <>
__device__ __forceinline__ void load8<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
}
template <>
__device__ __forceinline__ void load8<float>(const float* p, float* v) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Block b sums chunk b (fixed assignment) and writes partial[b].
template <typename T>
__global__ void __launch_bounds__(kThreads) chunk_sqsum(const T* g, int64_t n, double* partial) {
  __shared__ double warp_sums[kThreads / 32];
  const int64_t base = int64_t(blockIdx.x) * kChunk;
  double acc = 0.0;
#pragma unroll
  for (int j = 0; j < kVecPerThread; ++j) {
    const int64_t i = base + (int64_t(j) * kThreads + threadIdx.x) * 8;
    if (i < n) {
      float v[8];
      load8<T>(g + i, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc += double(v[k] * v[k]);
    }
  }
#pragma unroll
  for (int d = 16; d; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) s += warp_sums[w];
    partial[blockIdx.x] = s;
  }
}

// One block: thread t sums partials t, t+256, ... in order; then a fixed-order combine.
__global__ void __launch_bounds__(kThreads) finish_sqsum(const double* partial, int parts, double* out) {
  __shared__ double sums[kThreads];
  double s = 0.0;
  for (int p = threadIdx.x; p < parts; p += kThreads) s += partial[p];
  sums[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int i = 0; i < kThreads; ++i) t += sums[i];
    *out = t;
  }
}

// Per-device set-up: the device address of the scratch array.
int scratch_address(double** addr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return int(e);
  if (dev < 0 || dev >= kMaxDevices) return int(cudaErrorInvalidDevice);
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_sqsum_scratch);
    if (e != cudaSuccess) return int(e);
    g_scratch_addr[dev] = static_cast<double*>(p);
  }
  *addr = g_scratch_addr[dev];
  return 0;
}
}  // namespace

extern "C" int tn5b_grad_sqsum_noalloc(const void* grad, int grad_is_fp32, int64_t n, double* out,
                                       void* stream) {
  if (!grad || !out || n <= 0 || n % 8 || (reinterpret_cast<uintptr_t>(grad) & 15)) return -1;
  const int64_t parts = (n + kChunk - 1) / kChunk;
  if (parts > kMaxParts) return -2;  // n beyond 16384 * 16384 elements
  double* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (grad_is_fp32)
    chunk_sqsum<float><<<unsigned(parts), kThreads, 0, s>>>(static_cast<const float*>(grad), n, scratch);
  else
    chunk_sqsum<__nv_bfloat16><<<unsigned(parts), kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(grad), n,
                                                                   scratch);
  finish_sqsum<<<1, kThreads, 0, s>>>(scratch, int(parts), out);
  return int(cudaGetLastError());
}
