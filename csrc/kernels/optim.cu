// Global gradient norm and fused AdamW over flat parameter buffers (sm_100a).
//
// grad_sqsum: per-CTA FP64 partial sums of FP32 squares (a grid-stride loop of
// fixed assignment), then one CTA sums the partials in a fixed order into an
// FP64 accumulator -- deterministic for a given grid.
// adamw: FP32 master weights + moments, BF16 or FP32 gradient input, the clip
// coefficient min(max_norm / (sqrt(norm2) + 1e-6), 1) computed on the device
// from the all-reduced FP64 squared norm (no host round trip), decoupled weight
// decay on the first `n_decay` elements, BF16 copy-out of the updated weights.
// Update order follows torch.optim.AdamW (single-tensor): p *= 1 - lr*wd;
// m = lerp(m, g, 1-b1); v = b2*v + (1-b2)*g*g; p -= (lr/bc1) * m / (sqrt(v)/sqrt(bc2) + eps).
// A non-finite norm skips the update and records status 9.
#include "kernels_api.h"
#include <cuda_bf16.h>

namespace tn5b {
namespace kernels {
namespace {
constexpr int kThreads = 256;

template <typename G>
__device__ __forceinline__ void load8g(const G* p, float* v);
template <>
__device__ __forceinline__ void load8g<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
}
template <>
__device__ __forceinline__ void load8g<float>(const float* p, float* v) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename G>
__global__ void sqsum_partial(const G* g, int64_t n8, double* partial) {
  __shared__ double sh[kThreads / 32];
  double acc = 0.0;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += int64_t(gridDim.x) * blockDim.x) {
    float v[8];
    load8g<G>(g + i * 8, v);
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += double(v[k] * v[k]);
  }
#pragma unroll
  for (int d = 16; d; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x / 32] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) s += sh[w];
    partial[blockIdx.x] = s;
  }
}

__global__ void sqsum_finish(const double* partial, int parts, double* out, int accumulate) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double s = 0.0;
    for (int p = 0; p < parts; ++p) s += partial[p];
    *out = accumulate ? *out + s : s;
  }
}

template <typename G>
__global__ void adamw_kernel(float* master, float* m, float* v, const G* grad, __nv_bfloat16* param,
                             int64_t n8, int64_t n_decay, const double* norm2, float max_norm,
                             float lr, float decay_factor, float beta1, float beta2, float eps,
                             float step_size, float bc2_sqrt, int* status) {
  const double total = *norm2;
  if (!isfinite(total)) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && status) atomicCAS(status, 0, 9);
    return;
  }
  float coef = 1.0f;
  if (max_norm > 0.f) coef = float(fmin(double(max_norm) / (sqrt(total) + 1e-6), 1.0));
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t base = i * 8;
    float g[8];
    load8g<G>(grad + base, g);
    float4* mp = reinterpret_cast<float4*>(master + base);
    float4* m1 = reinterpret_cast<float4*>(m + base);
    float4* v1 = reinterpret_cast<float4*>(v + base);
    float p8[8], a8[8], b8[8];
    *reinterpret_cast<float4*>(p8) = mp[0];
    *reinterpret_cast<float4*>(p8 + 4) = mp[1];
    *reinterpret_cast<float4*>(a8) = m1[0];
    *reinterpret_cast<float4*>(a8 + 4) = m1[1];
    *reinterpret_cast<float4*>(b8) = v1[0];
    *reinterpret_cast<float4*>(b8 + 4) = v1[1];
    const bool decay = base < n_decay;
    __nv_bfloat16 out[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float gk = g[k] * coef;
      float p = p8[k];
      if (decay) p = p * decay_factor;
      const float mk = a8[k] + (1.0f - beta1) * (gk - a8[k]);
      const float vk = b8[k] * beta2 + (1.0f - beta2) * gk * gk;
      const float denom = sqrtf(vk) / bc2_sqrt + eps;
      p = p - step_size * (mk / denom);
      p8[k] = p;
      a8[k] = mk;
      b8[k] = vk;
      out[k] = __float2bfloat16_rn(p);
    }
    mp[0] = *reinterpret_cast<float4*>(p8);
    mp[1] = *reinterpret_cast<float4*>(p8 + 4);
    m1[0] = *reinterpret_cast<float4*>(a8);
    m1[1] = *reinterpret_cast<float4*>(a8 + 4);
    v1[0] = *reinterpret_cast<float4*>(b8);
    v1[1] = *reinterpret_cast<float4*>(b8 + 4);
    *reinterpret_cast<uint4*>(param + base) = *reinterpret_cast<uint4*>(out);
  }
}

int grid_for(int64_t n8) {
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (n8 + kThreads - 1) / kThreads;
  const int64_t cap = int64_t(sms) * 8;
  return int(want < cap ? (want > 0 ? want : 1) : cap);
}
}  // namespace

int grad_sqsum_parts(int64_t n) { return grid_for(n / 8); }

int grad_sqsum(const void* grad, int is_fp32, int64_t n, double* partial, double* out, int accumulate,
               cudaStream_t s) {
  if (n % 8) return -1;
  const int64_t n8 = n / 8;
  const int grid = grid_for(n8);
  if (is_fp32)
    sqsum_partial<float><<<grid, kThreads, 0, s>>>(static_cast<const float*>(grad), n8, partial);
  else
    sqsum_partial<__nv_bfloat16><<<grid, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(grad), n8,
                                                           partial);
  sqsum_finish<<<1, 32, 0, s>>>(partial, grid, out, accumulate);
  return int(cudaGetLastError());
}

int adamw_step(float* master, float* m, float* v, const void* grad, int grad_fp32, void* param,
               int64_t n, int64_t n_decay, const double* norm2, float max_norm, float lr, float wd,
               float beta1, float beta2, float eps, int step, int* status, cudaStream_t s) {
  if (n % 8 || n_decay % 8) return -1;
  const int64_t n8 = n / 8;
  const double bc1 = 1.0 - pow(double(beta1), step);
  const double bc2 = 1.0 - pow(double(beta2), step);
  const float step_size = float(double(lr) / bc1);
  const float bc2_sqrt = float(sqrt(bc2));
  const float decay_factor = float(1.0 - double(lr) * double(wd));
  const int grid = grid_for(n8);
  if (grad_fp32)
    adamw_kernel<float><<<grid, kThreads, 0, s>>>(
        master, m, v, static_cast<const float*>(grad), static_cast<__nv_bfloat16*>(param), n8, n_decay,
        norm2, max_norm, lr, decay_factor, beta1, beta2, eps, step_size, bc2_sqrt, status);
  else
    adamw_kernel<__nv_bfloat16><<<grid, kThreads, 0, s>>>(
        master, m, v, static_cast<const __nv_bfloat16*>(grad), static_cast<__nv_bfloat16*>(param), n8,
        n_decay, norm2, max_norm, lr, decay_factor, beta1, beta2, eps, step_size, bc2_sqrt, status);
  return int(cudaGetLastError());
}

}  // namespace kernels
}  // namespace tn5b
