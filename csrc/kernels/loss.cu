// Vocab-parallel cross-entropy (sm_100a).  Each rank holds logits [M, V/W]
// (BF16) for its vocabulary shard; softmax statistics are FP32.
//
//   pass 1  ce_stats:   row max over the shard, target logit if the target is local
//   (host)  all-reduce MAX of row max across the TP group
//   pass 2  ce_sumexp:  sum exp(x - gmax) over the shard
//   (host)  all-reduce SUM of (sumexp, selected)
//   pass 3  ce_loss:    loss_i = log(sum) + gmax - selected; mean in fixed order
//   bwd     ce_bwd:     dlogits = (exp(x - gmax) / sum - onehot) * scale, BF16, in place
//
// Semantics: VocabCrossEntropy of TempName-5090 python/flux_5090/model.py:143-176.
#include "kernels_api.h"
#include <cuda_bf16.h>

namespace tn5b {
namespace kernels {
namespace {
constexpr int kThreads = 256;

__device__ __forceinline__ float block_reduce_max(float v, float* sh) {
#pragma unroll
  for (int d = 16; d; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  const int w = threadIdx.x / 32, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < kThreads / 32 ? sh[l] : -INFINITY;
#pragma unroll
    for (int d = 16; d; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  const float r = sh[0];
  __syncthreads();
  return r;
}
__device__ __forceinline__ float block_reduce_sum(float v, float* sh) {
#pragma unroll
  for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  const int w = threadIdx.x / 32, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < kThreads / 32 ? sh[l] : 0.f;
#pragma unroll
    for (int d = 16; d; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  const float r = sh[0];
  __syncthreads();
  return r;
}

__global__ void ce_stats_kernel(const __nv_bfloat16* logits, int64_t ld, int V, const int64_t* targets,
                                int64_t start, float* rowmax, float* selected) {
  __shared__ float sh[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + int64_t(row) * ld;
  float m = -INFINITY;
  for (int c = threadIdx.x * 8; c < V; c += kThreads * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + c);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) m = fmaxf(m, __bfloat162float(h[i]));
  }
  m = block_reduce_max(m, sh);
  if (threadIdx.x == 0) {
    rowmax[row] = m;
    const int64_t t = targets[row] - start;
    selected[row] = (t >= 0 && t < V) ? __bfloat162float(x[t]) : 0.f;
  }
}

__global__ void ce_sumexp_kernel(const __nv_bfloat16* logits, int64_t ld, int V, const float* gmax,
                                 float* sumexp) {
  __shared__ float sh[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + int64_t(row) * ld;
  const float m = gmax[row];
  float s = 0.f;
  for (int c = threadIdx.x * 8; c < V; c += kThreads * 8) {
    const uint4 raw = *reinterpret_cast<const uint4*>(x + c);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) s += expf(__bfloat162float(h[i]) - m);
  }
  s = block_reduce_sum(s, sh);
  if (threadIdx.x == 0) sumexp[row] = s;
}

// Single CTA: per-row losses and their mean (fixed-order tree, deterministic).
__global__ void ce_loss_kernel(const float* gmax, const float* sumexp, const float* selected, int M,
                               float* row_loss, float* mean_loss, float scale) {
  __shared__ float sh[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < M; i += kThreads) {
    const float l = logf(sumexp[i]) + gmax[i] - selected[i];
    if (row_loss) row_loss[i] = l;
    acc += l;
  }
  acc = block_reduce_sum(acc, sh);
  if (threadIdx.x == 0) *mean_loss = acc * scale;
}

__global__ void ce_bwd_kernel(__nv_bfloat16* logits, int64_t ld, int V, const int64_t* targets,
                              int64_t start, const float* gmax, const float* sumexp, float scale,
                              const float* scale_ptr) {
  const int row = blockIdx.x;
  __nv_bfloat16* x = logits + int64_t(row) * ld;
  const float m = gmax[row];
  const float inv = sumexp[row];
  const float g = scale_ptr ? *scale_ptr * scale : scale;
  const int64_t t = targets[row] - start;
  for (int c = threadIdx.x * 8; c < V; c += kThreads * 8) {
    uint4 raw = *reinterpret_cast<const uint4*>(x + c);
    __nv_bfloat16* h = reinterpret_cast<__nv_bfloat16*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float p = expf(__bfloat162float(h[i]) - m) / inv;
      if (c + i == t) p -= 1.0f;
      h[i] = __float2bfloat16_rn(p * g);
    }
    *reinterpret_cast<uint4*>(x + c) = raw;
  }
}
}  // namespace

int ce_stats(const void* logits, int64_t ld, int M, int V, const int64_t* targets, int64_t start,
             float* rowmax, float* selected, cudaStream_t s) {
  if (V % 8 || ld % 8) return -1;
  ce_stats_kernel<<<M, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), ld, V, targets,
                                         start, rowmax, selected);
  return int(cudaGetLastError());
}
int ce_sumexp(const void* logits, int64_t ld, int M, int V, const float* gmax, float* sumexp,
              cudaStream_t s) {
  ce_sumexp_kernel<<<M, kThreads, 0, s>>>(static_cast<const __nv_bfloat16*>(logits), ld, V, gmax,
                                          sumexp);
  return int(cudaGetLastError());
}
int ce_loss(const float* gmax, const float* sumexp, const float* selected, int M, float* row_loss,
            float* mean_loss, float scale, cudaStream_t s) {
  ce_loss_kernel<<<1, kThreads, 0, s>>>(gmax, sumexp, selected, M, row_loss, mean_loss, scale);
  return int(cudaGetLastError());
}
int ce_bwd(void* logits, int64_t ld, int M, int V, const int64_t* targets, int64_t start,
           const float* gmax, const float* sumexp, float scale, const float* scale_ptr,
           cudaStream_t s) {
  ce_bwd_kernel<<<M, kThreads, 0, s>>>(static_cast<__nv_bfloat16*>(logits), ld, V, targets, start, gmax,
                                       sumexp, scale, scale_ptr);
  return int(cudaGetLastError());
}

}  // namespace kernels
}  // namespace tn5b
