// Vocab-parallel embedding lookup / backward and position embedding (sm_100a).
//
// Forward: out[i] = E[tok_i - start] if the token is in this rank's vocabulary
// shard, else 0 (the masked contribution that the TP reduce-scatter sums,
// model.py:240-245 of TempName-5090).  Position rows are added to the
// sequence-parallel shard after the reduce-scatter.
// Backward (deterministic, no float atomics): tokens are bucketed by a stable
// counting sort -- each token's rank inside its bucket is the number of equal
// earlier tokens, counted from a shared-memory copy of the token ids -- then
// one CTA per vocabulary row sums its tokens' gradient rows in position order
// in FP32 and adds the result to the row (which may already hold the tied
// LM-head gradient): dE[v] = bf16(dE[v] + bf16(sum)).
#include "kernels_api.h"
#include <cuda_bf16.h>

namespace tn5b {
namespace kernels {
namespace {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* v) {
  const uint4 raw = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(h[i]);
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float* v) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}

__global__ void embed_fwd_kernel(const int64_t* tok, const __nv_bfloat16* E, __nv_bfloat16* out, int M,
                                 int H, int64_t start, int64_t V) {
  const int row = blockIdx.x;
  const int64_t t = tok[row] - start;
  const bool local = t >= 0 && t < V;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (local) v = *reinterpret_cast<const uint4*>(E + t * H + c);
    *reinterpret_cast<uint4*>(out + int64_t(row) * H + c) = v;
  }
}

// x[i] = bf16(x[i] + P[(row0 + i) % S])
__global__ void add_position_kernel(__nv_bfloat16* x, const __nv_bfloat16* P, int rows, int H,
                                    int64_t row0, int S) {
  const int i = blockIdx.x;
  const int64_t p = (row0 + i) % S;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float a[8], b[8];
    load8(x + int64_t(i) * H + c, a);
    load8(P + p * H + c, b);
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] += b[k];
    store8(x + int64_t(i) * H + c, a);
  }
}

// dP[p] = sum over local rows i with (row0 + i) % S == p of g[i] (increasing i)
__global__ void position_bwd_kernel(const __nv_bfloat16* g, __nv_bfloat16* dP, int rows, int H,
                                    int64_t row0, int S) {
  const int p = blockIdx.x;
  const int first = int(((p - row0) % S + S) % S);
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0};
    for (int i = first; i < rows; i += S) {
      float v[8];
      load8(g + int64_t(i) * H + c, v);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc[k] += v[k];
    }
    store8(dP + int64_t(p) * H + c, acc);
  }
}

// Stable bucket rank: rank[i] = #{j < i : tok[j] == tok[i]}; counts[v] via int atomics.
__global__ void bucket_rank_kernel(const int64_t* tok, int M, int64_t start, int64_t V, int* rank,
                                   int* counts) {
  extern __shared__ int64_t sh_tok[];
  for (int j = threadIdx.x; j < M; j += blockDim.x) sh_tok[j] = tok[j];
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M) return;
  const int64_t t = sh_tok[i];
  if (t - start < 0 || t - start >= V) {
    rank[i] = -1;
    return;
  }
  int r = 0;
  for (int j = 0; j < i; ++j) r += sh_tok[j] == t;
  rank[i] = r;
  atomicAdd(counts + (t - start), 1);
}

// Exclusive scan of counts (single CTA, fixed order).
__global__ void scan_kernel(const int* counts, int* offsets, int64_t V) {
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < V; base += blockDim.x) {
    const int64_t v = base + threadIdx.x;
    const int c = v < V ? counts[v] : 0;
    // warp-inclusive scan
    int x = c;
    const int lane = threadIdx.x & 31, w = threadIdx.x / 32;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, d);
      if (lane >= d) x += y;
    }
    __shared__ int warp_tot[32];
    if (lane == 31) warp_tot[w] = x;
    __syncthreads();
    if (w == 0) {
      int t = lane < int(blockDim.x / 32) ? warp_tot[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, t, d);
        if (lane >= d) t += y;
      }
      warp_tot[lane] = t;
    }
    __syncthreads();
    const int prefix = (w ? warp_tot[w - 1] : 0) + x - c;
    if (v < V) offsets[v] = carry + prefix;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry += prefix + c;
    __syncthreads();
  }
  if (threadIdx.x == 0) offsets[V] = carry;
}

__global__ void bucket_fill_kernel(const int64_t* tok, const int* rank, const int* offsets, int M,
                                   int64_t start, int* sorted) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= M || rank[i] < 0) return;
  sorted[offsets[tok[i] - start] + rank[i]] = i;
}

// One CTA per vocabulary row with a non-empty bucket.
__global__ void embed_bwd_kernel(const __nv_bfloat16* g, const int* sorted, const int* offsets,
                                 __nv_bfloat16* dE, int H, int accumulate) {
  const int v = blockIdx.x;
  const int b = offsets[v], e = offsets[v + 1];
  if (b == e) return;
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8] = {0};
    for (int k = b; k < e; ++k) {
      float x[8];
      load8(g + int64_t(sorted[k]) * H + c, x);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += x[q];
    }
    if (accumulate) {
      float cur[8];
      load8(dE + int64_t(v) * H + c, cur);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] = cur[q] + __bfloat162float(__float2bfloat16_rn(acc[q]));
    }
    store8(dE + int64_t(v) * H + c, acc);
  }
}
}  // namespace

int embed_fwd(const int64_t* tok, const void* E, void* out, int M, int H, int64_t start, int64_t V,
              cudaStream_t s) {
  if (H % 8) return -1;
  embed_fwd_kernel<<<M, 128, 0, s>>>(tok, static_cast<const __nv_bfloat16*>(E),
                                     static_cast<__nv_bfloat16*>(out), M, H, start, V);
  return int(cudaGetLastError());
}
int add_position(void* x, const void* P, int rows, int H, int64_t row0, int S, cudaStream_t s) {
  add_position_kernel<<<rows, 128, 0, s>>>(static_cast<__nv_bfloat16*>(x),
                                           static_cast<const __nv_bfloat16*>(P), rows, H, row0, S);
  return int(cudaGetLastError());
}
int position_bwd(const void* g, void* dP, int rows, int H, int64_t row0, int S, cudaStream_t s) {
  position_bwd_kernel<<<S, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(g),
                                        static_cast<__nv_bfloat16*>(dP), rows, H, row0, S);
  return int(cudaGetLastError());
}
int64_t embed_bwd_workspace_ints(int M, int64_t V) { return 2 * int64_t(M) + 2 * (V + 1); }
int embed_bwd(const int64_t* tok, const void* g, void* dE, int M, int H, int64_t start, int64_t V,
              int* workspace, int accumulate, cudaStream_t s) {
  int* rank = workspace;
  int* sorted = rank + M;
  int* counts = sorted + M;
  int* offsets = counts + (V + 1);
  cudaMemsetAsync(counts, 0, sizeof(int) * (V + 1), s);
  const size_t sh = sizeof(int64_t) * size_t(M);
  if (sh > 200 * 1024) return -1;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(bucket_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    configured = true;
  }
  bucket_rank_kernel<<<(M + 255) / 256, 256, sh, s>>>(tok, M, start, V, rank, counts);
  scan_kernel<<<1, 1024, 0, s>>>(counts, offsets, V);
  bucket_fill_kernel<<<(M + 255) / 256, 256, 0, s>>>(tok, rank, offsets, M, start, sorted);
  embed_bwd_kernel<<<unsigned(V), 128, 0, s>>>(static_cast<const __nv_bfloat16*>(g), sorted, offsets,
                                                static_cast<__nv_bfloat16*>(dE), H, accumulate);
  return int(cudaGetLastError());
}

}  // namespace kernels
}  // namespace tn5b
