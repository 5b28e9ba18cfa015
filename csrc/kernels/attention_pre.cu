// Attention backward pre-pass: D[b*H + h][s] = sum_d dO[token, h, d] * O[token, h, d]
// (FP32), consumed by the tcgen05 backward kernels in attention_tc.cu.
#include "kernels_api.h"
#include <cuda_bf16.h>
#include <cstdint>

namespace tn5b {
namespace kernels {
namespace {
constexpr int D = 128;

// D[bh][q] = sum_d dO * O
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* out, int64_t ld_out, const __nv_bfloat16* dout,
                                    int64_t ld_dout, float* Dvec, int S, int H, int total_rows) {
  const int idx = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;  // (b*S + s)*H + h
  if (idx >= total_rows) return;
  const int lane = threadIdx.x & 31;
  const int h = idx % H, row = idx / H;
  const int b = row / S, s = row % S;
  const uint2 a = *reinterpret_cast<const uint2*>(out + int64_t(row) * ld_out + h * D + lane * 4);
  const uint2 c = *reinterpret_cast<const uint2*>(dout + int64_t(row) * ld_dout + h * D + lane * 4);
  const __nv_bfloat16* ah = reinterpret_cast<const __nv_bfloat16*>(&a);
  const __nv_bfloat16* ch = reinterpret_cast<const __nv_bfloat16*>(&c);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) acc += __bfloat162float(ah[i]) * __bfloat162float(ch[i]);
#pragma unroll
  for (int d = 16; d; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
  if (lane == 0) Dvec[int64_t(b * H + h) * S + s] = acc;
}

}  // namespace

int attention_bwd_pre(const void* out, int64_t ld_out, const void* dout, int64_t ld_dout, float* Dvec, int B,
                      int S, int H, cudaStream_t s) {
  const int rows = B * S * H;
  attn_bwd_pre_kernel<<<(rows + 7) / 8, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(out), ld_out,
                                                     static_cast<const __nv_bfloat16*>(dout), ld_dout, Dvec,
                                                     S, H, rows);
  return int(cudaGetLastError());
}

}  // namespace kernels
}  // namespace tn5b
