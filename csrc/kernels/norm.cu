// LayerNorm forward/backward and column reductions (sm_100a, SIMT).
//
// Forward: one warp per row, the row held in registers (H/32 values per lane,
// 16-byte loads), FP32 mean and variance by two passes over the registers,
// y = bf16((x - mean) * rstd * w + b); mean/rstd saved in FP32.
// Backward: dx per row by one warp (same register residency); dgamma/dbeta by a
// column-parallel two-stage deterministic reduction (per-CTA partial sums over
// a fixed row range, then a fixed-order final sum) -- no atomics.
// Semantics: F.layer_norm over the last dim with eps (model.py:231-233 of
// TempName-5090), computed in FP32 from BF16 storage.
#include "kernels_api.h"
#include <cuda_bf16.h>

namespace tn5b {
namespace kernels {
namespace {
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ float warp_allsum(float x) {
#pragma unroll
  for (int d = 16; d; d >>= 1) x += __shfl_xor_sync(kFull, x, d);
  return x;
}

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

// VPL = values per lane = H / 32 (multiple of 8).
template <int VPL>
__global__ void ln_fwd_kernel(const __nv_bfloat16* x, const __nv_bfloat16* w, const __nv_bfloat16* b,
                              __nv_bfloat16* y, float* mean_out, float* rstd_out, int rows,
                              int64_t ld_x, int64_t ld_y, float eps) {
  constexpr int H = VPL * 32;
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float v[VPL];
  const __nv_bfloat16* xr = x + int64_t(row) * ld_x;
#pragma unroll
  for (int c = 0; c < VPL / 8; ++c) load8(xr + c * 256 + lane * 8, v + c * 8);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) s += v[i];
  const float mean = warp_allsum(s) / H;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float d = v[i] - mean;
    q += d * d;
  }
  const float var = warp_allsum(q) / H;
  const float rstd = rsqrtf(var + eps);
  __nv_bfloat16* yr = y + int64_t(row) * ld_y;
#pragma unroll
  for (int c = 0; c < VPL / 8; ++c) {
    float wv[8], bv[8], o[8];
    load8(w + c * 256 + lane * 8, wv);
    load8(b + c * 256 + lane * 8, bv);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = (v[c * 8 + i] - mean) * rstd * wv[i] + bv[i];
    store8(yr + c * 256 + lane * 8, o);
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

template <int VPL>
__global__ void ln_bwd_dx_kernel(const __nv_bfloat16* dy, const __nv_bfloat16* x,
                                 const __nv_bfloat16* w, const float* mean, const float* rstd,
                                 __nv_bfloat16* dx, int rows, const __nv_bfloat16* dres) {
  // Two passes over the (L1/L2-resident) row keep register use at VPL values.
  constexpr int H = VPL * 32;
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float mu = mean[row], rs = rstd[row];
  const __nv_bfloat16* dyr = dy + int64_t(row) * H;
  const __nv_bfloat16* xr = x + int64_t(row) * H;
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int c = 0; c < VPL / 8; ++c) {
    float dv[8], xv[8], wv[8];
    load8(dyr + c * 256 + lane * 8, dv);
    load8(xr + c * 256 + lane * 8, xv);
    load8(w + c * 256 + lane * 8, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float gi = dv[i] * wv[i];
      s1 += gi;
      s2 += gi * ((xv[i] - mu) * rs);
    }
  }
  s1 = warp_allsum(s1) / H;
  s2 = warp_allsum(s2) / H;
#pragma unroll
  for (int c = 0; c < VPL / 8; ++c) {
    float dv[8], xv[8], wv[8], o[8];
    load8(dyr + c * 256 + lane * 8, dv);
    load8(xr + c * 256 + lane * 8, xv);
    load8(w + c * 256 + lane * 8, wv);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = rs * (dv[i] * wv[i] - s1 - ((xv[i] - mu) * rs) * s2);
    if (dres) {
      // Residual stream gradient joins here: dx = bf16(bf16(ln_dx) + dres).
      float r[8];
      load8(dres + int64_t(row) * H + c * 256 + lane * 8, r);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __bfloat162float(__float2bfloat16_rn(o[i])) + r[i];
    }
    store8(dx + int64_t(row) * H + c * 256 + lane * 8, o);
  }
}

// Partial column sums of dy*xhat (dgamma) and dy (dbeta) over rows
// [blockIdx.y * rows_per, ...); thread owns 8 consecutive columns.
__global__ void ln_bwd_dwdb_partial(const __nv_bfloat16* dy, const __nv_bfloat16* x,
                                    const float* mean, const float* rstd, float* part_w,
                                    float* part_b, int rows, int H, int rows_per) {
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (col >= H) return;
  const int r0 = blockIdx.y * rows_per, r1 = min(rows, r0 + rows_per);
  float aw[8] = {0}, ab[8] = {0};
  for (int r = r0; r < r1; ++r) {
    float dv[8], xv[8];
    load8(dy + int64_t(r) * H + col, dv);
    load8(x + int64_t(r) * H + col, xv);
    const float mu = mean[r], rs = rstd[r];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      aw[i] += dv[i] * ((xv[i] - mu) * rs);
      ab[i] += dv[i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    part_w[int64_t(blockIdx.y) * H + col + i] = aw[i];
    part_b[int64_t(blockIdx.y) * H + col + i] = ab[i];
  }
}

// out[c] = bf16(sum_p part[p][c]) in fixed order (optionally also into out2).
__global__ void column_finish(const float* part, int parts, int H, __nv_bfloat16* out, float* out32) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float s = 0.f;
  for (int p = 0; p < parts; ++p) s += part[int64_t(p) * H + c];
  if (out) out[c] = __float2bfloat16_rn(s);
  if (out32) out32[c] = s;
}

// Column sums of a bf16 [rows, cols] matrix (bias gradients).
__global__ void colsum_partial(const __nv_bfloat16* g, int64_t ld, float* part, int rows, int cols,
                               int rows_per) {
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (col >= cols) return;
  const int r0 = blockIdx.y * rows_per, r1 = min(rows, r0 + rows_per);
  float a[8] = {0};
  for (int r = r0; r < r1; ++r) {
    float v[8];
    load8(g + int64_t(r) * ld + col, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] += v[i];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) part[int64_t(blockIdx.y) * cols + col + i] = a[i];
}

// GeLU backward: dx = bf16(dy * gelu'(pre)), gelu'(z) = Phi(z) + z * phi(z).
__global__ void gelu_bwd_kernel(const __nv_bfloat16* dy, const __nv_bfloat16* pre, __nv_bfloat16* dx,
                                int64_t n8) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  float d[8], z[8], o[8];
  load8(dy + i * 8, d);
  load8(pre + i * 8, z);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float cdf = 0.5f * (1.0f + erff(z[k] * 0.70710678118654752440f));
    const float pdf = 0.39894228040143267794f * expf(-0.5f * z[k] * z[k]);
    o[k] = d[k] * (cdf + z[k] * pdf);
  }
  store8(dx + i * 8, o);
}

template <int VPL>
int ln_fwd_launch(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd,
                  int rows, int64_t ld_x, int64_t ld_y, float eps, cudaStream_t s) {
  const int warps = 4;
  ln_fwd_kernel<VPL><<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(w),
      static_cast<const __nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(y), mean, rstd, rows, ld_x,
      ld_y, eps);
  return int(cudaGetLastError());
}
template <int VPL>
int ln_bwd_launch(const void* dy, const void* x, const void* w, const float* mean, const float* rstd,
                  void* dx, int rows, const void* dres, cudaStream_t s) {
  const int warps = 4;
  ln_bwd_dx_kernel<VPL><<<(rows + warps - 1) / warps, warps * 32, 0, s>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
      static_cast<const __nv_bfloat16*>(w), mean, rstd, static_cast<__nv_bfloat16*>(dx), rows,
      static_cast<const __nv_bfloat16*>(dres));
  return int(cudaGetLastError());
}
}  // namespace

int layernorm_fwd(const void* x, const void* w, const void* b, void* y, float* mean, float* rstd,
                  int rows, int H, int64_t ld_x, int64_t ld_y, float eps, cudaStream_t s) {
  switch (H) {
    case 256: return ln_fwd_launch<8>(x, w, b, y, mean, rstd, rows, ld_x, ld_y, eps, s);
    case 512: return ln_fwd_launch<16>(x, w, b, y, mean, rstd, rows, ld_x, ld_y, eps, s);
    case 1024: return ln_fwd_launch<32>(x, w, b, y, mean, rstd, rows, ld_x, ld_y, eps, s);
    case 2048: return ln_fwd_launch<64>(x, w, b, y, mean, rstd, rows, ld_x, ld_y, eps, s);
    case 4096: return ln_fwd_launch<128>(x, w, b, y, mean, rstd, rows, ld_x, ld_y, eps, s);
    default: return -1;
  }
}

int layernorm_bwd(const void* dy, const void* x, const void* w, const float* mean, const float* rstd,
                  void* dx, void* dw, void* db, float* workspace, int rows, int H, const void* dres,
                  cudaStream_t s) {
  int r;
  switch (H) {
    case 256: r = ln_bwd_launch<8>(dy, x, w, mean, rstd, dx, rows, dres, s); break;
    case 512: r = ln_bwd_launch<16>(dy, x, w, mean, rstd, dx, rows, dres, s); break;
    case 1024: r = ln_bwd_launch<32>(dy, x, w, mean, rstd, dx, rows, dres, s); break;
    case 2048: r = ln_bwd_launch<64>(dy, x, w, mean, rstd, dx, rows, dres, s); break;
    case 4096: r = ln_bwd_launch<128>(dy, x, w, mean, rstd, dx, rows, dres, s); break;
    default: return -1;
  }
  if (r) return r;
  const int parts = layernorm_bwd_parts(rows);
  const int rows_per = (rows + parts - 1) / parts;
  float* pw = workspace;
  float* pb = workspace + int64_t(parts) * H;
  dim3 grid((H / 8 + 127) / 128, parts);
  ln_bwd_dwdb_partial<<<grid, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(dy),
                                           static_cast<const __nv_bfloat16*>(x), mean, rstd, pw, pb,
                                           rows, H, rows_per);
  column_finish<<<(H + 255) / 256, 256, 0, s>>>(pw, parts, H, static_cast<__nv_bfloat16*>(dw), nullptr);
  column_finish<<<(H + 255) / 256, 256, 0, s>>>(pb, parts, H, static_cast<__nv_bfloat16*>(db), nullptr);
  return int(cudaGetLastError());
}

int layernorm_bwd_parts(int rows) { return rows >= 4096 ? 64 : (rows >= 512 ? 32 : 1); }

int column_sum(const void* g, int64_t ld, int rows, int cols, void* out, float* workspace,
               cudaStream_t s) {
  if (cols % 8) return -1;
  const int parts = layernorm_bwd_parts(rows);
  const int rows_per = (rows + parts - 1) / parts;
  dim3 grid((cols / 8 + 127) / 128, parts);
  colsum_partial<<<grid, 128, 0, s>>>(static_cast<const __nv_bfloat16*>(g), ld, workspace, rows, cols,
                                      rows_per);
  column_finish<<<(cols + 255) / 256, 256, 0, s>>>(workspace, parts, cols,
                                                   static_cast<__nv_bfloat16*>(out), nullptr);
  return int(cudaGetLastError());
}

int gelu_bwd(const void* dy, const void* pre, void* dx, int64_t n, cudaStream_t s) {
  if (n % 8) return -1;
  const int64_t n8 = n / 8;
  gelu_bwd_kernel<<<unsigned((n8 + 255) / 256), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(pre),
      static_cast<__nv_bfloat16*>(dx), n8);
  return int(cudaGetLastError());
}

}  // namespace kernels
}  // namespace tn5b
