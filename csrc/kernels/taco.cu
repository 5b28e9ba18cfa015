// Standalone TACO H128/E4M3FN codec kernels (sm_100a).
//
// Packet format and arithmetic follow TempName-5090 src/taco/codec.cu:
// group = 128 consecutive BF16 elements; SoA packet
//   payload[E] u8 | quant[E/128] f32 | adaptive[E/128] f32   (136 B / group)
// Encode: adaptive = clamp(448 * rsqrt(max(mean(x^2) + 1e-6, 1e-12)), 1e-3, 1e3);
// x * adaptive -> normalised Walsh-Hadamard (butterfly distances 1..64,
// scale 1/sqrt(128)) -> quant = clamp(max|x| / 448, 1e-12, 1e6) ->
// e4m3(x / quant) with finite saturation, round-to-nearest-even.
// Decode is the inverse with the same butterfly.  One warp handles one group,
// lane l holding coefficients l + 32 j (encode) or 4l..4l+3 (decode); every
// FP32 op is an explicit correctly-rounded intrinsic (no contraction), so the
// bytes and values are identical to the reference kernels on the same input.
#include "kernels_api.h"
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace tn5b {
namespace kernels {
namespace {
constexpr int kWarps = 4;
constexpr unsigned kFull = 0xffffffffu;
constexpr float kNorm = 0.08838834764831844055f;

__device__ __forceinline__ float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

__device__ __forceinline__ float warp_sum_down(float x) {
#pragma unroll
  for (int d = 16; d; d >>= 1) x = __fadd_rn(x, __shfl_down_sync(kFull, x, d));
  return x;
}

__device__ __forceinline__ void butterfly_lanes(float (&x)[4], int first, int last) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int d = first; d <= last; d *= 2) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float o = __shfl_xor_sync(kFull, x[j], d);
      x[j] = (lane & d) ? __fsub_rn(o, x[j]) : __fadd_rn(x[j], o);
    }
  }
}
__device__ __forceinline__ void butterfly_regs(float (&x)[4], bool first_pairs_adjacent) {
  float a = x[0], b = x[1], c = x[2], d = x[3];
  if (first_pairs_adjacent) {  // (0,1),(2,3) then (0,2),(1,3)
    x[0] = __fadd_rn(a, b); x[1] = __fsub_rn(a, b); x[2] = __fadd_rn(c, d); x[3] = __fsub_rn(c, d);
    a = x[0]; b = x[1]; c = x[2]; d = x[3];
    x[0] = __fadd_rn(a, c); x[1] = __fadd_rn(b, d); x[2] = __fsub_rn(a, c); x[3] = __fsub_rn(b, d);
  }
}

// lane l owns x[j] = element l + 32 j of the group.
__device__ __forceinline__ void encode_warp(const __nv_bfloat16* in, uint8_t* payload, float* quant_out,
                                            float* adaptive_out) {
  const int lane = threadIdx.x & 31;
  float x[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = __bfloat162float(in[lane + 32 * j]);
  float part[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) part[j] = __shfl_sync(kFull, warp_sum_down(__fmul_rn(x[j], x[j])), 0);
  float s = lane < 4 ? part[lane] : 0.f;
  s = __shfl_sync(kFull, warp_sum_down(s), 0);
  const float variance = __fadd_rn(s / 128.f, 1e-6f);
  const float adaptive = clampf(__fmul_rn(448.f, rsqrtf(fmaxf(variance, 1e-12f))), 1e-3f, 1e3f);
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = __fmul_rn(x[j], adaptive);
  butterfly_lanes(x, 1, 16);
  {
    float a = x[0], b = x[1], c = x[2], d = x[3];
    x[0] = __fadd_rn(a, b); x[1] = __fsub_rn(a, b); x[2] = __fadd_rn(c, d); x[3] = __fsub_rn(c, d);
    a = x[0]; b = x[1]; c = x[2]; d = x[3];
    x[0] = __fadd_rn(a, c); x[1] = __fadd_rn(b, d); x[2] = __fsub_rn(a, c); x[3] = __fsub_rn(b, d);
  }
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    x[j] = __fmul_rn(x[j], kNorm);
    m = fmaxf(m, fabsf(x[j]));
  }
#pragma unroll
  for (int d = 16; d; d >>= 1) m = fmaxf(m, __shfl_down_sync(kFull, m, d));
  m = __shfl_sync(kFull, m, 0);
  const float quant = clampf(m / 448.f, 1e-12f, 1e6f);
  if (lane == 0) {
    *quant_out = quant;
    *adaptive_out = adaptive;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const unsigned q = unsigned(__nv_cvt_float_to_fp8(x[j] / quant, __NV_SATFINITE, __NV_E4M3)) & 0xFFu;
    const unsigned b1 = __shfl_down_sync(kFull, q, 1);
    const unsigned b2 = __shfl_down_sync(kFull, q, 2);
    const unsigned b3 = __shfl_down_sync(kFull, q, 3);
    if ((lane & 3) == 0)
      *reinterpret_cast<unsigned*>(payload + lane + 32 * j) = q | (b1 << 8) | (b2 << 16) | (b3 << 24);
  }
}

// lane l returns decoded elements 4l..4l+3 of the group.
__device__ __forceinline__ void decode_warp(const uint8_t* payload, float quant, float adaptive,
                                            float (&out)[4]) {
  const int lane = threadIdx.x & 31;
  const unsigned raw = *reinterpret_cast<const unsigned*>(payload + lane * 4);
  const __half2 lo(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(raw & 0xFFFFu), __NV_E4M3));
  const __half2 hi(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(raw >> 16), __NV_E4M3));
  float x[4] = {__fmul_rn(__low2float(lo), quant), __fmul_rn(__high2float(lo), quant),
                __fmul_rn(__low2float(hi), quant), __fmul_rn(__high2float(hi), quant)};
  butterfly_regs(x, true);
  butterfly_lanes(x, 1, 16);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    out[j] = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(__fmul_rn(x[j], kNorm), adaptive)));
}

__global__ void encode_kernel(const __nv_bfloat16* in, uint8_t* packet, int64_t elements) {
  const int64_t groups = elements / 128;
  const int64_t g = int64_t(blockIdx.x) * kWarps + threadIdx.x / 32;
  if (g >= groups) return;
  encode_warp(in + g * 128, packet + g * 128, reinterpret_cast<float*>(packet + elements) + g,
              reinterpret_cast<float*>(packet + elements + 4 * groups) + g);
}

__device__ __forceinline__ void store4(__nv_bfloat16* out, const float (&v)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
  uint2 w;
  w.x = *reinterpret_cast<uint32_t*>(&a);
  w.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(out) = w;
}

__global__ void decode_kernel(const uint8_t* packet, __nv_bfloat16* out, int64_t elements) {
  const int64_t groups = elements / 128;
  const int64_t g = int64_t(blockIdx.x) * kWarps + threadIdx.x / 32;
  if (g >= groups) return;
  const float quant = reinterpret_cast<const float*>(packet + elements)[g];
  const float adaptive = reinterpret_cast<const float*>(packet + elements + 4 * groups)[g];
  float v[4];
  decode_warp(packet + g * 128, quant, adaptive, v);
  store4(out + g * 128 + (threadIdx.x & 31) * 4, v);
}

// Ordered fused decode + reduce: sources 0..world-1, local BF16 partial at `rank`,
// remote slot = source - (source > rank); round to BF16 after every source.
__global__ void decode_reduce_kernel(const __nv_bfloat16* local, const uint8_t* packets,
                                     __nv_bfloat16* out, int64_t elements, int rank, int world) {
  const int64_t groups = elements / 128;
  const int64_t g = int64_t(blockIdx.x) * kWarps + threadIdx.x / 32;
  if (g >= groups) return;
  const int64_t index = g * 128 + (threadIdx.x & 31) * 4;
  const int64_t pbytes = groups * 136;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = 0; s < world; ++s) {
    float v[4];
    if (s == rank) {
      const uint2 raw = *reinterpret_cast<const uint2*>(local + index);
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = __bfloat162float(h[j]);
    } else {
      const uint8_t* p = packets + int64_t(s - (s > rank)) * pbytes;
      decode_warp(p + g * 128, reinterpret_cast<const float*>(p + elements)[g],
                  reinterpret_cast<const float*>(p + elements + 4 * groups)[g], v);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = __bfloat162float(__float2bfloat16_rn(__fadd_rn(acc[j], v[j])));
  }
  store4(out + index, acc);
}

__global__ void reduce_kernel(const __nv_bfloat16* local, const __nv_bfloat16* remote,
                              __nv_bfloat16* out, int64_t elements, int rank, int world) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= elements) return;
  float acc = 0.f;
  for (int s = 0; s < world; ++s) {
    const __nv_bfloat16 v = s == rank ? local[i] : remote[int64_t(s - (s > rank)) * elements + i];
    acc = __bfloat162float(__float2bfloat16_rn(__fadd_rn(acc, __bfloat162float(v))));
  }
  out[i] = __float2bfloat16_rn(acc);
}

__global__ void delay_kernel(unsigned long long cycles) {
  const unsigned long long start = clock64();
  while (clock64() - start < cycles) __nanosleep(100);
}

unsigned grid_groups(int64_t elements) { return unsigned((elements / 128 + kWarps - 1) / kWarps); }
}  // namespace

int taco_encode(const void* in, void* packet, int64_t elements, cudaStream_t s) {
  if (elements <= 0 || elements % 128) return -1;
  encode_kernel<<<grid_groups(elements), 32 * kWarps, 0, s>>>(
      static_cast<const __nv_bfloat16*>(in), static_cast<uint8_t*>(packet), elements);
  return int(cudaGetLastError());
}
int taco_decode(const void* packet, void* out, int64_t elements, cudaStream_t s) {
  if (elements <= 0 || elements % 128) return -1;
  decode_kernel<<<grid_groups(elements), 32 * kWarps, 0, s>>>(
      static_cast<const uint8_t*>(packet), static_cast<__nv_bfloat16*>(out), elements);
  return int(cudaGetLastError());
}
int taco_decode_reduce(const void* local, const void* packets, void* out, int64_t elements, int rank,
                       int world, cudaStream_t s) {
  if (elements <= 0 || elements % 128 || world < 2 || rank < 0 || rank >= world) return -1;
  decode_reduce_kernel<<<grid_groups(elements), 32 * kWarps, 0, s>>>(
      static_cast<const __nv_bfloat16*>(local), static_cast<const uint8_t*>(packets),
      static_cast<__nv_bfloat16*>(out), elements, rank, world);
  return int(cudaGetLastError());
}
int ordered_reduce(const void* local, const void* remote, void* out, int64_t elements, int rank,
                   int world, cudaStream_t s) {
  if (elements <= 0 || world < 2 || rank < 0 || rank >= world) return -1;
  reduce_kernel<<<unsigned((elements + 255) / 256), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(local), static_cast<const __nv_bfloat16*>(remote),
      static_cast<__nv_bfloat16*>(out), elements, rank, world);
  return int(cudaGetLastError());
}
int diagnostic_delay(unsigned long long cycles, cudaStream_t s) {
  if (!cycles || cycles > 100000000ULL) return -1;
  delay_kernel<<<1, 1, 0, s>>>(cycles);
  return int(cudaGetLastError());
}

}  // namespace kernels
}  // namespace tn5b
