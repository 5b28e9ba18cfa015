// Causal attention forward on the sm_100a tensor cores (tcgen05 + TMEM + TMA),
// head_dim 128, BF16 in/out, FP32 softmax statistics.
//
// One CTA per (128-query tile, batch*head); heavy (late) query tiles first.
//   warp 0     TMA producer: the Q tile once, then K_j (3-stage ring, up to two
//              blocks ahead) and V_j (2-stage ring), 128 keys each.  Q/K/V are
//              read in place from the fused QKV buffer [tokens, 3*heads*128]
//              with one 2-D tensor map.
//   warp 1     MMA issuer: S_j = Q K_j^T into one of two TMEM buffers
//              (M=128, N=128, K=16 x 8), then O_h += P_{j-1,h} V_{j-1,h} for the
//              two key halves h (A operand P, BF16, read from TMEM; V as an
//              MN-major smem operand), each half issued as soon as its softmax
//              warps are done -- S_j is issued before PV_{j-1} so the softmax of
//              block j overlaps the tensor work of block j-1.
//   warps 2-9  softmax: two warps per TMEM lane quarter, warp `half` owning key
//              columns [64*half, +64) of every block with its own running max
//              (log2 domain), row sum and accumulator O_half, so the two never
//              synchronise inside the loop; O_half is rescaled in TMEM only when
//              its max grows by more than 2^8 (a stale max is exact: numerator
//              and denominator share it); P = exp2(s - m) is written as packed
//              BF16 into the first half of the warp's own 64 score columns (the
//              PV MMA addresses those chunks).  At the end the two warps swap
//              (m, l) once and each writes 64 columns of
//              O = (O_0 2^(m_0-m) + O_1 2^(m_1-m)) / (l_0 2^(m_0-m) + l_1 2^(m_1-m))
//              (BF16) plus the row LSE (natural log).
// TMEM: S0 [0,128), S1 [128,256), O_0 [256,384), O_1 [384,512) of 512 columns.
// Every wait is bounded; on a timeout the status word is set and the CTA exits.
// Semantics: causal scaled_dot_product_attention (TempName-5090 model.py:255).
#include "kernels_api.h"
#include "../common/ptx.cuh"

#include <cuda_bf16.h>
#include <cstdint>
#include <mutex>

namespace tn5b {
namespace kernels {
namespace {
constexpr int kD = 128;
constexpr int kBlk = 128;
constexpr int kThreads = 320;    // warp 0 TMA, warp 1 MMA, warps 2-9 elementwise (2 per TMEM lane quarter)
constexpr int kEwWarps = 8;
// Backward: no running max to share, so four elementwise warps per TMEM lane
// quarter, one per 32-column quarter of the score block (more warps to hide
// the TMEM-load, exp2 and shared-memory latencies of the elementwise pass).
constexpr int kBwdEwWarps = 16;
constexpr int kBwdThreads = 64 + 32 * kBwdEwWarps;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;

constexpr int kSmQ = 0;               // 2 x 16 KB (d chunks)
constexpr int kKStages = 3;
constexpr int kSmK = 32768;           // kKStages stages x 32 KB
constexpr int kSmV = 32768 * 4;       // 2 stages x 32 KB
constexpr int kSmBar = 32768 * 6;
constexpr int kSmTotal = kSmBar + 256 + 1024;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}
// [rows, cols] bf16 row-major (ld elements), box 64 columns x 128 rows, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows, uint64_t ld) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Hardware base-2 exponential (MUFU), flush-to-zero.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// K-major operand tile [128 rows][128 d] stored as two 64-column SW128 chunks.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return make_sw128_desc(base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
}
// MN-major operand (V: rows = keys = K dim, columns = d = N dim), two 64-column chunks.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk) {
  return make_sw128_desc(base + kk * 2048, 16384, 1024);
}

// TMEM column of packed BF16 K-chunk kk (16 values per row) inside a 128-column
// score buffer: the elementwise warp of half h writes its 64 probabilities as
// 32 packed columns at [64h, 64h+32), inside the columns only it reads.
__device__ __forceinline__ uint32_t packed_col(int kk) { return uint32_t((kk >> 2) * 64 + (kk & 3) * 8); }

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tq, __nv_bfloat16* __restrict__ out,
                       int64_t ld_out, float* __restrict__ lse, int S, int H, float scale, int* status,
                       uint64_t timeout_ns, unsigned long long* trace) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kSmBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;   // kKStages
  uint64_t* v_full = bars + 4;
  uint64_t* k_empty = bars + 6;  // kKStages
  uint64_t* v_empty = bars + 9;
  uint64_t* s_full = bars + 11;
  uint64_t* p_full = bars + 13;  // [score buffer][half]
  uint64_t* o_done = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ uint64_t xbar[4];  // per lane quarter: the two softmax warps' handshake

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  // Grid (B*H, S/128): blocks are scheduled x-fastest, so every head's heaviest
  // (latest) query tile runs in the first wave and the light ones fill the tail.
  const int bh = blockIdx.x;
  const int qt = int(gridDim.y) - 1 - int(blockIdx.y);
  const int b = bh / H, h = bh % H;
  const int q0 = qt * kBlk;
  const int row0 = b * S;
  const int nkb = qt + 1;
  // Optional progress trace (16 words per CTA): [0] SM id and stage, [1] producer,
  // [2] MMA issuer, [3..10] elementwise warps (block index + 1 reached).
  unsigned long long* tr = trace ? trace + (size_t(bh) * gridDim.y + qt) * 16 : nullptr;
  const unsigned long long tsm = (unsigned long long)smid() << 16;
  if (threadIdx.x == 0) trace_put(tr, 0, tsm | 1);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(k_full + i, 1);
      mbar_init(k_empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(v_full + i, 1);
      mbar_init(v_empty + i, 1);
      mbar_init(s_full + i, 1);
      mbar_init(p_full + 2 * i, kEwWarps / 2);
      mbar_init(p_full + 2 * i + 1, kEwWarps / 2);
    }
    mbar_init(o_done, 1);
    for (int i = 0; i < 4; ++i) mbar_init(xbar + i, 2);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) tma_prefetch_desc(&tq);
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = smem_u32(sm + kSmQ);
  if (threadIdx.x == 0) trace_put(tr, 0, tsm | 2);

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 32768);
      tma_load_2d(sm + kSmQ, &tq, q_full, h * kD, row0 + q0);
      tma_load_2d(sm + kSmQ + 16384, &tq, q_full, h * kD + 64, row0 + q0);
      // K runs up to two blocks ahead of V: K_{j+2} only waits for S_{j-1}
      // (early), V_j waits for PV_{j-2} (after the softmax of block j-2), so a
      // K load is never queued behind a V wait.
      int kn = 0;  // next K block to load
      bool ok = true;
      for (int j = 0; j < nkb && ok; ++j) {
        for (; kn < nkb && kn <= j + kKStages - 1; ++kn) {
          const int ks = kn % kKStages;
          if (!mbar_wait(k_empty + ks, ((kn / kKStages) & 1) ^ 1, timeout_ns, status, kTimeoutProducerEmpty,
                         abort_flag)) {
            ok = false;
            break;
          }
          trace_put(tr, 1, kn + 1);
          mbar_arrive_expect_tx(k_full + ks, 32768);
          uint8_t* kdst = sm + kSmK + ks * 32768;
          tma_load_2d(kdst, &tq, k_full + ks, (H + h) * kD, row0 + kn * kBlk);
          tma_load_2d(kdst + 16384, &tq, k_full + ks, (H + h) * kD + 64, row0 + kn * kBlk);
        }
        if (!ok) break;
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(v_empty + st, ph ^ 1, timeout_ns, status, kTimeoutProducerEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(v_full + st, 32768);
        uint8_t* vdst = sm + kSmV + st * 32768;
        tma_load_2d(vdst, &tq, v_full + st, (2 * H + h) * kD, row0 + j * kBlk);
        tma_load_2d(vdst + 16384, &tq, v_full + st, (2 * H + h) * kD + 64, row0 + j * kBlk);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(128, 128, 0, 0);
      const uint32_t idesc_o = make_idesc_bf16(128, 128, 0, 1);
      bool ok = mbar_wait(q_full, 0, timeout_ns, status, kTimeoutMmaFull, abort_flag);
      // PV of block i, one half of the keys at a time: O_h += P_h V_h, issued
      // as soon as the four softmax warps of half h have written P_h.
      auto issue_pv = [&](int i) -> bool {
        if (!mbar_wait(v_full + (i & 1), (i >> 1) & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) return false;
        const uint32_t vb = smem_u32(sm + kSmV + (i & 1) * 32768);
        const uint32_t p_tmem = tmem + uint32_t((i & 1) * 128);
        for (int hh = 0; hh < 2; ++hh) {
          if (!mbar_wait(p_full + 2 * (i & 1) + hh, (i >> 1) & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag))
            return false;
          tc_fence_after();
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4)
            umma_f16_tmem_a(tmem + 256 + hh * 128, p_tmem + packed_col(hh * 4 + k4), mnmajor_desc(vb, hh * 4 + k4),
                            idesc_o, (i > 0 || k4 > 0) ? 1u : 0u);
        }
        umma_commit(v_empty + (i & 1));
        umma_commit(o_done);
        return true;
      };
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1, ks = j % kKStages;
        if (!mbar_wait(k_full + ks, (j / kKStages) & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) {
          ok = false;
          break;
        }
        // S_j overwrites the buffer whose P_{j-2} the PV MMAs of block j-2 read
        // from TMEM.  MMAs with different accumulators may overlap in the
        // tensor pipe, and an MMA's TMEM A-operand reads are not ordered with a
        // later MMA's accumulator writes, so wait until PV_{j-2} has completed.
        if (j >= 2 && !mbar_wait(o_done, (j - 2) & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        trace_put(tr, 2, j + 1);
        const uint32_t kb = smem_u32(sm + kSmK + ks * 32768);
        const uint32_t d = tmem + uint32_t(st * 128);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(d, kmajor_desc(sQ, kk), kmajor_desc(kb, kk), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(k_empty + ks);
        umma_commit(s_full + st);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok) issue_pv(nkb - 1);
      // Drain: all MMAs (including the last PV) done before TMEM is freed.
      mbar_wait(o_done, (nkb - 1) & 1, timeout_ns, status, kTimeoutDrain, nullptr);
    }
  } else {
    // ------------------------------------------------------------- softmax
    // Two warps per TMEM lane quarter: `half` owns score columns [64*half, +64)
    // -- half of each key block -- with its own running max, row sum and
    // accumulator O_half (TMEM columns 256 + 128*half), so the two warps never
    // wait for each other inside the loop.  They combine once at the end:
    //   O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m)).
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    const uint32_t o_col = uint32_t(256 + half * 128);
    const float sl2 = scale * kLog2e;
    __shared__ float xchg[2][2][128];  // [m, l][half][row]
    float m_run = -INFINITY, l = 0.f;  // m_run in log2 units (-inf: no unmasked score yet)
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      if (!warp_wait(s_full + (j & 1), (j >> 1) & 1, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[64];
      {
        uint32_t r0[32], r1[32];
        const uint32_t sb = tmem + lane_base + uint32_t((j & 1) * 128 + half * 64);
        tmem_ld_32x32b_x32(sb, r0);
        tmem_ld_32x32b_x32(sb + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          x[i] = __uint_as_float(r0[i]);
          x[32 + i] = __uint_as_float(r1[i]);
        }
      }
      const bool diag = j == nkb - 1;
      float mxa[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) mxa[a] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        if (diag && half * 64 + c > row) x[c] = -INFINITY;  // raw-score max: scale > 0 keeps the order
        mxa[c & 7] = fmaxf(mxa[c & 7], x[c]);
      }
      const float mx = fmaxf(fmaxf(fmaxf(mxa[0], mxa[1]), fmaxf(mxa[2], mxa[3])),
                             fmaxf(fmaxf(mxa[4], mxa[5]), fmaxf(mxa[6], mxa[7]))) * sl2;
      // Lazy rescale, decided per row but executed by the whole warp (the TMEM
      // load/store are warp-collective): rows that keep their max scale by 1.
      const bool grow = mx > m_run + kRescale;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = grow ? mx : m_run;
        if (j > 0) {
          const float factor = grow ? ex2(m_run - m_new) : 1.f;  // 0 while m_run = -inf (O_h row is 0)
          l *= factor;
          if (!warp_wait(o_done, (j - 1) & 1, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t addr = tmem + lane_base + o_col + uint32_t(c * 32);
            tmem_ld_32x32b_x32(addr, r);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
            tmem_st_32x32b_x32(addr, r);
          }
          tmem_wait_st();
        }
        m_run = m_new;
      }
      // A half-row with every score masked so far (the diagonal block's upper
      // half of the first query tile) keeps m_run = -inf: its P is 0.
      const float m_use = m_run == -INFINITY ? 0.f : m_run;
      float suma[8];
#pragma unroll
      for (int a = 0; a < 8; ++a) suma[a] = 0.f;
      uint32_t w[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float p0 = ex2(fmaf(x[c], sl2, -m_use));
        const float p1 = ex2(fmaf(x[c + 1], sl2, -m_use));
        suma[c & 7] += p0;
        suma[(c + 1) & 7] += p1;
        w[c / 2] = pack2(p0, p1);
      }
      l += ((suma[0] + suma[1]) + (suma[2] + suma[3])) + ((suma[4] + suma[5]) + (suma[6] + suma[7]));
      // P (BF16) for columns [64*half, +64) -> packed TMEM columns [64*half, +32).
      tmem_st_32x32b_x32(tmem + lane_base + uint32_t((j & 1) * 128 + half * 64), w);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(p_full + 2 * (j & 1) + half);
        trace_put(tr, 1 + warp, j + 1);
      }
    }
    // Final: exchange (m, l) with the partner warp of this lane quarter, then
    // each warp writes d columns [64*half, +64) from both accumulators.
    float other_m = -INFINITY, other_l = 0.f;
    if (ok) {
      xchg[0][half][row] = m_run;
      xchg[1][half][row] = l;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar + q);
      ok = warp_wait(xbar + q, 0, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag);
      if (ok) {
        other_m = xchg[0][half ^ 1][row];
        other_l = xchg[1][half ^ 1][row];
      }
    }
    if (ok && warp_wait(o_done, (nkb - 1) & 1, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag)) {
      tc_fence_after();
      const float m_tot = fmaxf(m_run, other_m);  // finite: column 0 of every row is unmasked
      const float w_me = ex2(m_run - m_tot), w_other = ex2(other_m - m_tot);
      const float l_tot = l * w_me + other_l * w_other;
      const float inv = 1.f / l_tot;
      const float w0 = (half == 0 ? w_me : w_other) * inv, w1 = (half == 0 ? w_other : w_me) * inv;
      const int qidx = q0 + row;
      if (half == 0) lse[int64_t(bh) * S + qidx] = (m_tot + log2f(l_tot)) / kLog2e;
      // Stage 32 rows x 64 columns (128 B per row) of this warp through smem (Q tile is dead).
      uint8_t* stg = sm + kSmQ + (q * 2 + half) * 4096;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t r0[32], r1[32];
        const uint32_t col = uint32_t(half * 64 + c * 32);
        tmem_ld_32x32b_x32(tmem + lane_base + 256 + col, r0);
        tmem_ld_32x32b_x32(tmem + lane_base + 384 + col, r1);
        tmem_wait_ld();
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = fmaf(__uint_as_float(r0[i]), w0, __uint_as_float(r1[i]) * w1);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint4 pk;
          pk.x = pack2(o[8 * u + 0], o[8 * u + 1]);
          pk.y = pack2(o[8 * u + 2], o[8 * u + 3]);
          pk.z = pack2(o[8 * u + 4], o[8 * u + 5]);
          pk.w = pack2(o[8 * u + 6], o[8 * u + 7]);
          const int unit = c * 4 + u;  // 8 units of 16 B per 64-column row
          *reinterpret_cast<uint4*>(stg + lane * 128 + ((unit ^ (lane & 7)) << 4)) = pk;
        }
      }
      __syncwarp();
      __nv_bfloat16* og = out + int64_t(row0 + q0 + q * 32) * ld_out + h * kD + half * 64;
#pragma unroll 4
      for (int i = lane; i < 32 * 8; i += 32) {
        const int r = i / 8, unit = i % 8;
        *reinterpret_cast<uint4*>(og + int64_t(r) * ld_out + unit * 8) =
            *reinterpret_cast<const uint4*>(stg + r * 128 + ((unit ^ (r & 7)) << 4));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
    if (lane == 0) trace_put(tr, 0, tsm | 3);
  }
}

// ============================================================================
// Backward.  D = rowsum(dO * O) comes from a small pre-pass.  Two kernels, no
// float atomics (deterministic):
//   dK/dV: CTA per 128-key block; for each query block i >= the key block:
//          S^T = K Q_i^T and dP^T = V dO_i^T into TMEM; the elementwise warps
//          write P^T = exp2(S^T*scale*log2e - LSE_i*log2e) and
//          dS^T = P^T (dP^T - D_i) back as packed BF16; then
//          dV += P^T dO_i and dK += dS^T Q_i (A from TMEM; Q_i / dO_i reused as
//          MN-major operands from the same 128-byte-swizzled smem tiles).
//   dQ:    CTA per 128-query block; for each key block j <= the query block:
//          S = Q K_j^T, dP = dO V_j^T; dS = P (dP - D); dQ += dS K_j.
// ============================================================================
// Optional per-CTA cycle counters of the backward kernels (8 words per CTA,
// CTA id blockIdx.y * gridDim.x + blockIdx.x; each word has one writer):
// [0] MMA thread waiting for Q/dO or K/V tiles, [1] waiting for the
// elementwise warps, [2] waiting for the previous block's MMAs, [3] MMA thread
// total; [4] elementwise warp 2 waiting for S/dP, [5] its elementwise work,
// [6] blocks.
// The counters compile away in the kernels launched without them (kOn false).
template <bool kOn>
struct BwdTrace {
  unsigned long long* w;
  __device__ long long now() const {
    if constexpr (kOn) return clock64();
    return 0;
  }
  __device__ void add(int i, long long since) const {
    if constexpr (kOn) w[i] += (unsigned long long)(clock64() - since);
  }
  __device__ void count(int i) const {
    if constexpr (kOn) w[i] += 1;
  }
};

constexpr int kBwdSmTotal = 6 * 32768 + 2048 + 256 + 1024;

// cp.async.bulk (non-tensor) global -> shared, completion counted on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Elementwise pass over one 32-column quarter (`quarter`) of a 128-column
// score row held in TMEM: reads S (cols s_col+32*quarter..+32) and dP
// (dp_col+32*quarter..+32) and writes P / dS as packed BF16 into the first 16
// of those same 32 columns, so the four warps sharing a lane quarter never
// touch each other's columns.  The MMA reads packed chunk kk (16 BF16 values)
// at column bwd_packed_col(kk).
// kColumnStats: per-column LSE/D from smem (dK/dV kernel) or per-row values.
__device__ __forceinline__ uint32_t bwd_packed_col(int kk) { return uint32_t((kk >> 1) * 32 + (kk & 1) * 8); }
template <bool kColumnStats>
__device__ __forceinline__ void softmax_grad_row(uint32_t tmem, uint32_t lane_base, uint32_t s_col, uint32_t dp_col,
                                                 float sl2, const float* lse_s, const float* d_s, float lse_row2,
                                                 float d_row, int row, bool diag, bool write_p, int quarter) {
  {
    uint32_t rs[32], rd[32];
    tmem_ld_32x32b_x32(tmem + lane_base + s_col + quarter * 32, rs);
    tmem_ld_32x32b_x32(tmem + lane_base + dp_col + quarter * 32, rd);
    tmem_wait_ld();
    uint32_t wp[16], wd[16];
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      float pp[2], dd[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int c = quarter * 32 + i + e;
        const float l2 = kColumnStats ? lse_s[c] : lse_row2;
        const float dv = kColumnStats ? d_s[c] : d_row;
        // dK/dV: rows are keys, columns queries -> masked when query < key.
        // dQ:    rows are queries, columns keys -> masked when key > query.
        const bool masked = diag && (kColumnStats ? (c < row) : (c > row));
        const float p = masked ? 0.f : ex2(fmaf(__uint_as_float(rs[i + e]), sl2, -l2));
        pp[e] = p;
        dd[e] = p * (__uint_as_float(rd[i + e]) - dv);
      }
      wp[i / 2] = pack2(pp[0], pp[1]);
      wd[i / 2] = pack2(dd[0], dd[1]);
    }
    const uint32_t packed = uint32_t(quarter * 32);
    if (write_p) tmem_st_32x32b_x16(tmem + lane_base + s_col + packed, wp);
    tmem_st_32x32b_x16(tmem + lane_base + dp_col + packed, wd);
  }
  tmem_wait_st();
}

// Write 32 rows x 64 columns (fp32 in TMEM, scaled) of this warp as BF16.
__device__ __forceinline__ void store_tmem_rows(uint32_t tmem_row, float mul, uint8_t* stg, __nv_bfloat16* g,
                                                int64_t ld, int lane) {
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(tmem_row + c * 32, r);
    tmem_wait_ld();
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint4 pk;
      pk.x = pack2(__uint_as_float(r[8 * u + 0]) * mul, __uint_as_float(r[8 * u + 1]) * mul);
      pk.y = pack2(__uint_as_float(r[8 * u + 2]) * mul, __uint_as_float(r[8 * u + 3]) * mul);
      pk.z = pack2(__uint_as_float(r[8 * u + 4]) * mul, __uint_as_float(r[8 * u + 5]) * mul);
      pk.w = pack2(__uint_as_float(r[8 * u + 6]) * mul, __uint_as_float(r[8 * u + 7]) * mul);
      const int unit = c * 4 + u;
      *reinterpret_cast<uint4*>(stg + lane * 128 + ((unit ^ (lane & 7)) << 4)) = pk;
    }
  }
  __syncwarp();
#pragma unroll 4
  for (int i = lane; i < 32 * 8; i += 32) {
    const int r = i / 8, unit = i % 8;
    *reinterpret_cast<uint4*>(g + int64_t(r) * ld + unit * 8) =
        *reinterpret_cast<const uint4*>(stg + r * 128 + ((unit ^ (r & 7)) << 4));
  }
  __syncwarp();
}

template <bool kTrace>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                            const float* __restrict__ lse, const float* __restrict__ Dvec,
                            __nv_bfloat16* __restrict__ dqkv, int64_t ld_dqkv, int S, int H, float scale,
                            int* status, uint64_t timeout_ns,
                            unsigned long long* dbg) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [K 32K][V 32K][Q st0 32K][Q st1 32K][dO st0 32K][dO st1 32K][LSE/D 2 x 1K][bars]
  uint8_t* sK = sm;
  uint8_t* sV = sm + 32768;
  uint8_t* sQ = sm + 65536;
  uint8_t* sO = sm + 65536 + 65536;
  float* sStat = reinterpret_cast<float*>(sm + 6 * 32768);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 6 * 32768 + 2048);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;
  uint64_t* q_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* p_full = bars + 6;
  uint64_t* done = bars + 7;
  uint64_t* mma_done = bars + 8;  // dV/dK MMAs of a block completed (they read P^T, dS^T in TMEM)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const BwdTrace<kTrace> trc{kTrace ? dbg + 8 * (size_t(blockIdx.y) * gridDim.x + blockIdx.x) : nullptr};
  // Grid (B*H, S/128), x-fastest: small key blocks carry the most query blocks
  // and run first for every head.
  const int bh = blockIdx.x;
  const int kb = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int row0 = b * S;
  const int k0 = kb * kBlk;
  const int nqb = S / kBlk;
  const int nblk = nqb - kb;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(q_full + i, 1);
      mbar_init(q_empty + i, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, kBwdEwWarps);
    mbar_init(done, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tdo);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 65536);
      tma_load_2d(sK, &tq, kv_full, (H + h) * kD, row0 + k0);
      tma_load_2d(sK + 16384, &tq, kv_full, (H + h) * kD + 64, row0 + k0);
      tma_load_2d(sV, &tq, kv_full, (2 * H + h) * kD, row0 + k0);
      tma_load_2d(sV + 16384, &tq, kv_full, (2 * H + h) * kD + 64, row0 + k0);
      for (int t = 0; t < nblk; ++t) {
        const int i = kb + t, st = t & 1;
        if (!mbar_wait(q_empty + st, ((t >> 1) & 1) ^ 1, timeout_ns, status, kTimeoutProducerEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(q_full + st, 65536 + 1024);
        tma_load_2d(sQ + st * 32768, &tq, q_full + st, h * kD, row0 + i * kBlk);
        tma_load_2d(sQ + st * 32768 + 16384, &tq, q_full + st, h * kD + 64, row0 + i * kBlk);
        tma_load_2d(sO + st * 32768, &tdo, q_full + st, h * kD, row0 + i * kBlk);
        tma_load_2d(sO + st * 32768 + 16384, &tdo, q_full + st, h * kD + 64, row0 + i * kBlk);
        bulk_load(sStat + st * 256, lse + int64_t(bh) * S + i * kBlk, 512, q_full + st);
        bulk_load(sStat + st * 256 + 128, Dvec + int64_t(bh) * S + i * kBlk, 512, q_full + st);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc_kk = make_idesc_bf16(128, 128, 0, 0);
      const uint32_t idesc_tm = make_idesc_bf16(128, 128, 0, 1);
      const long long t_start = trc.now();
      long long tw = trc.now();
      bool ok = mbar_wait(kv_full, 0, timeout_ns, status, kTimeoutMmaFull, abort_flag);
      trc.add(0, tw);
      tc_fence_after();
      const uint32_t kbase = smem_u32(sK), vbase = smem_u32(sV);
      for (int t = 0; t < nblk && ok; ++t) {
        const int st = t & 1;
        tw = trc.now();
        if (!mbar_wait(q_full + st, (t >> 1) & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) { ok = false; break; }
        trc.add(0, tw);
        tw = trc.now();
        // S^T_t / dP^T_t overwrite the P^T / dS^T that block t-1's dV/dK MMAs
        // read from TMEM; an MMA's TMEM A-operand reads are not ordered with a
        // later MMA's accumulator writes, so wait for those MMAs to complete.
        if (t > 0 && !mbar_wait(mma_done, (t - 1) & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) {
          ok = false;
          break;
        }
        trc.add(2, tw);
        tc_fence_after();
        const uint32_t qb = smem_u32(sQ + st * 32768), ob = smem_u32(sO + st * 32768);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) umma_f16(tmem, kmajor_desc(kbase, kk), kmajor_desc(qb, kk), idesc_kk, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16(tmem + 128, kmajor_desc(vbase, kk), kmajor_desc(ob, kk), idesc_kk, kk > 0);
        umma_commit(s_full);
        tw = trc.now();
        if (!mbar_wait(p_full, t & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) { ok = false; break; }
        trc.add(1, tw);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_tmem_a(tmem + 256, tmem + bwd_packed_col(kk), mnmajor_desc(ob, kk), idesc_tm, (t > 0 || kk > 0));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_f16_tmem_a(tmem + 384, tmem + 128 + bwd_packed_col(kk), mnmajor_desc(qb, kk), idesc_tm,
                          (t > 0 || kk > 0));
        umma_commit(q_empty + st);
        umma_commit(mma_done);
      }
      umma_commit(done);
      mbar_wait(done, 0, timeout_ns, status, kTimeoutDrain, nullptr);
      trc.add(3, t_start);
    }
  } else {
    const int q = warp & 3;            // TMEM lane quarter (key rows)
    const int cq = (warp - 2) >> 2;    // 32-column quarter of the query block
    const int half = cq;               // readout: warps of column quarters 0, 1 write 64 columns each
    const int row = q * 32 + lane;  // key row within the block
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    const float sl2 = scale * kLog2e;
    __shared__ float lse_l2[kBwdEwWarps][128];
    const int ew = warp - 2;
    bool ok = true;
    const bool tracer = warp == 2 && lane == 0;
    for (int t = 0; t < nblk; ++t) {
      const int st = t & 1;
      const long long tw = tracer ? trc.now() : 0;
      if (!warp_wait(s_full, t & 1, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag)) { ok = false; break; }
      if (tracer) trc.add(4, tw);
      const long long tk = tracer ? trc.now() : 0;
      // q_full(t) has completed before the MMA warp issued S^T(t): the stats are in smem.
      tc_fence_after();
      const float* ls = sStat + st * 256;
      const float* ds = sStat + st * 256 + 128;
      // Per-column LSE in log2 units for this warp's 32 columns (its own copy).
      lse_l2[ew][cq * 32 + lane] = ls[cq * 32 + lane] * kLog2e;
      __syncwarp();
      softmax_grad_row<true>(tmem, lane_base, 0, 128, sl2, lse_l2[ew], ds, 0.f, 0.f, row, t == 0, true, cq);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (tracer) {
        trc.add(5, tk);
        trc.count(6);
      }
    }
    if (cq < 2 && ok && warp_wait(done, 0, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag)) {
      tc_fence_after();
      uint8_t* stg = sQ + (q * 2 + half) * 4096;  // Q stage 0 is dead after the last MMA
      __nv_bfloat16* dK = dqkv + int64_t(row0 + k0 + q * 32) * ld_dqkv + (H + h) * kD + half * 64;
      __nv_bfloat16* dV = dqkv + int64_t(row0 + k0 + q * 32) * ld_dqkv + (2 * H + h) * kD + half * 64;
      store_tmem_rows(tmem + lane_base + 256 + half * 64, 1.f, stg, dV, ld_dqkv, lane);
      store_tmem_rows(tmem + lane_base + 384 + half * 64, scale, stg, dK, ld_dqkv, lane);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool kTrace>
__global__ void __launch_bounds__(kBwdThreads, 1)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tdo,
                          const float* __restrict__ lse, const float* __restrict__ Dvec,
                          __nv_bfloat16* __restrict__ dqkv, int64_t ld_dqkv, int S, int H, float scale,
                          int* status, uint64_t timeout_ns,
                          unsigned long long* dbg) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // [Q 32K][dO 32K][K st0 32K][K st1 32K][V st0 32K][V st1 32K][bars]
  uint8_t* sQ = sm;
  uint8_t* sO = sm + 32768;
  uint8_t* sK = sm + 65536;
  uint8_t* sV = sm + 65536 + 65536;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + 6 * 32768 + 2048);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;    // S_j and dP_j in TMEM
  uint64_t* consumed = bars + 6;  // every elementwise warp holds its S_j, dP_j in registers
  uint64_t* p_full = bars + 7;    // dS_j written (packed BF16, columns of its own)
  uint64_t* dq_done = bars + 8;   // dQ += dS_j K_j finished reading dS_j
  uint64_t* done = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const BwdTrace<kTrace> trc{kTrace ? dbg + 8 * (size_t(blockIdx.y) * gridDim.x + blockIdx.x) : nullptr};
  const int bh = blockIdx.x;  // grid (B*H, S/128), x-fastest: heavy query tiles first
  const int qt = int(gridDim.y) - 1 - int(blockIdx.y);
  const int b = bh / H, h = bh % H;
  const int row0 = b * S;
  const int q0 = qt * kBlk;
  const int nkb = qt + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(kv_full + i, 1);
      mbar_init(kv_empty + i, 1);
    }
    mbar_init(s_full, 1);
    mbar_init(consumed, kBwdEwWarps);
    mbar_init(p_full, kBwdEwWarps);
    mbar_init(dq_done, 1);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tdo);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 65536);
      tma_load_2d(sQ, &tq, q_full, h * kD, row0 + q0);
      tma_load_2d(sQ + 16384, &tq, q_full, h * kD + 64, row0 + q0);
      tma_load_2d(sO, &tdo, q_full, h * kD, row0 + q0);
      tma_load_2d(sO + 16384, &tdo, q_full, h * kD + 64, row0 + q0);
      for (int j = 0; j < nkb; ++j) {
        const int st = j & 1;
        if (!mbar_wait(kv_empty + st, ((j >> 1) & 1) ^ 1, timeout_ns, status, kTimeoutProducerEmpty, abort_flag)) break;
        mbar_arrive_expect_tx(kv_full + st, 65536);
        tma_load_2d(sK + st * 32768, &tq, kv_full + st, (H + h) * kD, row0 + j * kBlk);
        tma_load_2d(sK + st * 32768 + 16384, &tq, kv_full + st, (H + h) * kD + 64, row0 + j * kBlk);
        tma_load_2d(sV + st * 32768, &tq, kv_full + st, (2 * H + h) * kD, row0 + j * kBlk);
        tma_load_2d(sV + st * 32768 + 16384, &tq, kv_full + st, (2 * H + h) * kD + 64, row0 + j * kBlk);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // TMEM: S [0,128), dP [128,256), dQ [256,384), dS packed BF16 [384,448).
      // dS has columns of its own, so S_j and dP_j are issued as soon as every
      // elementwise warp holds S_{j-1}, dP_{j-1} in registers (`consumed`) and
      // run while the warps compute dS_{j-1}; dQ += dS_{j-1} K_{j-1} follows.
      // No MMA writes columns that an earlier MMA reads as its A operand.
      const uint32_t idesc_kk = make_idesc_bf16(128, 128, 0, 0);
      const uint32_t idesc_tm = make_idesc_bf16(128, 128, 0, 1);
      const long long t_start = trc.now();
      long long tw = trc.now();
      bool ok = mbar_wait(q_full, 0, timeout_ns, status, kTimeoutMmaFull, abort_flag);
      trc.add(0, tw);
      tc_fence_after();
      const uint32_t qbase = smem_u32(sQ), obase = smem_u32(sO);
      for (int j = 0; j <= nkb && ok; ++j) {
        if (j < nkb) {
          const int st = j & 1;
          tw = trc.now();
          if (!mbar_wait(kv_full + st, (j >> 1) & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) { ok = false; break; }
          trc.add(0, tw);
          tw = trc.now();
          if (j > 0 && !mbar_wait(consumed, (j - 1) & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) {
            ok = false;
            break;
          }
          trc.add(1, tw);
          tc_fence_after();
          const uint32_t kbase = smem_u32(sK + st * 32768), vbase = smem_u32(sV + st * 32768);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) umma_f16(tmem, kmajor_desc(qbase, kk), kmajor_desc(kbase, kk), idesc_kk, kk > 0);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16(tmem + 128, kmajor_desc(obase, kk), kmajor_desc(vbase, kk), idesc_kk, kk > 0);
          umma_commit(s_full);
        }
        if (j > 0) {
          const int pj = j - 1, pst = pj & 1;
          tw = trc.now();
          if (!mbar_wait(p_full, pj & 1, timeout_ns, status, kTimeoutMmaFull, abort_flag)) { ok = false; break; }
          trc.add(1, tw);
          tc_fence_after();
          const uint32_t kbase = smem_u32(sK + pst * 32768);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16_tmem_a(tmem + 256, tmem + 384 + uint32_t(8 * kk), mnmajor_desc(kbase, kk), idesc_tm,
                            (pj > 0 || kk > 0));
          umma_commit(kv_empty + pst);
          umma_commit(dq_done);
        }
      }
      umma_commit(done);
      mbar_wait(done, 0, timeout_ns, status, kTimeoutDrain, nullptr);
      trc.add(3, t_start);
    }
  } else {
    const int q = warp & 3;            // TMEM lane quarter (query rows)
    const int cq = (warp - 2) >> 2;    // 32-column quarter of the key block
    const int half = cq;               // readout: warps of column quarters 0, 1 write 64 columns each
    const int row = q * 32 + lane;
    const uint32_t lane_base = uint32_t(q * 32) << 16;
    const float sl2 = scale * kLog2e;
    const float lse2 = lse[int64_t(bh) * S + q0 + row] * kLog2e;
    const float drow = Dvec[int64_t(bh) * S + q0 + row];
    bool ok = true;
    const bool tracer = warp == 2 && lane == 0;
    for (int j = 0; j < nkb; ++j) {
      const long long tw = tracer ? trc.now() : 0;
      if (!warp_wait(s_full, j & 1, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag)) { ok = false; break; }
      if (tracer) trc.add(4, tw);
      const long long tk = tracer ? trc.now() : 0;
      tc_fence_after();
      uint32_t rs[32], rd[32];
      tmem_ld_32x32b_x32(tmem + lane_base + uint32_t(cq * 32), rs);
      tmem_ld_32x32b_x32(tmem + lane_base + uint32_t(128 + cq * 32), rd);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(consumed);
      // dS = P (dP - D), P = exp2(S * scale * log2e - LSE * log2e); keys > query masked.
      const bool diag = j == nkb - 1;
      uint32_t wd[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        float dd[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int c = cq * 32 + i + e;
          const bool masked = diag && (c > row);
          const float p = masked ? 0.f : ex2(fmaf(__uint_as_float(rs[i + e]), sl2, -lse2));
          dd[e] = p * (__uint_as_float(rd[i + e]) - drow);
        }
        wd[i / 2] = pack2(dd[0], dd[1]);
      }
      // dQ += dS_{j-1} K_{j-1} must have read the dS columns before they are rewritten.
      if (j > 0 && !warp_wait(dq_done, (j - 1) & 1, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tmem_st_32x32b_x16(tmem + lane_base + uint32_t(384 + cq * 16), wd);  // key chunks 2cq, 2cq+1
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
      if (tracer) {
        trc.add(5, tk);
        trc.count(6);
      }
    }
    if (cq < 2 && ok && warp_wait(done, 0, timeout_ns, status, kTimeoutEpiTmemFull, abort_flag)) {
      tc_fence_after();
      uint8_t* stg = sK + (q * 2 + half) * 4096;
      __nv_bfloat16* dQ = dqkv + int64_t(row0 + q0 + q * 32) * ld_dqkv + h * kD + half * 64;
      store_tmem_rows(tmem + lane_base + 256 + half * 64, scale, stg, dQ, ld_dqkv, lane);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
}  // namespace

int attention_fwd_tc(const void* qkv, int64_t ld_qkv, void* out, int64_t ld_out, float* lse, int B, int S,
                     int H, float scale, int* status, uint64_t timeout_ns, cudaStream_t s,
                     unsigned long long* trace) {
  if (S % kBlk || ld_qkv % 8 || ld_out % 8 || (reinterpret_cast<uintptr_t>(qkv) & 15)) return -1;
  CUtensorMap map;
  if (!make_map(&map, qkv, uint64_t(3) * H * kD, uint64_t(B) * S, uint64_t(ld_qkv))) return -1;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmTotal);
    configured[dev] = true;
  }
  dim3 grid(B * H, S / kBlk);
  attn_fwd_tc_kernel<<<grid, kThreads, kSmTotal, s>>>(map, static_cast<__nv_bfloat16*>(out), ld_out, lse, S, H,
                                                      scale, status, timeout_ns, trace);
  return int(cudaGetLastError());
}

int attention_bwd_tc(const void* qkv, int64_t ld_qkv, const void* dout, int64_t ld_dout, const float* lse,
                     const float* Dvec, void* dqkv, int64_t ld_dqkv, int B, int S, int H, float scale, int* status,
                     uint64_t timeout_ns, cudaStream_t s, unsigned long long* dbg_dkdv,
                     unsigned long long* dbg_dq) {
  if (S % kBlk || ld_qkv % 8 || ld_dout % 8 || ld_dqkv % 8) return -1;
  CUtensorMap mq, mo;
  if (!make_map(&mq, qkv, uint64_t(3) * H * kD, uint64_t(B) * S, uint64_t(ld_qkv))) return -1;
  if (!make_map(&mo, dout, uint64_t(H) * kD, uint64_t(B) * S, uint64_t(ld_dout))) return -1;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmTotal);
    cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmTotal);
    cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmTotal);
    cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmTotal);
    configured[dev] = true;
  }
  dim3 grid(B * H, S / kBlk);
  __nv_bfloat16* dq = static_cast<__nv_bfloat16*>(dqkv);
  if (dbg_dkdv && dbg_dq) {
    attn_bwd_dkdv_tc_kernel<true><<<grid, kBwdThreads, kBwdSmTotal, s>>>(mq, mo, lse, Dvec, dq, ld_dqkv, S, H, scale,
                                                                        status, timeout_ns, dbg_dkdv);
    attn_bwd_dq_tc_kernel<true><<<grid, kBwdThreads, kBwdSmTotal, s>>>(mq, mo, lse, Dvec, dq, ld_dqkv, S, H, scale,
                                                                      status, timeout_ns, dbg_dq);
  } else {
    attn_bwd_dkdv_tc_kernel<false><<<grid, kBwdThreads, kBwdSmTotal, s>>>(mq, mo, lse, Dvec, dq, ld_dqkv, S, H, scale,
                                                                         status, timeout_ns, nullptr);
    attn_bwd_dq_tc_kernel<false><<<grid, kBwdThreads, kBwdSmTotal, s>>>(mq, mo, lse, Dvec, dq, ld_dqkv, S, H, scale,
                                                                       status, timeout_ns, nullptr);
  }
  return int(cudaGetLastError());
}

}  // namespace kernels
}  // namespace tn5b
