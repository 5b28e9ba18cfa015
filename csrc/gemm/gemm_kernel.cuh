// Persistent, warp-specialised BF16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   C[M, N] = A[M, K] * B[N, K]^T          (fp32 accumulation in tensor memory)
//
// A and B may each be K-major (row-major [rows, K]) or MN-major (row-major
// [K, rows]); the operand major is carried by the TMA box shape and the UMMA
// descriptors, so forward (TN), dgrad (TT) and wgrad (NT) GEMMs all run here.
//
// CTA roles (192 threads):
//   warp 0      TMA producer: one elected lane streams A/B k-blocks into a
//               STAGES-deep shared-memory ring (128-byte swizzle).
//   warp 1      MMA issuer: allocates TMEM (512 columns: 2 accumulators x BN,
//               or one 2*BN accumulator for the wide pair tile), one lane
//               issues tcgen05.mma (K=16) and commits to mbarriers that free
//               smem stages / publish accumulators.
//   warps 2..5  epilogue: tcgen05.ld accumulator rows (warp w owns TMEM lanes
//               32*(w%4)..+31), apply the fused epilogue, stage through a
//               swizzled smem buffer and write coalesced 16-byte stores.
//
// The grid is persistent (<= one CTA per SM); CTA c walks tiles c, c+grid, ...
// of a tile order that is either a grouped raster (plain GEMMs) or an explicit
// table (reduce-scatter schedules: destination-major / interleaved / arrival).
//
// Every wait is bounded (see ptx.cuh); on a timeout the CTA records a status
// code, drains its in-flight TMA loads and MMAs, frees TMEM and returns.
//
// Reference parity: this replaces the CUTLASS Sm80 mma.sync GEMM with the
// OrderedDPSwizzle tile order of src/gemm/native.cu:33-114 (TempName-5090).
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include "../common/ptx.cuh"
#include "gemm_api.h"
#include "../common/push_lanes.h"

namespace tn5b {
namespace gemm {

constexpr int kBM = 128;             // UMMA M (one CTA, cta_group::1)
constexpr int kBK = 64;              // k-block: 64 bf16 = one 128-byte swizzle row
constexpr int kUmmaK = 16;           // K per tcgen05.mma for 16-bit inputs
constexpr int kThreads = 192;
// Pull reduce-scatter launches carry two more 128-thread groups: in the reducer
// CTAs they reduce alternate pieces (the GEMM CTAs' extra warps exit at once).
constexpr int kRedGroups = 2;
template <int MODE>
constexpr int kThreadsFor = MODE == 3 ? 64 + kRedGroups * 128 : kThreads;
constexpr int kEpiWarps = 4;
constexpr int kEpiFirstWarp = 2;

enum EpiFlags : int {
  kEpiBias = 1,        // + bias[n] (fp32 add before rounding)
  kEpiGelu = 2,        // aux = bf16(acc+bias); out = bf16(gelu(aux))
  kEpiResidual = 4,    // out = bf16(bf16(res + bf16(acc)) + bias)
  kEpiAccumulate = 8,  // out = bf16(float(out) + acc)
  kEpiGeluBwd = 16,    // out = bf16(bf16(acc) * gelu'(aux)), aux = saved pre-activation (input)
};

// Modes of the epilogue destination.
enum Mode : int {
  kModeLocal = 0,      // plain store into C
  kModeRsPush = 1,     // GEMM -> reduce-scatter: BF16 tile pushed to its owner rank
  kModeRsTaco = 2,     // GEMM -> reduce-scatter: remote tiles TACO-encoded, then pushed
  kModeRsPull = 3,     // GEMM -> reduce-scatter: partial tiles stored locally and published;
                       // the owner's reducer CTAs (same launch) pull and reduce them
};

struct RsArgs {
  // Peer base pointers of every rank's receive regions and flags (index =
  // rank).  Push transport: two lanes per owner (block parity), each with its
  // own receive region [source][lane blocks] and flag array [source][lane
  // tiles] (PushLanes, push_lanes.h).  Pull transport: flag[source * tiles_per_dest + t].
  uint8_t* const* recv;          // device array [world]
  uint32_t* const* flags;        // device array [world]
  int rank, world;
  int rows_per_dest;             // M / world
  int chunk_rows;                // block rows (reference macroblock; lane = block parity)
  uint32_t epoch;
  PushLanes lanes;               // push transport layout of every owner's regions
  // Diagnostic only (never in timed paths): delay the flag publication of one
  // tile (linear id) by a bounded `delay_ns` to create artificial lane skew.
  int delay_tile;
  uint64_t delay_ns;
};

// All-gather -> GEMM (pull): chunk c of the gathered A ([M/W rows, K] of rank
// c) arrives in this rank's gather buffer block by block (128 rows);
// ready[c][block] is set to the call's epoch once the block is stored.
// Counters sit kReadyStride words apart (one 128-byte line each, gemm_api.h),
// so GEMM CTAs polling one block do not contend with gatherers updating another.
struct GatherArgs {
  uint8_t* const* gather;          // device array [world]: every rank's gather buffer ([M, K] bf16)
  uint32_t* const* published;      // device array [world]: every rank's published[world][blocks] flags
  uint32_t* const* pulled;         // device array [world]: every rank's pulled counter
  const uint32_t* published_local; // this rank's published[world][blocks]
  const uint32_t* pulled_local;    // this rank's pulled counter
  uint32_t* ready;                 // local [world][rows_per_src / 128] counters, kReadyStride apart
  const uint8_t* shard;            // local shard [rows_per_src, K] bf16 (contiguous)
  int64_t chunk_bytes;             // rows_per_src * K * 2
  int rank, world, rows_per_src, K;
  uint32_t epoch;                  // this call's epoch (published block flags)
  uint32_t pulled_target;          // pulled value once every peer finished reading the previous call
  uint32_t ready_target;           // ready[c][b] once block b of chunk c has arrived (the epoch)
  int phase;                       // communication CTAs: bit0 own chunk + publish, bit1 pull peers
  int own_in_place;                // the shard already is the own chunk of the gather buffer: publish only
  unsigned long long* block_stamps; // optional [world * rows_per_src / 128]: when each block was stored
};

// GEMM -> reduce-scatter (pull): the reducer CTAs' view.  Flags are per
// "flag tile" of 128 rows x tile_n columns of the owner's rows.
struct PullRsArgs {
  const uint8_t* const* partial;   // device array [world]: partial buffers, [M/128][N/64][128][64] bf16
  const uint32_t* my_flags;        // local [world][tiles_per_dest]
  const int* order;                // consumption order of local flag tiles (null: 0, 1, ...)
  int tiles_per_dest, tiles_n;     // flag tiles per destination / per row
  __nv_bfloat16* out;              // [rows_per_dest, N]
  const __nv_bfloat16* residual;   // optional [rows_per_dest, N]
  const __nv_bfloat16* bias;       // optional [N]
  unsigned long long* stamps;      // optional: %globaltimer at each local flag tile's completion
  unsigned long long* produced;    // optional: %globaltimer at each produced flag tile's publication
};

struct Params {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles, k_blocks;
  int group_m;                   // raster group (plain GEMMs)
  // Tail launch of a split GEMM: linear tile t is half (t % 2) of tile
  // tail_from + t / 2 of the main launch's grouped raster over a grid of
  // tail_tiles_m x tail_tiles_n wide (256 x 2*BN) tiles; tail_from < 0 otherwise.
  int tail_from, tail_tiles_m, tail_tiles_n;
  const int* tile_order;         // optional: linear tile ids (tm * tiles_n + tn)
  // epilogue
  int epi;
  __nv_bfloat16* out; int64_t ldo;
  __nv_bfloat16* aux; int64_t ld_aux;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual; int64_t ld_res;
  RsArgs rs;
  GatherArgs gather;
  PullRsArgs pull;
  int comm_ctas;                 // CTAs [0, comm_ctas) run the communication role (dispatched first:
                                 // GEMM CTAs may wait on them, never the reverse)
  int gemm_ctas;                 // CTAs [comm_ctas, comm_ctas + gemm_ctas) compute
  int tma_store;                 // local mode: store the output tile with TMA (tmap_out)
  int* status;
  uint64_t timeout_ns;
  // Optional per-CTA cycle counters (profiling), 8 words per CTA: [0] MMA wait
  // for a loaded stage, [1] MMA role total, [2] producer wait for a free stage,
  // [3] epilogue wait for an accumulator (summed over its warps), [4] MMA wait
  // for a drained accumulator.
  unsigned long long* debug;
  // Optional [grid][2] %globaltimer stamps: start and end of every CTA (profiling).
  unsigned long long* cta_stamps;
};

template <int BN, int STAGES, int EPI_COLS, bool PAIR = false, bool WIDE = false, int STG_BUFS = 1>
struct SmemLayout {
  static constexpr int kABytes = kBM * kBK * 2;        // 16 KB
  // In a CTA pair each CTA holds half of B's N rows of every N=BN sub-tile
  // (two sub-tiles in the wide pair).
  static constexpr int kBSubBytes = (PAIR ? BN / 2 : BN) * kBK * 2;
  static constexpr int kBBytes = kBSubBytes * (WIDE ? 2 : 1);
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStagingBufBytes = 32 * EPI_COLS * 2;   // one warp's 32 rows x EPI_COLS bf16
  static constexpr int kStagingPerWarp = STG_BUFS * kStagingBufBytes;
  static constexpr int kStagingBytes = kEpiWarps * kStagingPerWarp;
  static constexpr int kBarrierBytes = 256;
  // [align 1024][stages][staging][barriers]
  static constexpr int kTotal = 1024 + STAGES * kStageBytes + kStagingBytes + kBarrierBytes;
};

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& tm, int& tn) {
  if (p.tile_order) {
    const int id = p.tile_order[t];
    tm = id / p.tiles_n;
    tn = id % p.tiles_n;
    return;
  }
  const bool tail = p.tail_from >= 0;
  const int tiles_m = tail ? p.tail_tiles_m : p.tiles_m;
  const int tiles_n = tail ? p.tail_tiles_n : p.tiles_n;
  const int u = tail ? p.tail_from + (t >> 1) : t;
  const int group_size = p.group_m * tiles_n;
  const int group = u / group_size;
  const int first_m = group * p.group_m;
  const int size_m = min(tiles_m - first_m, p.group_m);
  const int r = u % group_size;
  tm = first_m + r % size_m;
  tn = r / size_m;
  if (tail) tn = 2 * tn + (t & 1);  // the wide tile's two 256-column halves
}

__device__ __forceinline__ float bf16_round_f(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float gelu_exact(float x) {
  // 0.5 * x * (1 + erf(x / sqrt(2))), CUDA's erff called directly.
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

__device__ __forceinline__ float gelu_grad(float z) {
  // d/dz [z * Phi(z)] = Phi(z) + z * phi(z); erff / expf called directly.
  const float cdf = 0.5f * (1.0f + erff(z * 0.70710678118654752440f));
  const float pdf = 0.39894228040143267794f * expf(-0.5f * z * z);
  return cdf + z * pdf;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Swizzled staging: row r (0..31), 16-byte unit u -> byte offset.
template <int EPI_COLS>
__device__ __forceinline__ uint32_t staging_offset(int r, int u) {
  constexpr int kUnits = EPI_COLS / 8;  // 16-byte units per row
  return uint32_t(r * kUnits + (u ^ (r & 7))) * 16u;
}

// ===========================================================================
// TACO H128/E4M3 encode of one 128-element group held entirely by one thread.
// The FP32 operation sequence equals the warp-cooperative reference encoder
// (src/taco/codec.cu:69-103 of TempName-5090): the sum of squares follows its
// shuffle-down tree, the Walsh-Hadamard butterfly runs distances 1..64 in the
// same order with the same (lo+hi, lo-hi) operands, and every multiply, add,
// divide, rsqrtf and FP8 conversion is the same correctly-rounded operation,
// so packets are byte-identical.  Explicit _rn intrinsics forbid contraction.
// ===========================================================================
namespace taco {
constexpr float kNorm = 0.08838834764831844055f;

__device__ __forceinline__ float clampf(float x, float lo, float hi) {
  return fminf(fmaxf(x, lo), hi);
}

// Shuffle-down tree of one 32-lane warp_sum, evaluated for lane 0.
__device__ __forceinline__ float tree32(const float* a) {
  float b[16], c[8], d[4], e[2];
#pragma unroll
  for (int l = 0; l < 16; ++l) b[l] = __fadd_rn(a[l], a[l + 16]);
#pragma unroll
  for (int l = 0; l < 8; ++l) c[l] = __fadd_rn(b[l], b[l + 8]);
#pragma unroll
  for (int l = 0; l < 4; ++l) d[l] = __fadd_rn(c[l], c[l + 4]);
#pragma unroll
  for (int l = 0; l < 2; ++l) e[l] = __fadd_rn(d[l], d[l + 2]);
  return __fadd_rn(e[0], e[1]);
}

// x[c] holds element c (c = lane + 32*j in the reference layout).  On return
// x[c] holds the normalised Walsh coefficient c (natural order); the caller
// quantises each with e4m3(x[c] / quant) so no 128-byte code array is live.
__device__ __forceinline__ void encode_group(float (&x)[128], float& quant, float& adaptive) {
  float part[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float sq[32];
#pragma unroll
    for (int l = 0; l < 32; ++l) sq[l] = __fmul_rn(x[32 * j + l], x[32 * j + l]);
    part[j] = tree32(sq);
  }
  const float sum = __fadd_rn(__fadd_rn(part[0], part[2]), __fadd_rn(part[1], part[3]));
  const float variance = __fadd_rn(sum / 128.f, 1e-6f);
  adaptive = clampf(__fmul_rn(448.f, rsqrtf(fmaxf(variance, 1e-12f))), 1e-3f, 1e3f);
#pragma unroll
  for (int c = 0; c < 128; ++c) x[c] = __fmul_rn(x[c], adaptive);
#pragma unroll
  for (int d = 1; d < 128; d *= 2) {
#pragma unroll
    for (int c = 0; c < 128; ++c) {
      if ((c & d) == 0) {
        const float lo = x[c], hi = x[c + d];
        x[c] = __fadd_rn(lo, hi);
        x[c + d] = __fsub_rn(lo, hi);
      }
    }
  }
  float amax = 0.f;
#pragma unroll
  for (int c = 0; c < 128; ++c) {
    x[c] = __fmul_rn(x[c], kNorm);
    amax = fmaxf(amax, fabsf(x[c]));
  }
  quant = clampf(amax / 448.f, 1e-12f, 1e6f);
}
__device__ __forceinline__ uint32_t code(float x, float quant) {
  return uint32_t(__nv_cvt_float_to_fp8(x / quant, __NV_SATFINITE, __NV_E4M3)) & 0xFFu;
}
}  // namespace taco

// ===========================================================================
// The kernel.
// ===========================================================================
// PAIR: a cluster of two CTAs computes one 256 x BN tile with
// tcgen05.mma.cta_group::2 issued by the leader (cluster rank 0).  Each CTA
// TMA-loads its own 128 rows of A and its own BN/2 rows of B from this GPU's
// memory only; both CTAs' loads complete on the leader's "full"
// barrier, the leader's commits arrive on both CTAs' "empty" / "tmem full"
// barriers, and both CTAs' epilogues release the accumulator on the leader's
// "tmem empty" barrier.  Each CTA's TMEM holds its 128 rows x BN fp32.
// WIDE (implies PAIR): the pair's tile is 256 x 2*BN; every K step issues two
// N=BN MMAs that share the A operand, so each 48 KB stage feeds twice the
// tensor work of the 256 x BN pair tile (twice the latency cover per byte in
// flight).  The single 128 x 2*BN accumulator fills all 512 TMEM columns, so
// the next tile's MMAs wait for the epilogue (used for long K loops).
// Local-mode epilogues store the output tile with TMA (double-buffered staging
// per warp: the store of one 32 x EPI_COLS chunk overlaps the next chunk).
template <int BN, bool WIDE>
constexpr int kTileNOf = BN * (WIDE ? 2 : 1);

template <int MODE>
constexpr int kStagingBuffers = (MODE == kModeLocal || MODE == kModeRsPull) ? 2 : 1;

}  // namespace gemm
}  // namespace tn5b
#include "comm_roles.cuh"
namespace tn5b {
namespace gemm {

// AG: the A rows of chunk `rank` are read from the local shard (tmap_a2), the
// other chunks from the local gather buffer (tmap_a) once they have arrived.
// kModeRsPull: tmap_out maps the local partial buffer as a [M/128 * N/64 * 128, 64]
// matrix (tile-major pieces the reducer pulls with single bulk loads) and
// tmap_a2 the residual [M/W, N] that the reducer CTAs load tile by tile.
template <int BN, int STAGES, int EPI_COLS, int MODE, bool AG, bool PAIR = false, bool WIDE = false>
__global__ void __launch_bounds__(kThreadsFor<MODE>, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                const __grid_constant__ CUtensorMap tmap_b, const __grid_constant__ CUtensorMap tmap_out,
                const __grid_constant__ CUtensorMap tmap_a2, const __grid_constant__ Params p, int a_mn,
                int b_mn) {
  using L = SmemLayout<BN, STAGES, EPI_COLS, PAIR, WIDE, kStagingBuffers<MODE>>;
  static_assert(!PAIR || MODE == kModeLocal || MODE == kModeRsPull,
                "CTA pairs serve the local-store epilogues (plain and reduce-scatter partial)");
  static_assert(!WIDE || PAIR, "the wide tile is a CTA-pair tile");
  constexpr int kSub = WIDE ? 2 : 1;               // N=BN MMAs per K step
  constexpr int kTileN = BN * kSub;
  constexpr int kAccBufs = WIDE ? 1 : 2;           // TMEM accumulators
  constexpr int kTmemCols = kAccBufs * kTileN;     // 512 in every configuration
  static_assert(kTmemCols <= 512, "TMEM holds 512 columns");
  constexpr int kTileM = PAIR ? 2 * kBM : kBM;
  constexpr int kBRows = PAIR ? BN / 2 : BN;
  static_assert(BN % EPI_COLS == 0, "epilogue chunks must tile BN");
  static_assert(MODE != kModeRsTaco || EPI_COLS == 128, "TACO groups are 128 columns");
  static_assert(MODE != kModeRsPull || EPI_COLS == 64, "partial pieces are 64 columns wide");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  if (p.cta_stamps && threadIdx.x == 0) p.cta_stamps[2 * blockIdx.x] = globaltimer_ns();
  if (int(blockIdx.x) < p.comm_ctas) {
    // Communication role (no TMEM, no cluster barriers).
    if constexpr (MODE == kModeRsPull) rs_reducer<kTileNOf<BN, WIDE> / 64>(p, smem, &tmap_a2);
    else if constexpr (AG) ag_gatherer(p, smem);
    if (p.cta_stamps) {
      __syncthreads();
      if (threadIdx.x == 0) p.cta_stamps[2 * blockIdx.x + 1] = globaltimer_ns();
    }
    return;
  }
  uint8_t* stage_base = smem;
  uint8_t* staging = smem + STAGES * L::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(staging + L::kStagingBytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* tfull = bars + 2 * STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t cta_rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = cta_rank == 0;
  const int gid = int(blockIdx.x) - p.comm_ctas;  // GEMM CTA index (comm_ctas is even with CTA pairs)
  const int cluster_id = PAIR ? gid / 2 : gid;
  const int clusters = PAIR ? p.gemm_ctas / 2 : p.gemm_ctas;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps * (PAIR ? 2 : 1));
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if constexpr (AG) tma_prefetch_desc(&tmap_a2);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // peer barriers initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      long long dbg_empty = 0;
      int last_parity[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_parity[s] = -1;
      bool ok = true;
      int waited_chunk = -1;
      for (int t = cluster_id; t < p.num_tiles && ok; t += clusters) {
        int tm, tn;
        tile_coords(p, t, tm, tn);
        const int row_a = tm * kTileM + int(cta_rank) * kBM;   // this CTA's A rows
        const int row_b = tn * kTileN + int(cta_rank) * kBRows;  // this CTA's B rows (sub-tile 0)
        // A operand of this tile: AG reads its own chunk from the shard and waits
        // (bounded) until a peer chunk's 128-row block has fully arrived locally.
        const CUtensorMap* ta = &tmap_a;
        int ya = row_a;
        if constexpr (AG) {
          const int chunk = row_a / p.gather.rows_per_src;
          const int in_chunk = row_a - chunk * p.gather.rows_per_src;
          if (chunk == p.gather.rank) {
            ta = &tmap_a2;
            ya = in_chunk;
          } else {
            const int blk = chunk * (p.gather.rows_per_src / 128) + in_chunk / 128;
            if (blk != waited_chunk) {
              if (!wait_flag_geq_gpu(p.gather.ready + int64_t(blk) * kReadyStride, p.gather.ready_target,
                                     p.timeout_ns, p.status, kTimeoutAgChunk)) {
                *abort_flag = 1;
                ok = false;
                break;
              }
              fence_proxy_async_global();
              waited_chunk = blk;
            }
          }
        }
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const long long w0 = p.debug ? clock64() : 0;
          if (!mbar_wait(&empty[s], ph ^ 1, p.timeout_ns, p.status, kTimeoutProducerEmpty,
                         abort_flag)) {
            ok = false;
            break;
          }
          if (p.debug) dbg_empty += clock64() - w0;
          uint8_t* sa = stage_base + s * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          const int k0 = kb * kBK;
          if constexpr (PAIR) {
            // Both CTAs' bytes land on the leader's full barrier.
            const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * L::kStageBytes);
            if (!a_mn) {
              tma_load_2d_pair(sa, ta, fb, k0, ya);
            } else {
#pragma unroll
              for (int c = 0; c < kBM / 64; ++c) tma_load_2d_pair(sa + c * 8192, &tmap_a, fb, row_a + c * 64, k0);
            }
#pragma unroll
            for (int j = 0; j < kSub; ++j) {
              uint8_t* sbj = sb + j * L::kBSubBytes;
              const int rb = row_b + j * BN;
              if (!b_mn) {
                tma_load_2d_pair(sbj, &tmap_b, fb, k0, rb);
              } else {
#pragma unroll
                for (int c = 0; c < kBRows / 64; ++c) tma_load_2d_pair(sbj + c * 8192, &tmap_b, fb, rb + c * 64, k0);
              }
            }
          } else {
            mbar_arrive_expect_tx(&full[s], L::kStageBytes);
            if (!a_mn) {
              tma_load_2d(sa, ta, &full[s], k0, ya);
            } else {
#pragma unroll
              for (int c = 0; c < kBM / 64; ++c)
                tma_load_2d(sa + c * 8192, &tmap_a, &full[s], row_a + c * 64, k0);
            }
            if (!b_mn) {
              tma_load_2d(sb, &tmap_b, &full[s], k0, row_b);
            } else {
#pragma unroll
              for (int c = 0; c < BN / 64; ++c)
                tma_load_2d(sb + c * 8192, &tmap_b, &full[s], row_b + c * 64, k0);
            }
          }
          last_parity[s] = int(ph);
        }
      }
      if (p.debug) p.debug[gid * 8 + 2] = (unsigned long long)dbg_empty;
      if (!ok) {
        // Abort path: let every issued TMA load land before the CTA can exit.
        if (!PAIR) {
          for (int s = 0; s < STAGES; ++s)
            if (last_parity[s] >= 0)
              mbar_wait(&full[s], uint32_t(last_parity[s]), p.timeout_ns, p.status, kTimeoutDrain,
                        nullptr);
        } else {
          // The pair's full barriers live in the leader; loads are long complete
          // when a multi-second wait expires -- wait out their latency once more.
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 100000) __nanosleep(1000);
        }
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0 && leader) {
      long long dbg_full = 0, dbg_tempty = 0;
      const long long dbg_t0 = clock64();
      const uint32_t idesc = make_idesc_bf16(kTileM, BN, a_mn, b_mn);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = cluster_id; t < p.num_tiles && ok; t += clusters, ++local) {
        const int b = local % kAccBufs;
        const uint32_t use = uint32_t(local / kAccBufs);
        const long long we = p.debug ? clock64() : 0;
        if (!mbar_wait(&tempty[b], (use & 1) ^ 1, p.timeout_ns, p.status, kTimeoutMmaTmemEmpty,
                       abort_flag)) {
          ok = false;
          break;
        }
        if (p.debug) dbg_tempty += clock64() - we;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(b * kTileN);
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          const long long w0 = p.debug ? clock64() : 0;
          if (!mbar_wait(&full[s], ph, p.timeout_ns, p.status, kTimeoutMmaFull, abort_flag)) {
            ok = false;
            break;
          }
          if (p.debug) dbg_full += clock64() - w0;
          tc_fence_after();
          const uint32_t sa = smem_u32(stage_base + s * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            const uint64_t ad = a_mn ? make_sw128_desc(sa + k * 2048, 8192, 1024)
                                     : make_sw128_desc(sa + k * 32, 16, 1024);
#pragma unroll
            for (int j = 0; j < kSub; ++j) {
              const uint32_t sbj = sb + j * L::kBSubBytes;
              const uint64_t bd = b_mn ? make_sw128_desc(sbj + k * 2048, 8192, 1024)
                                       : make_sw128_desc(sbj + k * 32, 16, 1024);
              if constexpr (PAIR)
                umma_f16_pair(d_tmem + j * BN, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
              else
                umma_f16(d_tmem + j * BN, ad, bd, idesc, (kb | k) != 0 ? 1u : 0u);
            }
          }
          if constexpr (PAIR) {
            umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 0));
            umma_commit_pair(mapa_shared(smem_u32(&empty[s]), 1));
          } else {
            umma_commit(&empty[s]);
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          umma_commit_pair(mapa_shared(smem_u32(&tfull[b]), 0));
          umma_commit_pair(mapa_shared(smem_u32(&tfull[b]), 1));
        } else {
          umma_commit(&tfull[b]);
        }
      }
      // All issued MMAs must finish before TMEM is released (normal and abort path).
      if constexpr (PAIR)
        umma_commit_pair(mapa_shared(smem_u32(drain), 0));
      else
        umma_commit(drain);
      mbar_wait(drain, 0, p.timeout_ns, p.status, kTimeoutDrain, nullptr);
      if (p.debug) {
        p.debug[gid * 8 + 0] = (unsigned long long)dbg_full;
        p.debug[gid * 8 + 1] = (unsigned long long)(clock64() - dbg_t0);
        p.debug[gid * 8 + 4] = (unsigned long long)dbg_tempty;
      }
    }
  } else if (warp < kEpiFirstWarp + kEpiWarps) {
    // ------------------------------------------------------------- epilogue
    const int q = warp & 3;                       // TMEM lane quarter
    const int ew = warp - kEpiFirstWarp;          // staging buffer
    uint8_t* stg_base = staging + ew * L::kStagingPerWarp;
    int chunk_seq = 0;  // TMA-store chunks issued by this warp (staging buffer = parity)
    const bool tma_out = (MODE == kModeLocal && p.tma_store) || MODE == kModeRsPull;
    int local = 0;
    for (int t = cluster_id; t < p.num_tiles; t += clusters, ++local) {
      int tm, tn;
      tile_coords(p, t, tm, tn);
      const int b = local % kAccBufs;
      const uint32_t use = uint32_t(local / kAccBufs);
      int ok = 1;
      if (lane == 0) {
        const long long we = p.debug ? clock64() : 0;
        ok = mbar_wait(&tfull[b], use & 1, p.timeout_ns, p.status, kTimeoutEpiTmemFull,
                       abort_flag);
        if (p.debug) atomicAdd(p.debug + gid * 8 + 3, (unsigned long long)(clock64() - we));
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      const int row_w = tm * kTileM + int(cta_rank) * kBM + q * 32;  // first row of this warp
      const int my_row = row_w + lane;
      const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(b * kTileN);

      // Destination of this tile (reduce-scatter modes).
      int dest = 0;
      bool remote_taco = false;
      if constexpr (MODE != kModeLocal) {
        dest = (tm * kBM) / p.rs.rows_per_dest;
        remote_taco = (MODE == kModeRsTaco) && dest != p.rs.rank;
      }

      for (int c0 = 0; c0 < kTileN; c0 += EPI_COLS) {
        const int col0 = tn * kTileN + c0;
        uint8_t* stg = stg_base + (kStagingBuffers<MODE> == 2 ? (chunk_seq & 1) * L::kStagingBufBytes : 0);
        const uint32_t stg_addr = smem_u32(stg);
        if (tma_out && chunk_seq >= 2) {
          // This buffer's previous TMA store (two chunks ago) must have read it.
          if (lane == 0) bulk_wait_group_read<1>();
          __syncwarp();
        }
        float v[EPI_COLS];
#pragma unroll
        for (int j = 0; j < EPI_COLS; j += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(t_row + uint32_t(c0 + j), r);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) v[j + i] = __uint_as_float(r[i]);
        }
        if (c0 + EPI_COLS >= kTileN) {
          // Accumulator fully read: hand the TMEM buffer back to the MMA warp.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            if constexpr (PAIR)
              mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[b]), 0));
            else
              mbar_arrive(&tempty[b]);
          }
        }
        if (col0 >= p.N) continue;  // whole chunk beyond N (tail tile)

        if constexpr (MODE == kModeLocal) {
          const bool row_ok = my_row < p.M;
          // ---- fused elementwise epilogue, result rounded to bf16 in v[]
          if ((p.epi & (kEpiBias | kEpiGelu)) && !(p.epi & kEpiResidual)) {
            if (p.bias) {
#pragma unroll
              for (int i = 0; i < EPI_COLS; ++i) {
                const int col = col0 + i;
                v[i] = __fadd_rn(v[i], col < p.N ? __bfloat162float(p.bias[col]) : 0.f);
              }
            }
          }
          if (p.epi & kEpiGelu) {
            // aux = pre-activation (bf16); v = gelu(aux)
#pragma unroll
            for (int u = 0; u < EPI_COLS / 8; ++u) {
              uint4 pk;
              pk.x = pack_bf16x2(v[8 * u + 0], v[8 * u + 1]);
              pk.y = pack_bf16x2(v[8 * u + 2], v[8 * u + 3]);
              pk.z = pack_bf16x2(v[8 * u + 4], v[8 * u + 5]);
              pk.w = pack_bf16x2(v[8 * u + 6], v[8 * u + 7]);
              asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(
                               stg_addr + staging_offset<EPI_COLS>(lane, u)),
                           "r"(pk.x), "r"(pk.y), "r"(pk.z), "r"(pk.w));
            }
            __syncwarp();
            constexpr int kUnits = EPI_COLS / 8;
#pragma unroll 4
            for (int idx = lane; idx < 32 * kUnits; idx += 32) {
              const int r = idx / kUnits, u = idx % kUnits;
              const int row = row_w + r, col = col0 + u * 8;
              uint4 val;
              asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                           : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                           : "r"(stg_addr + staging_offset<EPI_COLS>(r, u)));
              if (row < p.M && col < p.N) st_global_v4(p.aux + int64_t(row) * p.ld_aux + col, val);
            }
            __syncwarp();
#pragma unroll
            for (int i = 0; i < EPI_COLS; ++i) v[i] = gelu_exact(bf16_round_f(v[i]));
          }
          if (p.epi & kEpiResidual) {
            // out = bf16(bf16(res + bf16(acc)) + bias)
#pragma unroll
            for (int u = 0; u < EPI_COLS / 8; ++u) {
              const int col = col0 + 8 * u;
              uint4 rv = make_uint4(0, 0, 0, 0);
              if (row_ok && col < p.N) rv = ld_global_v4(p.residual + int64_t(my_row) * p.ld_res + col);
              const __nv_bfloat16* rb = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const float y = bf16_round_f(v[8 * u + i]);
                const float s = bf16_round_f(__fadd_rn(__bfloat162float(rb[i]), y));
                const float bb = (p.bias && col + i < p.N) ? __bfloat162float(p.bias[col + i]) : 0.f;
                v[8 * u + i] = p.bias ? __fadd_rn(s, bb) : s;
              }
            }
          }
          if (p.epi & kEpiGeluBwd) {
#pragma unroll
            for (int u = 0; u < EPI_COLS / 8; ++u) {
              const int col = col0 + 8 * u;
              uint4 zv = make_uint4(0, 0, 0, 0);
              if (row_ok && col < p.N) zv = ld_global_v4(p.aux + int64_t(my_row) * p.ld_aux + col);
              const __nv_bfloat16* zb = reinterpret_cast<const __nv_bfloat16*>(&zv);
#pragma unroll
              for (int i = 0; i < 8; ++i)
                v[8 * u + i] = bf16_round_f(v[8 * u + i]) * gelu_grad(__bfloat162float(zb[i]));
            }
          }
          if (p.epi & kEpiAccumulate) {
#pragma unroll
            for (int u = 0; u < EPI_COLS / 8; ++u) {
              const int col = col0 + 8 * u;
              uint4 ov = make_uint4(0, 0, 0, 0);
              if (row_ok && col < p.N) ov = ld_global_v4(p.out + int64_t(my_row) * p.ldo + col);
              const __nv_bfloat16* ob = reinterpret_cast<const __nv_bfloat16*>(&ov);
#pragma unroll
              for (int i = 0; i < 8; ++i) v[8 * u + i] = __fadd_rn(__bfloat162float(ob[i]), v[8 * u + i]);
            }
          }
        }

        if constexpr (MODE == kModeRsTaco) {
          if (remote_taco) {
            // Encode my row's 128-column group (bf16-rounded partial, as the
            // reference encodes the stored BF16 partial) and stage the payload.
            // v[] is reused in place as the group (bf16-rounded first).
#pragma unroll
            for (int i = 0; i < 128; ++i) v[i] = bf16_round_f(v[i]);
            float quant, adaptive;
            taco::encode_group(v, quant, adaptive);
            // payload: 128 bytes per row = 8 units of 16 B, swizzled like bf16 staging
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              uint32_t w[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int c = 16 * u + 4 * k;
                w[k] = taco::code(v[c], quant) | (taco::code(v[c + 1], quant) << 8) |
                       (taco::code(v[c + 2], quant) << 16) | (taco::code(v[c + 3], quant) << 24);
              }
              asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(
                               stg_addr + staging_offset<64>(lane, u)),
                           "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]));
            }
            __syncwarp();
            // Receiver packet of source `rank`, block = chunk_rows x N (reference SoA layout).
            // Packets of a lane's blocks sit back to back in its region.
            const int row_local0 = row_w - dest * p.rs.rows_per_dest;
            const int blk = row_local0 / p.rs.chunk_rows;
            const int64_t elems = int64_t(p.rs.chunk_rows) * p.N;
            const int64_t groups = elems / 128;
            uint8_t* pkt = p.rs.recv[dest] + p.rs.lanes.slot_offset(blk & 1, p.rs.rank) +
                           int64_t(blk >> 1) * (elems + 8 * groups);
            const int rib0 = row_local0 % p.rs.chunk_rows;  // row in block of lane 0
#pragma unroll 4
            for (int idx = lane; idx < 32 * 8; idx += 32) {
              const int r = idx / 8, u = idx % 8;
              const int64_t g = (int64_t(rib0 + r) * p.N + col0) / 128;
              uint4 val;
              asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                           : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                           : "r"(stg_addr + staging_offset<64>(r, u)));
              st_global_v4(pkt + g * 128 + u * 16, val);
            }
            {
              const int64_t g = (int64_t(rib0 + lane) * p.N + col0) / 128;
              reinterpret_cast<float*>(pkt + elems)[g] = quant;
              reinterpret_cast<float*>(pkt + elems + 4 * groups)[g] = adaptive;
            }
            __syncwarp();
            continue;
          }
        }

        // ---- bf16 staging + coalesced 16-byte stores
#pragma unroll
        for (int u = 0; u < EPI_COLS / 8; ++u) {
          uint4 pk;
          pk.x = pack_bf16x2(v[8 * u + 0], v[8 * u + 1]);
          pk.y = pack_bf16x2(v[8 * u + 2], v[8 * u + 3]);
          pk.z = pack_bf16x2(v[8 * u + 4], v[8 * u + 5]);
          pk.w = pack_bf16x2(v[8 * u + 6], v[8 * u + 7]);
          asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(
                           stg_addr + staging_offset<EPI_COLS>(lane, u)),
                       "r"(pk.x), "r"(pk.y), "r"(pk.z), "r"(pk.w));
        }
        if (tma_out) {
          // Swizzled staging == the SWIZZLE_128B box layout: hand it to TMA.
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (MODE == kModeRsPull)  // piece (row block, column chunk), rows q*32..+31
              tma_store_2d(&tmap_out, stg_addr, 0, ((row_w / 128) * (p.N / 64) + col0 / 64) * 128 + row_w % 128);
            else
              tma_store_2d(&tmap_out, stg_addr, col0, row_w);
            bulk_commit_group();
          }
          ++chunk_seq;
          continue;
        }
        __syncwarp();
        {
          constexpr int kUnits = EPI_COLS / 8;
          __nv_bfloat16* base;
          int64_t ld;
          int row_base;
          if constexpr (MODE == kModeLocal) {
            base = p.out;
            ld = p.ldo;
            row_base = row_w;
          } else {
            // A 128-row tile lies inside one block (128 | chunk_rows): one lane.
            const int row_local = row_w - dest * p.rs.rows_per_dest;
            base = reinterpret_cast<__nv_bfloat16*>(
                p.rs.recv[dest] + p.rs.lanes.slot_offset(p.rs.lanes.lane_of(row_local), p.rs.rank));
            ld = p.N;
            row_base = p.rs.lanes.lane_row(row_local);
          }
#pragma unroll 4
          for (int idx = lane; idx < 32 * kUnits; idx += 32) {
            const int r = idx / kUnits, u = idx % kUnits;
            const int col = col0 + u * 8;
            uint4 val;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(val.x), "=r"(val.y), "=r"(val.z), "=r"(val.w)
                         : "r"(stg_addr + staging_offset<EPI_COLS>(r, u)));
            if (row_w + r < p.M && col < p.N) st_global_v4(base + int64_t(row_base + r) * ld + col, val);
          }
        }
        __syncwarp();
      }

      if constexpr (MODE == kModeRsPull) {
        // Publish this CTA's 128-row flag tile to its owner once all four
        // epilogue warps' TMA stores have completed in local memory: a
        // system-scope release of flag[source][flag tile] = epoch on the owner.
        if (lane == 0) {
          bulk_wait_group_all();
          fence_proxy_async_global();
        }
        __syncwarp();
        named_barrier_sync(1, kEpiWarps * 32);
        if (warp == kEpiFirstWarp && lane == 0) {
          const int row = tm * kTileM + int(cta_rank) * kBM;
          const int d = row / p.rs.rows_per_dest;
          const int tiles_n = p.N / kTileN;
          const int local_tile = ((row - d * p.rs.rows_per_dest) / kBM) * tiles_n + tn;
          const int per_dest = (p.rs.rows_per_dest / kBM) * tiles_n;
          if (p.rs.delay_ns && tm * p.tiles_n + tn == p.rs.delay_tile) {
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < p.rs.delay_ns) __nanosleep(1000);
          }
          fence_acq_rel_sys();
          st_release_sys(p.rs.flags[d] + int64_t(p.rs.rank) * per_dest + local_tile, p.rs.epoch);
          if (p.pull.produced) p.pull.produced[(row / kBM) * tiles_n + tn] = globaltimer_ns();
        }
      }
      if constexpr (MODE == kModeRsPush || MODE == kModeRsTaco) {
        // Publish the tile to its owner: all four epilogue warps' stores, then
        // one system-scope release of flag[source][tile] = epoch on the owner.
        named_barrier_sync(1, kEpiWarps * 32);
        if (warp == kEpiFirstWarp && lane == 0) {
          const int row_local = tm * kBM - dest * p.rs.rows_per_dest;
          if (p.rs.delay_ns && tm * p.tiles_n + tn == p.rs.delay_tile) {
            const uint64_t t0 = globaltimer_ns();
            while (globaltimer_ns() - t0 < p.rs.delay_ns) __nanosleep(1000);
          }
          fence_acq_rel_sys();
          st_release_sys(p.rs.flags[dest] + p.rs.lanes.flag_index(p.rs.rank, row_local, tn), p.rs.epoch);
        }
      }
    }
    if (tma_out && lane == 0) bulk_wait_group_all();  // stores complete before the CTA exits
  }

  // ------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (p.cta_stamps && threadIdx.x == 0) p.cta_stamps[2 * blockIdx.x + 1] = globaltimer_ns();
  if constexpr (PAIR) cluster_sync();  // the leader's MMAs into this CTA's TMEM are done
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, kTmemCols);
    else
      tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace gemm
}  // namespace tn5b
