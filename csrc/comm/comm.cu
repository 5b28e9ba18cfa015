// Receiver side of the fused GEMM -> reduce-scatter and the bounded-wait probe.
//
// Each rank's producer GEMM pushes tile (source=s) of destination d into the
// receive region of the tile's lane on d (lane = parity of its block within the
// destination; push_lanes.h) and release-stores that lane's flag[s][tile] =
// epoch on d.  This kernel runs
// on d after its own GEMM (same stream), waits (bounded) for every source's
// tile flag and reduces in the fixed source order 0..W-1, rounding to BF16
// after every source ("bf16_after_each_source", src/taco/codec.cu:155-196 of
// TempName-5090).  Remote TACO packets are decoded in the same pass with the
// reference decoder's FP32 operation sequence, so the output is bit-identical
// to the reference's decode_reduce / reduce kernels.
//
// Consumption policies:
//   ordered   CTA c takes tiles order[c], order[c+grid], ... and blocks on each.
//   arrival   CTAs are split over the two lanes; each scans its lane's tiles
//             (its lane's flag array) and claims whichever is fully ready
//             first (per-tile claim words tagged with the epoch).
#include "comm_api.h"
#include "../common/ptx.cuh"
#include "../common/push_lanes.h"
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace tn5b {
namespace comm {

namespace {
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr float kNorm = 0.08838834764831844055f;

__device__ __forceinline__ uint2 ld_cg_v2(const void* p) {
  uint2 v;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_cg_u32(const void* p) {
  uint32_t v;
  asm volatile("ld.global.cg.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}
__device__ __forceinline__ float ld_cg_f32(const void* p) {
  return __uint_as_float(ld_cg_u32(p));
}

// Reference decoder arithmetic for lane l's four coefficients 4l..4l+3.
__device__ __forceinline__ void decode4(uint32_t raw, float quant, float adaptive, float (&o)[4]) {
  const int lane = threadIdx.x & 31;
  const __half2 lo(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(raw & 0xFFFFu), __NV_E4M3));
  const __half2 hi(__nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(raw >> 16), __NV_E4M3));
  float x[4] = {__fmul_rn(__low2float(lo), quant), __fmul_rn(__high2float(lo), quant),
                __fmul_rn(__low2float(hi), quant), __fmul_rn(__high2float(hi), quant)};
  float a = x[0], b = x[1], c = x[2], d = x[3];
  x[0] = __fadd_rn(a, b); x[1] = __fsub_rn(a, b); x[2] = __fadd_rn(c, d); x[3] = __fsub_rn(c, d);
  a = x[0]; b = x[1]; c = x[2]; d = x[3];
  x[0] = __fadd_rn(a, c); x[1] = __fadd_rn(b, d); x[2] = __fsub_rn(a, c); x[3] = __fsub_rn(b, d);
#pragma unroll
  for (int stride = 1; stride < 32; stride *= 2) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float other = __shfl_xor_sync(0xffffffffu, x[j], stride);
      x[j] = (lane & stride) ? __fsub_rn(other, x[j]) : __fadd_rn(x[j], other);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) o[j] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(x[j], kNorm) / adaptive));
}

__device__ __forceinline__ PushLanes lanes_of(const RsReduceCall& c) {
  return PushLanes{c.rows, c.n, c.chunk_rows, c.world, c.tile_n};
}

// Flag of source s for local tile `tile` (in its lane's flag array).
__device__ __forceinline__ const uint32_t* tile_flag(const RsReduceCall& c, int s, int tile, int tiles_n) {
  return c.flags + lanes_of(c).flag_index(s, (tile / tiles_n) * 128, tile % tiles_n);
}

__device__ __forceinline__ bool tile_ready(const RsReduceCall& c, int tile, int tiles_n) {
  for (int s = 0; s < c.world; ++s)
    if (int32_t(ld_acquire_sys(tile_flag(c, s, tile, tiles_n)) - c.epoch) < 0) return false;
  return true;
}

// Reduce one producer tile (128 rows x tile_n cols) of the local output.
__device__ void reduce_tile(const RsReduceCall& c, int tile, int tiles_n) {
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int tm = tile / tiles_n, tn = tile % tiles_n;
  const int cols = min(c.tile_n, c.n - tn * c.tile_n);
  const int groups_per_row = cols / 128;  // n, tile_n multiples of 128
  const int total = 128 * groups_per_row;
  const int64_t elems = int64_t(c.chunk_rows) * c.n;
  const int64_t block_groups = elems / 128;
  const PushLanes L = lanes_of(c);
  const int tile_lane = L.lane_of(tm * 128);  // a tile lies inside one block
  for (int gi = warp; gi < total; gi += kWarps) {
    const int r = tm * 128 + gi / groups_per_row;
    const int col = tn * c.tile_n + (gi % groups_per_row) * 128 + lane * 4;
    const int64_t idx = int64_t(r) * c.n + col;                // output element
    const int64_t lidx = int64_t(L.lane_row(r)) * c.n + col;   // element in the lane's BF16 blocks
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < c.world; ++s) {
      float v[4];
      const uint8_t* slot = c.recv + L.slot_offset(tile_lane, s);
      if (s == c.rank || !c.quantized) {
        const uint2 raw = ld_cg_v2(slot + lidx * 2);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __bfloat162float(h[j]);
      } else {
        const int blk = r / c.chunk_rows;
        const int64_t g = (int64_t(r % c.chunk_rows) * c.n + (col - lane * 4)) / 128;
        const uint8_t* pkt = slot + int64_t(blk >> 1) * (elems + 8 * block_groups);
        const uint32_t raw = ld_cg_u32(pkt + g * 128 + lane * 4);
        const float quant = ld_cg_f32(pkt + elems + 4 * g);
        const float adaptive = ld_cg_f32(pkt + elems + 4 * block_groups + 4 * g);
        decode4(raw, quant, adaptive, v);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = __bfloat162float(__float2bfloat16_rn(__fadd_rn(acc[j], v[j])));
    }
    if (c.residual) {
      const uint2 rr = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(c.residual) + idx);
      const __nv_bfloat16* rh = reinterpret_cast<const __nv_bfloat16*>(&rr);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float t = __bfloat162float(__float2bfloat16_rn(__fadd_rn(__bfloat162float(rh[j]), acc[j])));
        if (c.bias) t = __fadd_rn(t, __bfloat162float(static_cast<const __nv_bfloat16*>(c.bias)[col + j]));
        acc[j] = t;
      }
    } else if (c.bias) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        acc[j] = __fadd_rn(acc[j], __bfloat162float(static_cast<const __nv_bfloat16*>(c.bias)[col + j]));
    }
    __nv_bfloat162 o0 = __floats2bfloat162_rn(acc[0], acc[1]);
    __nv_bfloat162 o1 = __floats2bfloat162_rn(acc[2], acc[3]);
    uint2 ov;
    ov.x = *reinterpret_cast<uint32_t*>(&o0);
    ov.y = *reinterpret_cast<uint32_t*>(&o1);
    *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(c.out) + idx) = ov;
  }
}

__global__ void __launch_bounds__(kThreads) rs_reduce_kernel(const __grid_constant__ RsReduceCall c) {
  const int tiles_n = (c.n + c.tile_n - 1) / c.tile_n;
  const int tiles = (c.rows / 128) * tiles_n;
  __shared__ int s_tile;
  __shared__ int s_ok;
  if (!c.arrival) {
    for (int i = blockIdx.x; i < tiles; i += gridDim.x) {
      const int tile = c.tile_order ? c.tile_order[i] : i;
      if (threadIdx.x == 0) {
        int ok = 1;
        for (int s = 0; s < c.world && ok; ++s)
          ok = wait_flag_geq(tile_flag(c, s, tile, tiles_n), c.epoch, c.timeout_ns, c.status,
                             kTimeoutPeerFlag);
        s_ok = ok;
      }
      __syncthreads();
      if (!s_ok) return;
      reduce_tile(c, tile, tiles_n);
      __syncthreads();
      if (c.stamps && threadIdx.x == 0) c.stamps[tile] = globaltimer_ns();
    }
    return;
  }
  // Arrival-first: lane = parity of the tile's block-within-destination.  Each
  // CTA of a lane scans a window of kWindow positions of the consumer order
  // starting at its low-water mark (every earlier position of its lane is
  // claimed), and claims (CAS tagged with the epoch) the first ready unclaimed
  // tile of its lane found from its own offset in the window, cyclically -- the
  // offsets of a lane's CTAs are spread over the window, so they do not all race
  // for one tile, and a scan polls at most kWindow tiles' flags instead of all.
  constexpr int kWindow = 128;
  const int lane_id = blockIdx.x & 1;
  const int offset = int((blockIdx.x >> 1) * 37) % kWindow;
  const uint64_t start = globaltimer_ns();
  __shared__ int s_best, s_lwm;
  if (threadIdx.x == 0) s_lwm = 0;
  __syncthreads();
  auto lane_of = [&](int i) {
    const int tile = c.tile_order ? c.tile_order[i] : i;
    return ((tile / tiles_n) * 128 / c.chunk_rows) & 1;
  };
  auto claimed = [&](int i) {
    const int tile = c.tile_order ? c.tile_order[i] : i;
    return int32_t(uint32_t(*reinterpret_cast<volatile int*>(c.claims + tile)) - c.epoch) >= 0;
  };
  for (;;) {
    if (threadIdx.x == 0) {
      // Advance the low-water mark over other lanes' positions and claimed ones.
      int lwm = s_lwm;
      while (lwm < tiles && (lane_of(lwm) != lane_id || claimed(lwm))) ++lwm;
      s_lwm = lwm;
      s_best = 0x7fffffff;
    }
    __syncthreads();
    const int lwm = s_lwm;
    if (lwm >= tiles) return;  // lane drained
    const int span = min(kWindow, tiles - lwm);
    int best = 0x7fffffff;  // cyclic distance from this CTA's offset inside the window
    for (int w = threadIdx.x; w < span; w += kThreads) {
      const int i = lwm + w;
      if (lane_of(i) != lane_id || claimed(i)) continue;
      const int tile = c.tile_order ? c.tile_order[i] : i;
      const int dist = (w - offset % span + span) % span;
      if (dist < best && tile_ready(c, tile, tiles_n)) best = dist;
    }
    if (best != 0x7fffffff) atomicMin(&s_best, best);
    __syncthreads();
    if (threadIdx.x == 0) {
      int found = -1;
      if (s_best != 0x7fffffff) {
        const int i = lwm + (offset % span + s_best) % span;
        const int tile = c.tile_order ? c.tile_order[i] : i;
        const int old = *reinterpret_cast<volatile int*>(c.claims + tile);
        // tile_ready is this thread's own acquire of the flags (monotonic epochs:
        // ready for the scanning thread implies ready here).
        if (int32_t(uint32_t(old) - c.epoch) < 0 && tile_ready(c, tile, tiles_n) &&
            atomicCAS(c.claims + tile, old, int(c.epoch)) == old)
          found = tile;
      }
      if (found == -1 && globaltimer_ns() - start > c.timeout_ns) {
        record_status(c.status, kTimeoutPeerFlag);
        found = -2;
      }
      s_tile = found;
    }
    __syncthreads();
    const int tile = s_tile;
    if (tile == -2) return;
    if (tile == -1) {
      if (s_best == 0x7fffffff) __nanosleep(256);
      continue;
    }
    reduce_tile(c, tile, tiles_n);
    __syncthreads();
    if (c.stamps && threadIdx.x == 0) c.stamps[tile] = globaltimer_ns();
  }
}

// Bounded wait on a flag that nothing sets: lets tests check the timeout path
// (status code returned, context still usable) without faulting a GPU.
__global__ void wait_probe_kernel(const uint32_t* flag, uint32_t target, uint64_t timeout_ns,
                                  int* status) {
  if (threadIdx.x == 0 && blockIdx.x == 0)
    wait_flag_geq(flag, target, timeout_ns, status, kTimeoutPeerFlag);
}
// Grid-stride 16-byte copy with eight loads in flight per thread; `dst` may be
// a peer's memory (CUDA-IPC mapping): plain stores, no TMA.
__global__ void __launch_bounds__(256) copy16_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                     int64_t n16) {
  constexpr int kUnroll = 8;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + (kUnroll - 1) * stride < n16; i += kUnroll * stride) {
    uint4 v[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) v[u] = __ldg(src + i + u * stride);
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) dst[i + u * stride] = v[u];
  }
  for (; i < n16; i += stride) dst[i] = __ldg(src + i);
}

// Bulk-engine copy: one elected thread per CTA streams `chunk`-byte pieces of
// `src` (this GPU's memory or a peer's CUDA-IPC mapping; untiled bulk loads,
// no multicast) through a `stages`-deep shared-memory ring and writes each
// piece to `dst` (this GPU's memory) with an untiled bulk store.  CTA c copies
// pieces c, c + grid, ... so every CTA sweeps the whole buffer in step.
__global__ void __launch_bounds__(32) bulk_copy_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src,
                                                       int64_t bytes, int chunk, int stages, uint64_t timeout_ns,
                                                       int* status) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ uint64_t full[16];
  if (threadIdx.x != 0) return;
  for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
  fence_mbar_init();
  const int64_t pieces = (bytes + chunk - 1) / chunk;
  auto piece_bytes = [&](int64_t p) { const int64_t left = bytes - p * chunk; return uint32_t(left < chunk ? left : chunk); };
  int64_t issued = 0, done = 0;  // per-CTA piece counters
  const int64_t mine = pieces > blockIdx.x ? (pieces - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  for (; issued < mine && issued < stages; ++issued) {
    const int64_t p = blockIdx.x + issued * gridDim.x;
    const int s = int(issued % stages);
    mbar_arrive_expect_tx(&full[s], piece_bytes(p));
    bulk_load(ring + int64_t(s) * chunk, src + p * chunk, piece_bytes(p), &full[s]);
  }
  bool ok = true;
  for (; done < mine; ++done) {
    const int s = int(done % stages);
    const uint32_t parity = uint32_t((done / stages) & 1);
    if (!mbar_wait(&full[s], parity, timeout_ns, status, kTimeoutPeerFlag, nullptr)) {
      ok = false;
      break;
    }
    const int64_t p = blockIdx.x + done * gridDim.x;
    bulk_store(dst + p * chunk, smem_u32(ring + int64_t(s) * chunk), piece_bytes(p));
    bulk_commit_group();
    if (issued < mine) {
      bulk_wait_group_read<0>();  // the store has read stage s: refill it
      const int64_t q = blockIdx.x + issued * gridDim.x;
      mbar_arrive_expect_tx(&full[s], piece_bytes(q));
      bulk_load(ring + int64_t(s) * chunk, src + q * chunk, piece_bytes(q), &full[s]);
      ++issued;
    }
  }
  if (!ok) {
    // Abort: let every issued load land before the CTA exits (bounded).
    for (; done < issued; ++done)
      mbar_wait(&full[done % stages], uint32_t((done / stages) & 1), timeout_ns, status, kTimeoutDrain, nullptr);
  }
  bulk_wait_group_all();
}
// Pack a row-major [M, N] BF16 tensor into the pull reduce-scatter's partial
// layout [M/128][N/64][128][64] (16-byte units; one thread per unit).
__global__ void __launch_bounds__(256) pack_pieces_kernel(const uint4* __restrict__ src, int64_t ld_units,
                                                          uint4* __restrict__ dst, int M, int N) {
  const int units_per_row = N / 8;
  const int64_t total = int64_t(M) * units_per_row;
  const int n_chunks = N / 64;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int r = int(i / units_per_row), u = int(i % units_per_row);
    const int64_t piece = int64_t(r / 128) * n_chunks + u / 8;
    dst[piece * 1024 + (r % 128) * 8 + (u % 8)] = src[int64_t(r) * ld_units + u];
  }
}

// Release flag[source = rank][tile] = epoch on every destination, for all of
// its flag tiles (128 rows x tile_n), after the preceding pack (stream order).
__global__ void publish_tiles_kernel(uint32_t* const* flags, int rank, int world, int per_dest, uint32_t epoch) {
  const int total = world * per_dest;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int d = i / per_dest, t = i % per_dest;
    fence_acq_rel_sys();
    st_release_sys(flags[d] + int64_t(rank) * per_dest + t, epoch);
  }
}
}  // namespace

int pack_pieces(const void* src, int64_t ld, void* dst, int M, int N, cudaStream_t stream) {
  if (M % 128 || N % 64 || ld % 8 || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return -1;
  const int64_t units = int64_t(M) * (N / 8);
  const int grid = int(units / 256 < 148 * 8 ? (units + 255) / 256 : 148 * 8);
  pack_pieces_kernel<<<grid, 256, 0, stream>>>(static_cast<const uint4*>(src), ld / 8, static_cast<uint4*>(dst), M, N);
  return int(cudaGetLastError());
}

int publish_tiles(uint32_t* const* flags, int rank, int world, int per_dest, uint32_t epoch, cudaStream_t stream) {
  if (world < 1 || per_dest < 1) return -1;
  publish_tiles_kernel<<<(world * per_dest + 255) / 256, 256, 0, stream>>>(flags, rank, world, per_dest, epoch);
  return int(cudaGetLastError());
}

int bulk_copy(void* dst, const void* src, int64_t bytes, int ctas, int chunk, int stages, uint64_t timeout_ns,
              int* status, cudaStream_t stream) {
  if (bytes <= 0 || bytes % 16 || chunk <= 0 || chunk % 16 || stages < 1 || stages > 16 || ctas <= 0 ||
      (reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 15))
    return -1;
  const int64_t smem = int64_t(chunk) * stages;
  if (smem > 200 * 1024) return -1;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(bulk_copy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return int(e);
    if (dev < 64) configured[dev] = true;
  }
  bulk_copy_kernel<<<ctas, 32, smem, stream>>>(static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src),
                                                bytes, chunk, stages, timeout_ns, status);
  return int(cudaGetLastError());
}

int copy16(void* dst, const void* src, int64_t bytes, int ctas, cudaStream_t stream) {
  if (bytes <= 0 || bytes % 16 || (reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 15))
    return -1;
  if (ctas <= 0) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    ctas = 4 * sms;
  }
  copy16_kernel<<<ctas, 256, 0, stream>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src), bytes / 16);
  return int(cudaGetLastError());
}

int rs_reduce(const RsReduceCall& c, cudaStream_t stream) {
  if (c.rows % 128 || c.n % c.tile_n || c.tile_n % 128 || !c.recv || !c.flags || !c.out) return -1;
  if (c.chunk_rows <= 0 || c.chunk_rows % 128 || c.rows % c.chunk_rows) return -1;
  if (c.slot_bytes != PushLanes{c.rows, c.n, c.chunk_rows, c.world, c.tile_n}.lane_slot_bytes()) return -1;
  if (c.arrival && !c.claims) return -1;
  const int tiles = (c.rows / 128) * ((c.n + c.tile_n - 1) / c.tile_n);
  int sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int grid = c.arrival ? (tiles < 2 * sms ? tiles : 2 * sms) : tiles;
  if (c.arrival && grid < 2) grid = 2;
  if (c.max_ctas > 0 && grid > c.max_ctas) grid = c.max_ctas;
  rs_reduce_kernel<<<grid, kThreads, 0, stream>>>(c);
  return int(cudaGetLastError());
}

int wait_probe(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status,
               cudaStream_t stream) {
  wait_probe_kernel<<<1, 32, 0, stream>>>(flag, target, timeout_ns, status);
  return int(cudaGetLastError());
}

}  // namespace comm
}  // namespace tn5b
