// Host launcher for the tcgen05 GEMM family: TMA descriptor encoding, kernel
// instantiation selection, argument validation and persistent-grid sizing.
#include "gemm_api.h"
#include "gemm_kernel.cuh"

#include <cmath>
#include <mutex>
#include <cstdio>

namespace tn5b {
namespace gemm {

namespace {
// Wave-model constants of the auto tile choice (measured tensor-pipe busy
// fractions on B200 at 8192^3, and the wide tile's unoverlapped epilogue
// expressed as an equivalent K length).
constexpr double kEffSingle = 0.74;
constexpr double kEffWide = 0.93;
constexpr double kWideEpilogueK = 256.0;
thread_local std::string g_last_error;

int fail(const char* msg) {
  g_last_error = msg;
  return -1;
}

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
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor map, 128-byte swizzle. `inner` is the contiguous extent.
bool make_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t ld,
              uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int sm_count() {
  static int n[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && n[dev]) return n[dev];
  int v = 0;
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  if (dev < 64) n[dev] = v;
  return v;
}

template <int BN, int STAGES, int EPI_COLS, int MODE, bool AG, bool PAIR = false, bool WIDE = false>
int launch(const GemmCall& c, const Params& p, const CUtensorMap& ma, const CUtensorMap& mb,
           const CUtensorMap& mo, const CUtensorMap& ma2, int grid, cudaStream_t stream) {
  using L = SmemLayout<BN, STAGES, EPI_COLS, PAIR, WIDE, kStagingBuffers<MODE>>;
  static_assert(L::kTotal <= 232448, "dynamic shared memory above the 227 KB per-block limit");
  static_assert(!(MODE == kModeRsPull || AG) || L::kTotal >= 1024 + kCommStages * (kPiece + 16) + 16,
                "communication CTAs need their ring in the same dynamic shared memory");
  if (grid <= 0) return 0;
  auto kern = gemm_kernel<BN, STAGES, EPI_COLS, MODE, AG, PAIR, WIDE>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 64 || !configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (e != cudaSuccess) return int(e);
    if (dev < 64) configured[dev] = true;
  }
  const int threads = kThreadsFor<MODE>;
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(grid), 1, 1);
    cfg.blockDim = dim3(unsigned(threads), 1, 1);
    cfg.dynamicSmemBytes = L::kTotal;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return int(cudaLaunchKernelEx(&cfg, kern, ma, mb, mo, ma2, p, c.a_mn, c.b_mn));
  } else {
    kern<<<grid, threads, L::kTotal, stream>>>(ma, mb, mo, ma2, p, c.a_mn, c.b_mn);
    return int(cudaGetLastError());
  }
}

// Tile kinds: single-CTA 128 x BN (double-buffered accumulators), CTA pair
// 256 x 256, wide CTA pair 256 x 512 (one accumulator, twice the tensor work per
// byte in flight).  Auto picks between single and wide with a wave model: the
// wide tile keeps the tensor pipe busier on long K loops, but its epilogue is
// not overlapped and its 4x larger tiles quantise into fewer, coarser waves.
enum TileKind { kSingle = 0, kPair = 1, kWide = 2 };

// The split tail (below) pays only on long K: measured at M=8192, N=4096 it
// took 5 % off K=16384, nothing at K=4096 and added 5-15 % at K=2048 (the
// CTA-pair tail launch runs at a lower tensor-pipe occupancy than wide tiles).
constexpr int kSplitMinK = 8192;

// Wave-model choice between the single-CTA and the wide tile on `sms` SMs.
int auto_kind(int M, int N, int K, double sms) {
  if (K < 1024 || sms < 2) return kSingle;
  const double tiles_s = double((M + 127) / 128) * double((N + 255) / 256);
  const double tiles_w = double((M + 255) / 256) * double((N + 511) / 512);
  const double clusters = std::floor(sms / 2);
  const double waves_s = std::ceil(tiles_s / sms);
  double waves_w = std::ceil(tiles_w / clusters);
  // A partial last wave of at most half the clusters runs as CTA-pair tiles
  // (run_split): about half a wide wave instead of a full one.
  const double full = std::floor(tiles_w / clusters), rest = tiles_w - full * clusters;
  if (K >= kSplitMinK && full >= 1 && rest > 0 && 2 * rest <= clusters) waves_w = full + 0.55;
  // Per-SM work of one wave: 1 unit (128 x 256 x K) single, 2 units wide.
  const double cost_s = waves_s / kEffSingle;
  const double cost_w = 2.0 * waves_w * (1.0 + kWideEpilogueK / double(K)) / kEffWide;
  return cost_w < cost_s ? kWide : kSingle;
}

int tile_kind(const GemmCall& c, int bn) {
  // The push epilogues write 16-byte stores into peers' slots per single-CTA tile.
  if (bn != 256 || c.mode == 1 || c.mode == 2) return kSingle;
  if (c.pair >= 0) return c.pair <= kWide ? c.pair : kSingle;  // explicit (tables built in its units)
  if (c.tile_order) return kSingle;                            // a table without a kind: single-CTA units
  const bool comm_mode = c.mode == 3 || c.ag;
  return auto_kind(c.M, c.N, c.K, double(sm_count() - (comm_mode ? c.comm_ctas : 0)));
}

// Split of a wide-tile GEMM: the main launch runs `full` waves of wide tiles,
// a second launch runs the rest as CTA-pair 256 x 256 tiles (two per wide
// tile) in one wave.  Returns the number of wide tiles of the main launch, or
// 0 when the last wave is more than half full (or the shape does not allow it).
int split_main_tiles(const GemmCall& c, int tiles_m_w, int tiles_n_w) {
  if (c.tile_order || c.mode != 0 || c.ag || c.N % 512 || c.max_ctas > 0 || c.K < kSplitMinK) return 0;
  const int clusters = sm_count() / 2;
  const int tiles = tiles_m_w * tiles_n_w;
  const int full = tiles / clusters, rest = tiles - full * clusters;
  if (full < 1 || rest == 0 || 2 * rest > clusters) return 0;
  return full * clusters;
}

int pick_bn(const GemmCall& c) {
  if (c.bn == 128 || c.bn == 256) return c.bn;
  if (c.mode != 0) return 256;
  if (c.N <= 128) return 128;
  // Prefer the wider tile unless it leaves too few tiles to fill the machine.
  const int sms = sm_count();
  const long tiles256 = long((c.M + 127) / 128) * ((c.N + 255) / 256);
  if (tiles256 < sms) return 128;
  return 256;
}
}  // namespace

std::string last_error() { return g_last_error; }

namespace {
// Reads the tile order back exactly as the GEMM kernel's CTAs see it
// (tile_coords over the uploaded table or the grouped raster).
__global__ void tile_map_kernel(const __grid_constant__ Params p, int* out) {
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < p.num_tiles; t += gridDim.x * blockDim.x) {
    int tm, tn;
    tile_coords(p, t, tm, tn);
    out[2 * t] = tm;
    out[2 * t + 1] = tn;
  }
}
}  // namespace

int tile_map(const GemmCall& c, int* out, cudaStream_t stream) {
  if (c.M <= 0 || c.N <= 0 || !out) return fail("tile_map: bad args");
  const int bn = pick_bn(c);
  const int kind = tile_kind(c, bn);
  const bool pair = kind != kSingle;
  const int tile_n = kind == kWide ? 2 * bn : bn;
  Params p{};
  p.tail_from = -1;
  p.M = c.M; p.N = c.N; p.K = c.K;
  p.tiles_m = (c.M + (pair ? 2 * kBM : kBM) - 1) / (pair ? 2 * kBM : kBM);
  p.tiles_n = (c.N + tile_n - 1) / tile_n;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.group_m = c.group_m > 0 ? c.group_m : 8;
  p.tile_order = c.tile_order;
  tile_map_kernel<<<(p.num_tiles + 255) / 256, 256, 0, stream>>>(p, out);
  return int(cudaGetLastError());
}

int tile_count(const GemmCall& c) {
  const int bn = pick_bn(c);
  const int kind = tile_kind(c, bn);
  const bool pair = kind != kSingle;
  const int tile_n = kind == kWide ? 2 * bn : bn;
  return ((c.M + (pair ? 2 * kBM : kBM) - 1) / (pair ? 2 * kBM : kBM)) * ((c.N + tile_n - 1) / tile_n);
}

int fused_tile_kind(int M, int N, int K, int comm_ctas) {
  return auto_kind(M, N, K, double(sm_count() - comm_ctas));
}

int comm_active(const GemmCall& c) {
  const bool comm_mode = c.mode == 3 || c.ag;
  return (comm_mode && (c.phase & 3)) ? c.comm_ctas : 0;
}

int gemm_ctas(const GemmCall& c) {
  if (!(c.phase & 4)) return 0;
  const int bn = pick_bn(c);
  const int kind = tile_kind(c, bn);
  const bool pair = kind != kSingle;
  const int tile_m = pair ? 2 * kBM : kBM;
  const int tile_n = kind == kWide ? 2 * bn : bn;
  const long tiles = long((c.M + tile_m - 1) / tile_m) * ((c.N + tile_n - 1) / tile_n);
  const bool comm_mode = c.mode == 3 || c.ag;
  int g = sm_count() - (comm_mode ? c.comm_ctas : 0);
  if (c.max_ctas > 0 && c.max_ctas < g) g = c.max_ctas;
  if (g < (pair ? 2 : 1)) g = pair ? 2 : 1;
  if (pair) {
    const long clusters = tiles < g / 2 ? tiles : g / 2;
    return int(2 * clusters);
  }
  return int(tiles < g ? tiles : g);
}

int grid_ctas(const GemmCall& c) { return gemm_ctas(c) + comm_active(c); }

int run(const GemmCall& c, cudaStream_t stream) {
  if (c.M <= 0 || c.N <= 0 || c.K <= 0) return fail("gemm: non-positive M/N/K");
  if (!c.A || !c.B) return fail("gemm: null operand");
  if ((reinterpret_cast<uintptr_t>(c.A) | reinterpret_cast<uintptr_t>(c.B)) & 15)
    return fail("gemm: operands must be 16-byte aligned");
  if ((c.lda * 2) % 16 || (c.ldb * 2) % 16) return fail("gemm: leading dims must be 16-byte multiples");
  if (c.N % 8) return fail("gemm: N must be a multiple of 8");
  if (c.mode == 0) {
    if (!c.out) return fail("gemm: null output");
    if ((reinterpret_cast<uintptr_t>(c.out) & 15) || (c.ldo % 8))
      return fail("gemm: output must be 16-byte aligned with ldo % 8 == 0");
    if ((c.epi & kEpiGelu) && (c.epi & kEpiGeluBwd)) return fail("gemm: gelu and gelu-backward are exclusive");
    if ((c.epi & kEpiGeluBwd) && (!c.aux || (reinterpret_cast<uintptr_t>(c.aux) & 15) || c.ld_aux % 8))
      return fail("gemm: gelu-backward epilogue needs an aligned pre-activation input");
    if ((c.epi & kEpiGelu) && (!c.aux || (reinterpret_cast<uintptr_t>(c.aux) & 15) || c.ld_aux % 8))
      return fail("gemm: gelu epilogue needs an aligned aux output");
    if ((c.epi & kEpiResidual) && (!c.residual || (reinterpret_cast<uintptr_t>(c.residual) & 15) || c.ld_res % 8))
      return fail("gemm: residual epilogue needs an aligned residual");
  }
  const int bn = pick_bn(c);
  const int kind = tile_kind(c, bn);
  const bool pair = kind != kSingle;
  const int tile_n = kind == kWide ? 2 * bn : bn;
  Params p{};
  p.tail_from = -1;  // only a split GEMM's tail launch decodes tiles from the main grid
  p.M = c.M; p.N = c.N; p.K = c.K;
  p.tiles_m = (c.M + (pair ? 2 * kBM : kBM) - 1) / (pair ? 2 * kBM : kBM);
  p.tiles_n = (c.N + tile_n - 1) / tile_n;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.k_blocks = (c.K + kBK - 1) / kBK;
  p.group_m = c.group_m > 0 ? c.group_m : 8;
  p.tile_order = c.tile_order;
  p.epi = c.epi;
  p.out = static_cast<__nv_bfloat16*>(c.out); p.ldo = c.ldo;
  p.aux = static_cast<__nv_bfloat16*>(c.aux); p.ld_aux = c.ld_aux;
  p.bias = static_cast<const __nv_bfloat16*>(c.bias);
  p.residual = static_cast<const __nv_bfloat16*>(c.residual); p.ld_res = c.ld_res;
  p.status = c.status;
  p.timeout_ns = c.timeout_ns;
  p.debug = c.debug;
  p.cta_stamps = c.cta_stamps;
  p.gemm_ctas = gemm_ctas(c);
  p.comm_ctas = comm_active(c);
  if ((p.comm_ctas & 1) && pair) return fail("gemm: CTA-pair tiles need an even number of communication CTAs");
  if (c.mode == 3) {
    if (!c.rs_partial_local || !c.rs_partials || !c.rs_flags || !c.rs_my_flags || !c.rs_out || c.world < 1 ||
        c.M % c.world)
      return fail("gemm-rs-pull: bad args");
    const int rows = c.M / c.world;
    if (rows % (pair ? 2 * kBM : kBM) || c.N % tile_n)
      return fail("gemm-rs-pull: rows per destination must be a multiple of the tile height and N of its width");
    if ((c.phase & 2) && c.comm_ctas < 1) return fail("gemm-rs-pull: the reduce phase needs comm_ctas >= 1");
    if ((reinterpret_cast<uintptr_t>(c.rs_partial_local) | reinterpret_cast<uintptr_t>(c.rs_out)) & 15)
      return fail("gemm-rs-pull: partial and output must be 16-byte aligned");
    if (c.rs_residual && (reinterpret_cast<uintptr_t>(c.rs_residual) & 15))
      return fail("gemm-rs-pull: residual must be 16-byte aligned");
    if (c.rs_bias && (reinterpret_cast<uintptr_t>(c.rs_bias) & 15))
      return fail("gemm-rs-pull: bias must be 16-byte aligned");
    p.rs.flags = c.rs_flags;
    p.rs.rank = c.rank; p.rs.world = c.world;
    p.rs.rows_per_dest = rows; p.rs.chunk_rows = c.chunk_rows;
    p.rs.epoch = c.epoch;
    if (c.delay_ns > 100000000ull) return fail("gemm-rs: diagnostic delay above 100 ms");
    p.rs.delay_tile = c.delay_tile; p.rs.delay_ns = c.delay_ns;
    p.pull.partial = c.rs_partials;
    p.pull.my_flags = c.rs_my_flags;
    p.pull.order = c.rs_consumer_order;
    p.pull.tiles_n = c.N / tile_n;
    p.pull.tiles_per_dest = (rows / kBM) * p.pull.tiles_n;
    p.pull.out = static_cast<__nv_bfloat16*>(c.rs_out);
    p.pull.residual = static_cast<const __nv_bfloat16*>(c.rs_residual);
    p.pull.bias = static_cast<const __nv_bfloat16*>(c.rs_bias);
    p.pull.stamps = c.rs_stamps;
    p.pull.produced = c.rs_produced;
  } else if (c.mode != 0) {
    if (!c.rs_recv || !c.rs_flags || c.world < 1 || c.M % c.world) return fail("gemm-rs: bad args");
    const int rows = c.M / c.world;
    if (rows % kBM) return fail("gemm-rs: rows per destination must be a multiple of 128");
    if (c.chunk_rows <= 0 || rows % c.chunk_rows || c.chunk_rows % kBM || c.N % 256)
      return fail("gemm-rs: the push lanes need chunk_rows | rows, 128 | chunk_rows, 256 | N");
    p.rs.recv = c.rs_recv; p.rs.flags = c.rs_flags;
    p.rs.rank = c.rank; p.rs.world = c.world;
    p.rs.rows_per_dest = rows; p.rs.chunk_rows = c.chunk_rows;
    p.rs.epoch = c.epoch;
    p.rs.lanes = PushLanes{rows, c.N, c.chunk_rows, c.world, 256};
    if (c.slot_bytes != p.rs.lanes.lane_slot_bytes())
      return fail("gemm-rs: slot_bytes must be one lane region of one source (push_lanes.h)");
    if (c.delay_ns > 100000000ull) return fail("gemm-rs: diagnostic delay above 100 ms");
    p.rs.delay_tile = c.delay_tile; p.rs.delay_ns = c.delay_ns;
  }
  if (c.ag) {
    if (!c.ag_shard || !c.ag_gather || !c.ag_published || !c.ag_pulled || !c.ag_published_local ||
        !c.ag_pulled_local || !c.ag_ready || c.world < 2 || c.M % c.world || c.a_mn)
      return fail("ag-gemm: bad args");
    const int rows = c.M / c.world;
    if (rows % (pair ? 2 * kBM : kBM)) return fail("ag-gemm: rows per source must be a multiple of the tile height");
    if (reinterpret_cast<uintptr_t>(c.ag_shard) & 15 || c.lda != c.K)
      return fail("ag-gemm: shard must be 16-byte aligned and the gather buffer dense [M, K]");
    if ((c.phase & 3) && c.comm_ctas < 1) return fail("ag-gemm: the gather phases need comm_ctas >= 1");
    GatherArgs& g = p.gather;
    g.gather = c.ag_gather;
    g.published = c.ag_published;
    g.pulled = c.ag_pulled;
    g.published_local = c.ag_published_local;
    g.pulled_local = c.ag_pulled_local;
    g.ready = c.ag_ready;
    g.shard = static_cast<const uint8_t*>(c.ag_shard);
    g.chunk_bytes = int64_t(rows) * c.K * 2;
    g.rank = c.rank; g.world = c.world; g.rows_per_src = rows; g.K = c.K;
    g.epoch = c.ag_epoch;
    g.pulled_target = c.ag_pulled_target;
    g.ready_target = c.ag_ready_target;
    g.phase = c.phase;
    g.block_stamps = c.ag_block_stamps;
    g.own_in_place = c.ag_own_in_place;
  }
  CUtensorMap ma, mb;
  const bool ok_a = c.a_mn ? make_map(&ma, c.A, c.M, c.K, c.lda, 64, 64)
                           : make_map(&ma, c.A, c.K, c.M, c.lda, 64, kBM);
  const bool ok_b = c.b_mn ? make_map(&mb, c.B, c.N, c.K, c.ldb, 64, 64)
                           : make_map(&mb, c.B, c.K, c.N, c.ldb, 64, pair ? bn / 2 : bn);
  if (!ok_a || !ok_b) return fail("gemm: cuTensorMapEncodeTiled failed");
  // Output tensor map for the TMA-store epilogue (local mode, aligned output);
  // in the pull reduce-scatter it maps this rank's partial buffer as a
  // [M/128 * N/64 * 128, 64] matrix of 128 x 64 pieces.
  CUtensorMap mo = ma;
  p.tma_store = 0;
  if (c.mode == 3) {
    const uint64_t piece_rows = uint64_t(c.M / kBM) * uint64_t(c.N / 64) * kBM;
    if (!make_map(&mo, c.rs_partial_local, 64, piece_rows, 64, 64, 32))
      return fail("gemm-rs-pull: partial tensor map");
    p.tma_store = 1;
  } else if (c.mode == 0 && c.out && !(reinterpret_cast<uintptr_t>(c.out) & 15) && c.ldo % 8 == 0 &&
             make_map(&mo, c.out, c.N, c.M, c.ldo, 64, 32)) {
    p.tma_store = 1;
  }
  // AG: the own chunk is read straight from the shard ([M/W, K]); pull RS: the
  // reducer CTAs load the residual [M/W, N] in 128 x 64 tiles.
  CUtensorMap ma2 = ma;
  if (c.ag && !make_map(&ma2, c.ag_shard, c.K, c.M / c.world, c.K, 64, kBM))
    return fail("ag-gemm: shard tensor map");
  if (c.mode == 3 && c.rs_residual && !make_map(&ma2, c.rs_residual, c.N, c.M / c.world, c.N, 64, kBM))
    return fail("gemm-rs-pull: residual tensor map");
  const int grid = grid_ctas(c);
  if (c.ag) {
    if (kind == kWide) return launch<256, 4, 64, kModeLocal, true, true, true>(c, p, ma, mb, mo, ma2, grid, stream);
    if (pair) return launch<256, 6, 64, kModeLocal, true, true>(c, p, ma, mb, mo, ma2, grid, stream);
    if (bn == 256) return launch<256, 4, 64, kModeLocal, true>(c, p, ma, mb, mo, ma2, grid, stream);
    return launch<128, 6, 64, kModeLocal, true>(c, p, ma, mb, mo, ma2, grid, stream);
  }
  switch (c.mode) {
    case 0:
      if (kind == kWide) {
        const int main_tiles = split_main_tiles(c, p.tiles_m, p.tiles_n);
        if (main_tiles > 0) {
          // Main launch: whole waves of wide tiles; tail launch: the remaining
          // wide tiles as pairs of 256 x 256 CTA-pair tiles, one wave.
          const int wide_m = p.tiles_m, wide_n = p.tiles_n;
          Params main = p;
          main.num_tiles = main_tiles;
          main.gemm_ctas = 2 * (sm_count() / 2);
          int r = launch<256, 4, 64, kModeLocal, false, true, true>(c, main, ma, mb, mo, ma2, main.gemm_ctas,
                                                                    stream);
          if (r) return r;
          Params tail = p;
          tail.debug = nullptr;
          tail.cta_stamps = nullptr;
          tail.tail_from = main_tiles;
          tail.tail_tiles_m = wide_m;
          tail.tail_tiles_n = wide_n;
          tail.tiles_m = wide_m;
          tail.tiles_n = 2 * wide_n;
          tail.num_tiles = 2 * (wide_m * wide_n - main_tiles);
          const int clusters = tail.num_tiles < sm_count() / 2 ? tail.num_tiles : sm_count() / 2;
          tail.gemm_ctas = 2 * clusters;
          return launch<256, 6, 64, kModeLocal, false, true>(c, tail, ma, mb, mo, ma2, tail.gemm_ctas, stream);
        }
        return launch<256, 4, 64, kModeLocal, false, true, true>(c, p, ma, mb, mo, ma2, grid, stream);
      }
      if (pair) return launch<256, 6, 64, kModeLocal, false, true>(c, p, ma, mb, mo, ma2, grid, stream);
      if (bn == 256) return launch<256, 4, 64, kModeLocal, false>(c, p, ma, mb, mo, ma2, grid, stream);
      return launch<128, 6, 64, kModeLocal, false>(c, p, ma, mb, mo, ma2, grid, stream);
    case 1:
      return launch<256, 4, 64, kModeRsPush, false>(c, p, ma, mb, mo, ma2, grid, stream);
    case 2:
      return launch<256, 4, 128, kModeRsTaco, false>(c, p, ma, mb, mo, ma2, grid, stream);
    case 3:
      if (kind == kWide) return launch<256, 4, 64, kModeRsPull, false, true, true>(c, p, ma, mb, mo, ma2, grid, stream);
      if (pair) return launch<256, 6, 64, kModeRsPull, false, true>(c, p, ma, mb, mo, ma2, grid, stream);
      return launch<256, 4, 64, kModeRsPull, false>(c, p, ma, mb, mo, ma2, grid, stream);
    default:
      return fail("gemm: unknown mode");
  }
}

}  // namespace gemm
}  // namespace tn5b
