// Host-side API of the tcgen05 GEMM family (plain, GEMM->reduce-scatter push,
// all-gather->GEMM).  Pointers are device pointers; all launches are async on
// the given stream.  Returns 0 or a cudaError_t / negative argument code.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <string>

namespace tn5b {
namespace gemm {

// AG->GEMM: u32 words between two per-block arrival counters (one 128-byte line each).
constexpr int kReadyStride = 32;

struct GemmCall {
  // Operands: A is [M,K] row-major (a_mn=0) or [K,M] row-major (a_mn=1);
  //           B is [N,K] row-major (b_mn=0) or [K,N] row-major (b_mn=1).
  const void* A = nullptr; int64_t lda = 0; int a_mn = 0;
  const void* B = nullptr; int64_t ldb = 0; int b_mn = 0;
  int M = 0, N = 0, K = 0;
  // Epilogue
  int epi = 0;
  void* out = nullptr; int64_t ldo = 0;
  void* aux = nullptr; int64_t ld_aux = 0;
  const void* bias = nullptr;
  const void* residual = nullptr; int64_t ld_res = 0;
  // Tile order (device int array of length tiles) or null for grouped raster.
  const int* tile_order = nullptr;
  int group_m = 8;
  int bn = 0;            // 0 = auto, else 128 / 256
  int pair = -1;         // tile kind: -1 auto, 0 single CTA 128xBN, 1 CTA pair 256x256, 2 wide pair 256x512
  int max_ctas = 0;      // 0 = all SMs
  // mode 0 local, 1 RS push bf16, 2 RS push TACO
  int mode = 0;
  // reduce-scatter
  uint8_t* const* rs_recv = nullptr;     // device array [world]
  uint32_t* const* rs_flags = nullptr;   // device array [world]
  int rank = 0, world = 1;
  int chunk_rows = 128;
  uint32_t epoch = 0;
  int64_t slot_bytes = 0;      // push: one lane region of one source (PushLanes::lane_slot_bytes)
  int delay_tile = -1;         // diagnostic: bounded publication delay of one tile
  uint64_t delay_ns = 0;
  // Communication role (pull transports): CTAs [gemm_ctas, grid) move data over
  // NVLink inside the same launch.  `phase` selects what a launch runs:
  // bit0 AG own chunk + publish, bit1 AG peer pulls / RS reduce, bit2 the GEMM
  // (7: everything in one launch; tests emulating several ranks on one GPU run
  // the phases as separate launches so that no launch waits on another).
  int comm_ctas = 0;
  int phase = 7;
  // GEMM -> reduce-scatter, pull (mode 3)
  void* rs_partial_local = nullptr;               // this rank's partial buffer [M/128][N/64][128][64]
  const uint8_t* const* rs_partials = nullptr;    // device array [world]: every rank's partial buffer
  const uint32_t* rs_my_flags = nullptr;          // this rank's flags [world][tiles_per_dest]
  const int* rs_consumer_order = nullptr;         // consumption order of local flag tiles
  void* rs_out = nullptr;                         // [M/world, N]
  const void* rs_residual = nullptr;              // optional [M/world, N]
  const void* rs_bias = nullptr;                  // optional [N]
  unsigned long long* rs_stamps = nullptr;        // optional per-local-tile completion times
  unsigned long long* rs_produced = nullptr;      // optional per-produced-tile publication times
  // all-gather -> GEMM, pull: A is this rank's gather buffer [M, K]
  int ag = 0;
  const void* ag_shard = nullptr;                 // [M/world, K] local shard (contiguous)
  uint8_t* const* ag_gather = nullptr;            // device array [world]: gather buffers
  uint32_t* const* ag_published = nullptr;        // device array [world]: published[world][blocks] flags
  uint32_t* const* ag_pulled = nullptr;           // device array [world]: pulled counters
  const uint32_t* ag_published_local = nullptr;
  const uint32_t* ag_pulled_local = nullptr;
  uint32_t* ag_ready = nullptr;                   // local [world][M/world/128]
  uint32_t ag_epoch = 0, ag_pulled_target = 0, ag_ready_target = 0;
  int ag_own_in_place = 0;                        // shard == own chunk of the gather buffer
  unsigned long long* ag_block_stamps = nullptr;  // optional: arrival time of every gathered block
  unsigned long long* cta_stamps = nullptr;       // optional [grid][2]: start / end of every CTA
  // status / bounded waits
  int* status = nullptr;
  uint64_t timeout_ns = 10ull * 1000 * 1000 * 1000;
  unsigned long long* debug = nullptr;  // optional per-CTA cycle counters (4 per CTA)
};

// Number of CTAs the persistent kernel will launch for this call (GEMM CTAs
// plus communication CTAs).
int grid_ctas(const GemmCall& c);
// GEMM-role CTAs of this call (0 when the call runs communication phases only).
int gemm_ctas(const GemmCall& c);
// Tile kind (0 single CTA 128x256, 2 wide CTA pair 256x512) the wave model picks
// for a fused launch whose GEMM runs on all SMs but `comm_ctas`.
int fused_tile_kind(int M, int N, int K, int comm_ctas);
// Mapping probe: writes (tile_m, tile_n) of every linear tile index as the
// kernel's CTAs decode them (explicit table or grouped raster) into out[2 * tiles].
int tile_map(const GemmCall& c, int* out, cudaStream_t stream);
int tile_count(const GemmCall& c);
int run(const GemmCall& c, cudaStream_t stream);
std::string last_error();

}  // namespace gemm
}  // namespace tn5b
