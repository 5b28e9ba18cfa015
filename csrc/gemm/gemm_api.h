// Host-side API of the tcgen05 GEMM family (plain, GEMM->reduce-scatter push,
// all-gather->GEMM).  Pointers are device pointers; all launches are async on
// the given stream.  Returns 0 or a cudaError_t / negative argument code.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <string>

namespace tn5b {
namespace gemm {

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
  int64_t slot_bytes = 0;
  int delay_tile = -1;         // diagnostic: bounded publication delay of one tile
  uint64_t delay_ns = 0;
  // all-gather
  int ag = 0;
  const uint32_t* ag_chunk_flags = nullptr;
  uint32_t ag_target = 0;
  const void* ag_shard = nullptr;
  int64_t ag_shard_bytes = 0;
  uint8_t* const* ag_gather = nullptr;
  uint32_t* const* ag_peer_flags = nullptr;
  // status / bounded waits
  int* status = nullptr;
  uint64_t timeout_ns = 10ull * 1000 * 1000 * 1000;
  unsigned long long* debug = nullptr;  // optional per-CTA cycle counters (4 per CTA)
};

// Number of CTAs the persistent kernel will launch for this call.
int grid_ctas(const GemmCall& c);
int run(const GemmCall& c, cudaStream_t stream);
std::string last_error();

}  // namespace gemm
}  // namespace tn5b
