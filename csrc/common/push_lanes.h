// Lanes of the push transport of the fused GEMM -> reduce-scatter.
//
// A destination's M/W rows are cut into blocks of `chunk_rows` rows; block b
// travels on lane b % 2, the way the reference splits its per-block exchange
// over two lane communicators and streams (python/flux_5090/runtime.py:50-56,
// 192-214).  Here a lane is a channel in the owner's memory: its own receive
// region and its own flag array, written by the producers' epilogues and
// consumed lane by lane by the receiver.
//
//   receive regions: [lane][source][lane block][block bytes]
//   flags:           [lane][source][lane tile]   (producer tiles of 128 rows x tile_n)
//
// Lane block j of lane l is the destination's block 2j + l.  Both lanes are
// sized for ceil(blocks / 2) blocks, so a region's offset does not depend on
// the lane's parity.  The same arithmetic runs on the host (slot sizes,
// validation) and on the device (producer stores, receiver loads).
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define TN5B_HD __host__ __device__ __forceinline__
#else
#define TN5B_HD inline
#endif

namespace tn5b {

struct PushLanes {
  int rows_per_dest = 0;  // M / world
  int n = 0;              // GEMM N (output columns)
  int chunk_rows = 128;   // block rows (a multiple of 128 dividing rows_per_dest)
  int world = 1;
  int tile_n = 256;       // producer tile width (flag granularity)

  TN5B_HD int blocks() const { return rows_per_dest / chunk_rows; }
  TN5B_HD int lane_blocks() const { return (blocks() + 1) / 2; }
  TN5B_HD int tiles_n() const { return n / tile_n; }
  TN5B_HD int lane_tiles() const { return lane_blocks() * (chunk_rows / 128) * tiles_n(); }
  // One lane's region of one source: BF16 blocks (a TACO packet is smaller).
  TN5B_HD int64_t lane_slot_bytes() const { return int64_t(lane_blocks()) * chunk_rows * n * 2; }
  TN5B_HD int64_t recv_bytes() const { return 2 * int64_t(world) * lane_slot_bytes(); }
  TN5B_HD int64_t flag_words() const { return 2 * int64_t(world) * lane_tiles(); }

  // Destination-local row -> lane, and row inside the lane's packed blocks.
  TN5B_HD int lane_of(int row_local) const { return (row_local / chunk_rows) & 1; }
  TN5B_HD int lane_row(int row_local) const {
    return ((row_local / chunk_rows) >> 1) * chunk_rows + row_local % chunk_rows;
  }
  TN5B_HD int64_t slot_offset(int lane, int source) const {
    return (int64_t(lane) * world + source) * lane_slot_bytes();
  }
  // Flag of the producer tile whose first row is `row_local` (a multiple of 128)
  // and whose column tile is `tn`.
  TN5B_HD int64_t flag_index(int source, int row_local, int tn) const {
    const int lane = lane_of(row_local);
    return (int64_t(lane) * world + source) * lane_tiles() + int64_t(lane_row(row_local) / 128) * tiles_n() + tn;
  }
};

}  // namespace tn5b
