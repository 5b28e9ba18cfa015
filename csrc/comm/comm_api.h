// Symmetric-memory plumbing: CUDA IPC export/import of device allocations so
// every rank can address every peer's buffer over NVLink, plus the receiver
// kernels of the fused reduce-scatter (ordered BF16 reduce, fused TACO
// decode + ordered reduce) with bounded per-tile readiness waits.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace tn5b {
namespace comm {

struct RsReduceCall {
  const uint8_t* recv = nullptr;   // this rank's receive regions [lane][world][slot_bytes] (push_lanes.h)
  const uint32_t* flags = nullptr; // this rank's flags [lane][world][lane tiles]
  int64_t slot_bytes = 0;          // one lane region of one source (PushLanes::lane_slot_bytes)
  int rank = 0, world = 1;
  int rows = 0, n = 0;             // output [rows, n] (rows = M / world)
  int tile_n = 256;                // producer tile width (flag granularity)
  int chunk_rows = 128;            // TACO block rows
  int quantized = 0;               // remote slots hold TACO packets
  uint32_t epoch = 0;
  void* out = nullptr;             // bf16 [rows, n]
  const void* residual = nullptr;  // optional bf16 [rows, n]: out = bf16(bf16(res + y) + bias)
  const void* bias = nullptr;      // optional bf16 [n]
  const int* tile_order = nullptr; // optional consumption order of local tiles
  int arrival = 0;                 // 1: per-lane any-ready consumption (arrival-first)
  int* claims = nullptr;           // arrival mode: per-tile claim words [tiles]
  unsigned long long* stamps = nullptr;  // optional: %globaltimer at each tile's completion
  int* status = nullptr;
  uint64_t timeout_ns = 0;
  int max_ctas = 0;
};
int rs_reduce(const RsReduceCall& c, cudaStream_t stream);

}  // namespace comm
}  // namespace tn5b

namespace tn5b {
namespace comm {
// 16-byte-aligned device copy (dst may be a peer's IPC-mapped memory); ctas <= 0: 4 per SM.
int copy16(void* dst, const void* src, int64_t bytes, int ctas, cudaStream_t stream);
// Bulk-engine copy through shared memory (src may be a peer's IPC mapping; untiled
// bulk loads without multicast; dst is this GPU's memory): `ctas` CTAs of one
// issuing thread, `stages` x `chunk` bytes in flight per CTA.
int bulk_copy(void* dst, const void* src, int64_t bytes, int ctas, int chunk, int stages, uint64_t timeout_ns,
              int* status, cudaStream_t stream);
int wait_probe(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status,
               cudaStream_t stream);
// Pull reduce-scatter of an existing tensor: pack it into the partial buffer's
// [M/128][N/64][128][64] layout, then release its flag tiles to their owners.
int pack_pieces(const void* src, int64_t ld, void* dst, int M, int N, cudaStream_t stream);
int publish_tiles(uint32_t* const* flags, int rank, int world, int per_dest, uint32_t epoch, cudaStream_t stream);
}  // namespace comm
}  // namespace tn5b
