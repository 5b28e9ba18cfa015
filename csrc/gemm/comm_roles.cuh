// Communication roles of the fused GEMM kernels: CTAs [0, comm_ctas) of a
// gemm_kernel launch do not compute; they move data over NVLink with the bulk
// copy engine while the other CTAs run the tcgen05 GEMM.
//
//   rs_reducer   (GEMM -> reduce-scatter, kModeRsPull)  every rank's GEMM CTAs
//                write their BF16 partial tiles into a LOCAL buffer and
//                release-store one epoch flag per tile on the tile's owner.  The
//                owner's reducer CTAs wait (bounded) on the flags of each of
//                their tiles, pull the 16 KB pieces of that tile from every
//                source (untiled bulk loads from the peers' memory, no
//                multicast) into a shared-memory ring and reduce them in source
//                order 0..W-1 with BF16 rounding after every source, fusing
//                residual + bias, while the GEMM is still producing later tiles.
//   ag_gatherer  (all-gather -> GEMM)  each rank copies its own shard into its
//                own chunk of its gather buffer and publishes every 128-row
//                block to every peer as soon as the block is complete; every
//                rank pulls the peers' published blocks (bulk loads from the
//                peers' memory) into its local gather buffer and counts the
//                arrived 16 KB pieces per block; the GEMM CTAs wait for a
//                block's count before their TMA loads read it (local memory).
//                After its last load from a peer a gatherer CTA adds 1 to that
//                peer's `pulled` counter; a rank overwrites its own chunk only
//                after every peer's CTAs have signalled for the previous call,
//                so back-to-back calls never overwrite data a peer still reads.
//
// One thread of each communication CTA drives the bulk engine (one issuing
// thread per CTA reached the NVLink ceiling with 16-24 CTAs on B200); in the
// reducer four more warps do the arithmetic.  Every wait is bounded: on a
// timeout the CTA records a status code, waits (bounded) for its own loads in
// flight and returns.
//
// Reference parity: this replaces the per-block stream waits, sparse
// all_to_all lanes and consumer streams of TempName-5090
// python/flux_5090/runtime.py:189-231 (and its all_gather + GEMM,
// model.py:110-117) with in-kernel roles.
#pragma once

namespace tn5b {
namespace gemm {

constexpr int kPiece = 128 * 64 * 2;   // one 128-row x 64-column BF16 piece (16 KB)
constexpr int kCommStages = 12;        // shared-memory ring depth of a communication CTA
constexpr int kRedWarps = 4;           // reducer arithmetic warps (warps 2..5)

// Byte offset of piece (row block rb, column chunk cc) in a partial buffer laid
// out [M/128][N/64][128][64] (the GEMM's TMA stores write this layout).
__device__ __forceinline__ int64_t piece_offset(int rb, int cc, int n_chunks) {
  return (int64_t(rb) * n_chunks + cc) * kPiece;
}

__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  // IEEE round-to-nearest-even BF16 add: for BF16 operands this equals
  // bf16(fp32(a) + fp32(b)) (the FP32 sum of two BF16 values is exact unless
  // one operand is below half an ulp of the other), i.e. the reference's
  // "add in FP32, round to BF16 after every source".
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_acq_rel_gpu_add(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// ---------------------------------------------------------------- reducer
// Flag tiles are 128 rows x TILE_CC 64-column chunks of this rank's rows (one
// GEMM CTA's share of a tile); the flag of (source s, local flag tile t) is
// my_flags[s * tiles + t].
// `tres` maps the residual [rows_per_dest, N] (box 64 x 128, 128-byte swizzle):
// with a residual, the loader brings each piece's residual tile into the ring
// ahead of the piece's sources, so it never waits on a global load.
template <int TILE_CC>
__device__ void rs_reducer(const Params& p, uint8_t* smem, const CUtensorMap* tres) {
  constexpr int TILE_RB = 1;
  const PullRsArgs& a = p.pull;
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kCommStages * kPiece);
  uint64_t* empty = full + kCommStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kCommStages);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kCommStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRedWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int cta = int(blockIdx.x);
  const int ctas = p.comm_ctas;
  const int world = p.rs.world;
  const int tiles = a.tiles_per_dest;
  const int tiles_n = a.tiles_n;
  const int n_chunks = p.N / 64;
  const int rb_base = p.rs.rank * (p.rs.rows_per_dest / 128);  // first global row block of my rows

  if (warp == 0) {
    if (lane != 0) return;
    // ------------------------------------------------------------ loader
    uint32_t seq = 0;
    int last_parity[kCommStages];
#pragma unroll
    for (int s = 0; s < kCommStages; ++s) last_parity[s] = -1;
    bool ok = true;
    for (int i = cta; i < tiles && ok; i += ctas) {
      const int lt = a.order ? a.order[i] : i;
      const int ltm = lt / tiles_n, tn = lt % tiles_n;
      uint32_t waited = 0;
      for (int pr = 0; pr < TILE_RB && ok; ++pr) {
        for (int pc = 0; pc < TILE_CC && ok; ++pc) {
          const int64_t off = piece_offset(rb_base + ltm * TILE_RB + pr, tn * TILE_CC + pc, n_chunks);
          if (a.residual) {
            const int st = int(seq % kCommStages);
            const uint32_t ph = (seq / kCommStages) & 1u;
            if (!mbar_wait(&empty[st], ph ^ 1u, p.timeout_ns, p.status, kTimeoutProducerEmpty, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[st], kPiece);
            tma_load_2d(ring + st * kPiece, tres, &full[st], (tn * TILE_CC + pc) * 64, (ltm * TILE_RB + pr) * 128);
            last_parity[st] = int(ph);
            ++seq;
          }
          for (int s = 0; s < world; ++s) {
            if (!((waited >> s) & 1u)) {
              if (!wait_flag_geq(a.my_flags + int64_t(s) * tiles + lt, p.rs.epoch, p.timeout_ns, p.status,
                                 kTimeoutPeerFlag)) {
                ok = false;
                break;
              }
              fence_proxy_async_global();  // flag acquire before the bulk engine reads the piece
              waited |= 1u << s;
            }
            const int st = int(seq % kCommStages);
            const uint32_t ph = (seq / kCommStages) & 1u;
            if (!mbar_wait(&empty[st], ph ^ 1u, p.timeout_ns, p.status, kTimeoutProducerEmpty, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[st], kPiece);
            bulk_load(ring + st * kPiece, a.partial[s] + off, kPiece, &full[st]);
            last_parity[st] = int(ph);
            ++seq;
          }
        }
      }
    }
    if (!ok) {
      *abort_flag = 1;
      for (int s = 0; s < kCommStages; ++s)
        if (last_parity[s] >= 0)
          mbar_wait(&full[s], uint32_t(last_parity[s]), p.timeout_ns, p.status, kTimeoutDrain, nullptr);
    }
    return;
  }
  if (warp < 2) return;
  // --------------------------------------------------------- reducer warps
  const int rt = threadIdx.x - 64;  // 0..127
  const uint32_t zero = 0u;         // two +0.0 BF16 values
  uint32_t seq = 0;
  for (int i = cta; i < tiles; i += ctas) {
    const int lt = a.order ? a.order[i] : i;
    const int ltm = lt / tiles_n, tn = lt % tiles_n;
    for (int pr = 0; pr < TILE_RB; ++pr) {
      for (int pc = 0; pc < TILE_CC; ++pc) {
        // This thread's eight 16-byte units: unit rt + 128u is row rt/8 + 16u,
        // columns (rt % 8) * 8 .. +8 of the piece.  The residual tile arrives in
        // the ring first (swizzled: unit c of row r sits at c ^ (r & 7)); the
        // bias load is issued here and completes during the source loop.
        const int col = (tn * TILE_CC + pc) * 64 + (rt % 8) * 8;
        const int row0 = (ltm * TILE_RB + pr) * 128 + rt / 8;
        uint4 bias4 = make_uint4(0, 0, 0, 0);
        if (a.bias) bias4 = ld_global_nc_v4(a.bias + col);
        uint4 res[8];
        if (a.residual) {
          const int st = int(seq % kCommStages);
          const uint32_t ph = (seq / kCommStages) & 1u;
          if (!warp_wait(&full[st], ph, p.timeout_ns, p.status, kTimeoutMmaFull, abort_flag)) return;
          const uint32_t buf = smem_u32(ring + st * kPiece);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int r = rt / 8 + 16 * u;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(res[u].x), "=r"(res[u].y), "=r"(res[u].z), "=r"(res[u].w)
                         : "r"(buf + uint32_t(r * 128 + (((rt % 8) ^ (r & 7)) << 4))));
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[st]);
          ++seq;
        }
        uint32_t acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = zero;
        for (int s = 0; s < world; ++s) {
          const int st = int(seq % kCommStages);
          const uint32_t ph = (seq / kCommStages) & 1u;
          if (!warp_wait(&full[st], ph, p.timeout_ns, p.status, kTimeoutMmaFull, abort_flag)) return;
          const uint32_t buf = smem_u32(ring + st * kPiece);
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            uint32_t v0, v1, v2, v3;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(v0), "=r"(v1), "=r"(v2), "=r"(v3)
                         : "r"(buf + uint32_t(rt + 128 * u) * 16u));
            acc[4 * u + 0] = add_bf16x2(acc[4 * u + 0], v0);
            acc[4 * u + 1] = add_bf16x2(acc[4 * u + 1], v1);
            acc[4 * u + 2] = add_bf16x2(acc[4 * u + 2], v2);
            acc[4 * u + 3] = add_bf16x2(acc[4 * u + 3], v3);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[st]);
          ++seq;
        }
        // Epilogue: out = bf16(bf16(residual + y) + bias), written to this rank's rows.
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int64_t idx = int64_t(row0 + 16 * u) * p.N + col;
          uint32_t* q = acc + 4 * u;
          if (a.residual) {
            const uint4 r = res[u];
            q[0] = add_bf16x2(r.x, q[0]);
            q[1] = add_bf16x2(r.y, q[1]);
            q[2] = add_bf16x2(r.z, q[2]);
            q[3] = add_bf16x2(r.w, q[3]);
          }
          if (a.bias) {
            q[0] = add_bf16x2(q[0], bias4.x);
            q[1] = add_bf16x2(q[1], bias4.y);
            q[2] = add_bf16x2(q[2], bias4.z);
            q[3] = add_bf16x2(q[3], bias4.w);
          }
          *reinterpret_cast<uint4*>(a.out + idx) = make_uint4(q[0], q[1], q[2], q[3]);
        }
      }
    }
    if (a.stamps) {
      named_barrier_sync(2, kRedWarps * 32);
      if (rt == 0) a.stamps[lt] = globaltimer_ns();
    }
  }
}

// --------------------------------------------------------------- gatherer
// The single issuing thread streams a sequence of pieces (source address, local
// destination) through the ring: up to kLoads loads are in flight, each landed
// piece is bulk-stored to local memory.  Pieces travel in runs (consecutive
// pieces of one 128-row block): synchronisation happens once per run, not per
// piece -- when a run's last store has completed (confirmed kLag bulk groups
// late, so the engine never waits for a write to land) the block's counter is
// advanced by the run's length.  The ring keeps kCommStages - kLoads stages of
// slack, so reusing a stage never waits for the store just issued to finish
// reading shared memory.  A piece may carry a remote counter to bump (release,
// system scope) once it has landed: the "no longer reading" signal to its source.
struct PieceStream {
  static constexpr int kLoads = kCommStages - 2;
  static constexpr int kLag = 24;
  uint8_t* ring;
  uint64_t* full;
  const Params* p;
  uint32_t issued, stored;            // pieces loaded / stored
  uint32_t* pending[kLag + 1];        // run counters to advance, by store index of the run's last piece
  uint32_t pending_n[kLag + 1];
  int last_parity[kCommStages];
  uint8_t* q_dst[kCommStages];
  uint32_t* q_ctr[kCommStages];       // set on a run's last piece
  uint32_t q_n[kCommStages];          // that run's length
  uint32_t* q_landed[kCommStages];
  uint32_t q_bytes[kCommStages];

  __device__ void init(uint8_t* r, uint64_t* f, const Params* params) {
    ring = r;
    full = f;
    p = params;
    issued = stored = 0;
    for (int s = 0; s < kCommStages; ++s) last_parity[s] = -1;
    for (int j = 0; j <= kLag; ++j) pending[j] = nullptr;
  }
  // Store the oldest landed piece.  Returns false on a timeout.
  __device__ bool store_one() {
    const int st = int(stored % kCommStages);
    const uint32_t ph = (stored / kCommStages) & 1u;
    if (!mbar_wait(&full[st], ph, p->timeout_ns, p->status, kTimeoutPeerFlag, nullptr)) return false;
    if (q_landed[st]) red_release_sys_add(q_landed[st], 1u);
    bulk_store(q_dst[st], smem_u32(ring + st * kPiece), q_bytes[st]);
    bulk_commit_group();
    const int slot = int(stored % (kLag + 1));
    pending[slot] = q_ctr[st];
    pending_n[slot] = q_n[st];
    ++stored;
    // The store issued kLag groups ago has completed: advance its run's counter.
    const int done = int(stored % (kLag + 1));  // store index stored - 1 - kLag
    if (pending[done]) {
      bulk_wait_group<kLag>();
      fence_proxy_async_global();
      count(pending[done], pending_n[done]);
      pending[done] = nullptr;
    }
    return true;
  }
  // Queue one piece (ctr/n on a run's last piece); stores the oldest piece first
  // when kLoads are in flight.
  __device__ bool push(const uint8_t* src, uint8_t* dst, uint32_t bytes, uint32_t* ctr, uint32_t n,
                       uint32_t* landed) {
    if (issued - stored == uint32_t(kLoads) && !store_one()) return false;
    const int st = int(issued % kCommStages);
    // The stage's previous piece (issued - kCommStages) was stored at least
    // kCommStages - kLoads stores ago: all but the newest store have read their stage.
    if (issued >= uint32_t(kCommStages)) bulk_wait_group_read<kCommStages - kLoads - 1>();
    q_dst[st] = dst;
    q_ctr[st] = ctr;
    q_n[st] = n;
    q_landed[st] = landed;
    q_bytes[st] = bytes;
    mbar_arrive_expect_tx(&full[st], bytes);
    bulk_load(ring + st * kPiece, src, bytes, &full[st]);
    last_parity[st] = int((issued / kCommStages) & 1u);
    ++issued;
    return true;
  }
  // Store everything queued and advance every counter.
  __device__ bool finish() {
    while (stored < issued)
      if (!store_one()) return false;
    bulk_wait_group_all();
    fence_proxy_async_global();
    for (int j = 0; j <= kLag; ++j) {
      if (pending[j]) count(pending[j], pending_n[j]);
      pending[j] = nullptr;
    }
    return true;
  }
  // A run of n pieces of one block is stored.  The run that completes an
  // own-chunk block publishes the block to every peer; with block stamps the
  // completing run also records the time.
  __device__ void count(uint32_t* ctr, uint32_t n) {
    const GatherArgs& g = p->gather;
    const int64_t idx = ctr - g.ready;
    const int blocks = g.rows_per_src / 128;
    const bool own = idx / blocks == g.rank;
    if (!own && !g.block_stamps) {
      red_release_gpu_add(ctr, n);
      return;
    }
    if (atom_acq_rel_gpu_add(ctr, n) + n != g.ready_target) return;
    if (g.block_stamps) g.block_stamps[idx] = globaltimer_ns();
    if (own) {
      // Every piece of own block idx % blocks is in local memory (acquired through
      // the counter): release it to the peers at system scope.
      fence_acq_rel_sys();
      const int b = int(idx % blocks);
      for (int d = 0; d < g.world; ++d)
        if (d != g.rank) st_release_sys(g.published[d] + g.rank * blocks + b, g.epoch);
    }
  }
  // Abort path: wait (bounded) for every load in flight, then for the stores.
  __device__ void drain() {
    for (int s = 0; s < kCommStages; ++s)
      if (last_parity[s] >= 0)
        mbar_wait(&full[s], uint32_t(last_parity[s]), p->timeout_ns, p->status, kTimeoutDrain, nullptr);
    bulk_wait_group_all();
  }
};

constexpr int kRunPieces = 8;  // pieces per run (128 KB): one counter update per run

__device__ void ag_gatherer(const Params& p, uint8_t* smem) {
  if (threadIdx.x != 0) return;
  const GatherArgs& g = p.gather;
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kCommStages * kPiece);
  for (int s = 0; s < kCommStages; ++s) mbar_init(&full[s], 1);
  fence_mbar_init();
  const int cta = int(blockIdx.x);
  const int ctas = p.comm_ctas;
  const int rank = g.rank, world = g.world;
  const int64_t block_bytes = int64_t(128) * g.K * 2;
  const int pieces_per_block = int((block_bytes + kPiece - 1) / kPiece);
  const int runs_per_block = (pieces_per_block + kRunPieces - 1) / kRunPieces;
  const int blocks = g.rows_per_src / 128;
  const int runs = runs_per_block * blocks;  // per chunk
  uint8_t* local = g.gather[rank];
  PieceStream ps;
  ps.init(ring, full, &p);
  bool ok = true;
  // Queue run r of a chunk (src / dst chunk bases); `landed` on its last piece.
  auto queue_run = [&](const uint8_t* src, uint8_t* dst, int chunk, int r, uint32_t* landed) -> bool {
    const int b = r / runs_per_block;
    const int first = (r % runs_per_block) * kRunPieces;
    const int n = min(kRunPieces, pieces_per_block - first);
    uint32_t* ctr = g.ready + int64_t(chunk) * blocks + b;
    for (int k = first; k < first + n; ++k) {
      const int64_t off = b * block_bytes + int64_t(k) * kPiece;
      const uint32_t bytes = uint32_t(min(int64_t(kPiece), block_bytes - int64_t(k) * kPiece));
      const bool last = k == first + n - 1;
      if (!ps.push(src + off, dst + off, bytes, last ? ctr : nullptr, last ? uint32_t(n) : 0u,
                   last ? landed : nullptr))
        return false;
    }
    return true;
  };

  if (g.phase & 1) {
    // Own shard -> own chunk of the gather buffer, once every peer has finished
    // reading this chunk's previous contents.  Each block is published to the
    // peers as soon as its last run is stored (PieceStream::count).
    if (!wait_flag_geq(g.pulled_local, g.pulled_target, p.timeout_ns, p.status, kTimeoutPeerFlag)) return;
    fence_proxy_async_global();
    uint8_t* own = local + int64_t(rank) * g.chunk_bytes;
    for (int r = cta; r < runs && ok; r += ctas) ok = queue_run(g.shard, own, rank, r, nullptr);
    if (ok) ok = ps.finish();
    if (!ok) {
      ps.drain();
      return;
    }
  }
  if (g.phase & 2) {
    // Peers' chunks, rank+1 first (every rank reads a different peer at a
    // time), each 128-row block once its owner has published it.
    for (int step = 1; step < world && ok; ++step) {
      const int c = (rank + step) % world;
      const uint8_t* src = g.gather[c] + int64_t(c) * g.chunk_bytes;
      uint8_t* dst = local + int64_t(c) * g.chunk_bytes;
      int last = -1;  // this CTA's last run of chunk c
      for (int r = cta; r < runs; r += ctas) last = r;
      if (last < 0) red_release_sys_add(g.pulled[c], 1u);  // nothing to read from c
      int waited = -1;
      for (int r = cta; r < runs && ok; r += ctas) {
        const int b = r / runs_per_block;
        if (b != waited) {
          if (!wait_flag_geq(g.published_local + c * blocks + b, g.epoch, p.timeout_ns, p.status,
                             kTimeoutAgChunk)) {
            ok = false;
            break;
          }
          fence_proxy_async_global();
          waited = b;
        }
        ok = queue_run(src, dst, c, r, r == last ? g.pulled[c] : nullptr);
      }
    }
    if (ok) ok = ps.finish();
    if (!ok) ps.drain();
  }
}

}  // namespace gemm
}  // namespace tn5b
