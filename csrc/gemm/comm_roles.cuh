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
//                peers' memory) into its local gather buffer and flags each
//                block (epoch) once it is stored; the GEMM CTAs wait for a
//                block's flag before their TMA loads read it (local memory).
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
  constexpr int kUnit = TILE_CC / 2;                 // pieces per work unit (half a flag tile)
  constexpr int kUnitsPerTile = TILE_CC / kUnit;
  const PullRsArgs& a = p.pull;
  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kCommStages * kPiece);
  uint64_t* empty = full + kCommStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kCommStages);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kCommStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kRedWarps);  // each stage is consumed by one group of kRedWarps warps
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
    // Work unit: half a flag tile (kUnit pieces), assigned round-robin over the
    // consumption order, so the GEMM's last tiles are spread over twice as many
    // reducer CTAs as whole tiles would be.  A unit first waits for the flags
    // of all W sources, then issues one proxy fence (each fence is paid with
    // the bulk loads in flight) before its loads.
    for (int q = cta; q < tiles * kUnitsPerTile && ok; q += ctas) {
      const int i = q / kUnitsPerTile;
      const int lt = a.order ? a.order[i] : i;
      const int ltm = lt / tiles_n, tn = lt % tiles_n;
      for (int s = 0; s < world && ok; ++s)
        ok = wait_flag_geq(a.my_flags + int64_t(s) * tiles + lt, p.rs.epoch, p.timeout_ns, p.status,
                           kTimeoutPeerFlag);
      if (!ok) break;
      fence_proxy_async_global();  // flag acquires before the bulk engine reads the pieces
      for (int pc = (q % kUnitsPerTile) * kUnit; pc < (q % kUnitsPerTile + 1) * kUnit && ok; ++pc) {
        const int64_t off = piece_offset(rb_base + ltm, tn * TILE_CC + pc, n_chunks);
        if (a.residual) {
          const int st = int(seq % kCommStages);
          const uint32_t ph = (seq / kCommStages) & 1u;
          if (!mbar_wait(&empty[st], ph ^ 1u, p.timeout_ns, p.status, kTimeoutProducerEmpty, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[st], kPiece);
          tma_load_2d(ring + st * kPiece, tres, &full[st], (tn * TILE_CC + pc) * 64, ltm * 128);
          last_parity[st] = int(ph);
          ++seq;
        }
        for (int s = 0; s < world; ++s) {
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
  // kRedGroups groups of four warps; group `grp` reduces the pieces whose
  // position in this CTA's piece sequence is grp modulo kRedGroups.  The loader
  // issues each piece's stages contiguously (residual, then W sources), so a
  // group finds its piece's first stage at piece_index * stages_per_piece.
  const int grp = (warp - 2) / kRedWarps;
  const int rt = threadIdx.x - 64 - grp * 128;  // 0..127 inside the group
  const uint32_t zero = 0u;                      // two +0.0 BF16 values
  const uint32_t stages_per_piece = uint32_t(world + (a.residual ? 1 : 0));
  uint32_t piece_index = 0;                      // pieces of this CTA seen so far
  for (int q = cta; q < tiles * kUnitsPerTile; q += ctas) {
    const int i = q / kUnitsPerTile;
    const int lt = a.order ? a.order[i] : i;
    const int ltm = lt / tiles_n, tn = lt % tiles_n;
    constexpr int pr = 0;
    for (int pc = (q % kUnitsPerTile) * kUnit; pc < (q % kUnitsPerTile + 1) * kUnit; ++pc, ++piece_index) {
      if (int(piece_index % kRedGroups) != grp) continue;
      uint32_t seq = piece_index * stages_per_piece;
      {
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
          uint32_t* o = acc + 4 * u;
          if (a.residual) {
            const uint4 r = res[u];
            o[0] = add_bf16x2(r.x, o[0]);
            o[1] = add_bf16x2(r.y, o[1]);
            o[2] = add_bf16x2(r.z, o[2]);
            o[3] = add_bf16x2(r.w, o[3]);
          }
          if (a.bias) {
            o[0] = add_bf16x2(o[0], bias4.x);
            o[1] = add_bf16x2(o[1], bias4.y);
            o[2] = add_bf16x2(o[2], bias4.z);
            o[3] = add_bf16x2(o[3], bias4.w);
          }
          *reinterpret_cast<uint4*>(a.out + idx) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    if (a.stamps) {
      // A flag tile is complete when its last piece is: keep the latest piece time.
      named_barrier_sync(2 + grp, kRedWarps * 32);
      if (rt == 0) atomicMax(a.stamps + lt, (unsigned long long)globaltimer_ns());
    }
  }
}

// --------------------------------------------------------------- gatherer
// Each gatherer CTA moves whole 128-row blocks (own-chunk copies and peer
// pulls), assigned round-robin over the sequence [own blocks, then every peer
// block in pull order rank+1, rank+2, ...].  One thread streams a block's
// 16 KB pieces through the ring (bulk load -> bulk store, up to kLoads loads in
// flight, two stages of slack for stores still reading), exactly the copy loop
// of the bulk-copy probe; synchronisation happens once per block: when the
// block's last store is kLag bulk groups old, the thread waits for it, then
// release-stores the block's epoch flag -- ready[c][b] (read by this GPU's
// GEMM CTAs) for a peer block, published[d][rank][b] on every peer d for an
// own block.  After the last piece this CTA loads from peer c has landed, it
// adds 1 to c's `pulled` counter.
struct BlockStream {
  static constexpr int kLoads = kCommStages - 2;
  static constexpr int kLag = 24;
  static constexpr int kJobs = 8;    // blocks whose completion is pending
  uint8_t* ring;
  uint64_t* full;
  const Params* p;
  uint32_t issued, stored;
  int last_parity[kCommStages];
  uint8_t* q_dst[kCommStages];
  uint32_t* q_landed[kCommStages];
  uint32_t q_bytes[kCommStages];
  int q_job[kCommStages];            // block (chunk * blocks + b) finished by this piece, or -1
  int jobs[kJobs];                   // pending blocks, by completion store index
  uint32_t job_store[kJobs];
  int job_head, job_tail;

  __device__ void init(uint8_t* r, uint64_t* f, const Params* params) {
    ring = r;
    full = f;
    p = params;
    issued = stored = 0;
    job_head = job_tail = 0;
    for (int s = 0; s < kCommStages; ++s) last_parity[s] = -1;
  }
  __device__ void finish_block(int blk) {
    const GatherArgs& g = p->gather;
    const int blocks = g.rows_per_src / 128;
    fence_proxy_async_global();
    if (blk / blocks == g.rank) {
      // Own block complete in local memory: release it to every peer.
      fence_acq_rel_sys();
      for (int d = 0; d < g.world; ++d)
        if (d != g.rank) st_release_sys(g.published[d] + blk, g.epoch);
    } else {
      st_release_gpu(g.ready + int64_t(blk) * kReadyStride, g.epoch);
    }
    if (g.block_stamps) g.block_stamps[blk] = globaltimer_ns();
  }
  // Publish every pending block whose last store is at least `lag` groups old.
  template <int LAG>
  __device__ void retire() {
    while (job_head != job_tail && job_store[job_head % kJobs] + LAG < stored) {
      bulk_wait_group<LAG>();
      finish_block(jobs[job_head % kJobs]);
      ++job_head;
    }
  }
  __device__ bool store_one() {
    const int st = int(stored % kCommStages);
    const uint32_t ph = (stored / kCommStages) & 1u;
    if (!mbar_wait(&full[st], ph, p->timeout_ns, p->status, kTimeoutPeerFlag, nullptr)) return false;
    if (q_landed[st]) red_release_sys_add(q_landed[st], 1u);
    bulk_store(q_dst[st], smem_u32(ring + st * kPiece), q_bytes[st]);
    bulk_commit_group();
    if (q_job[st] >= 0) {
      jobs[job_tail % kJobs] = q_job[st];
      job_store[job_tail % kJobs] = stored;
      ++job_tail;
    }
    ++stored;
    retire<kLag>();
    return true;
  }
  __device__ bool push(const uint8_t* src, uint8_t* dst, uint32_t bytes, int job, uint32_t* landed) {
    if (issued - stored == uint32_t(kLoads) && !store_one()) return false;
    // A block completion may not be queued while kJobs are pending.
    if (job >= 0 && job_tail - job_head >= kJobs - 1) {
      while (stored < issued)
        if (!store_one()) return false;
      retire<0>();
    }
    const int st = int(issued % kCommStages);
    if (issued >= uint32_t(kCommStages)) bulk_wait_group_read<kCommStages - kLoads - 1>();
    q_dst[st] = dst;
    q_landed[st] = landed;
    q_bytes[st] = bytes;
    q_job[st] = job;
    mbar_arrive_expect_tx(&full[st], bytes);
    bulk_load(ring + st * kPiece, src, bytes, &full[st]);
    last_parity[st] = int((issued / kCommStages) & 1u);
    ++issued;
    return true;
  }
  __device__ bool finish() {
    while (stored < issued)
      if (!store_one()) return false;
    retire<0>();
    bulk_wait_group_all();
    return true;
  }
  __device__ void drain() {
    for (int s = 0; s < kCommStages; ++s)
      if (last_parity[s] >= 0)
        mbar_wait(&full[s], uint32_t(last_parity[s]), p->timeout_ns, p->status, kTimeoutDrain, nullptr);
    bulk_wait_group_all();
  }
};

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
  const int pieces = int((block_bytes + kPiece - 1) / kPiece);
  const int blocks = g.rows_per_src / 128;
  uint8_t* local = g.gather[rank];
  BlockStream bs;
  bs.init(ring, full, &p);
  bool ok = true;
  // Stream one block (pieces in order); the last piece carries the block's
  // completion and, if given, the landed signal to its source.
  auto stream_block = [&](const uint8_t* src, uint8_t* dst, int job, uint32_t* landed) -> bool {
    for (int k = 0; k < pieces; ++k) {
      const int64_t off = int64_t(k) * kPiece;
      const uint32_t bytes = uint32_t(min(int64_t(kPiece), block_bytes - off));
      const bool last = k == pieces - 1;
      if (!bs.push(src + off, dst + off, bytes, last ? job : -1, last ? landed : nullptr)) return false;
    }
    return true;
  };
  // Job sequence: own blocks 0..blocks-1, then peer (rank+step) block b as job
  // blocks + (step-1) * blocks + b; this CTA takes jobs cta, cta + ctas, ...
  if ((g.phase & 1) && g.own_in_place) {
    // The caller wrote the shard straight into the own chunk (after a bounded
    // wait for the peers' previous reads, launched before the writer): the
    // blocks are complete in local memory since the previous kernel -- release
    // them to every peer.
    for (int b = cta; b < blocks; b += ctas) {
      fence_acq_rel_sys();
      for (int d = 0; d < world; ++d)
        if (d != rank) st_release_sys(g.published[d] + rank * blocks + b, g.epoch);
    }
  }
  const int own_jobs = ((g.phase & 1) && !g.own_in_place) ? blocks : 0;
  const int total = own_jobs + ((g.phase & 2) ? (world - 1) * blocks : 0);
  if (own_jobs) {
    // Own chunk: overwrite it only once every peer has finished reading the
    // previous call's contents.
    if (!wait_flag_geq(g.pulled_local, g.pulled_target, p.timeout_ns, p.status, kTimeoutPeerFlag)) return;
    fence_proxy_async_global();
  }
  // This CTA's last job per peer step (its `pulled` signal rides on that block).
  int last_of_step[64];
  for (int s = 0; s < world; ++s) last_of_step[s] = -1;
  for (int j = cta; j < total; j += ctas)
    if (j >= own_jobs) last_of_step[1 + (j - own_jobs) / blocks] = j;
  if (g.phase & 2)
    for (int step = 1; step < world; ++step)
      if (last_of_step[step] < 0) red_release_sys_add(g.pulled[(rank + step) % world], 1u);  // reads nothing
  bool own_published = own_jobs == 0;
  for (int j = cta; j < total && ok; j += ctas) {
    if (j < own_jobs) {
      const int64_t off = int64_t(j) * block_bytes;
      ok = stream_block(g.shard + off, local + int64_t(rank) * g.chunk_bytes + off, rank * blocks + j, nullptr);
      continue;
    }
    if (!own_published) {
      // The stream publishes a block only once its stores are kLag groups old.
      // Before this CTA waits for a peer's block, every own block it copied
      // must be published: the peer's CTA may be waiting for one of ours the
      // same way (with few blocks per rank that wait is circular).
      ok = bs.finish();
      own_published = true;
      if (!ok) break;
    }
    const int step = 1 + (j - own_jobs) / blocks, b = (j - own_jobs) % blocks;
    const int c = (rank + step) % world;
    if (!wait_flag_geq(g.published_local + c * blocks + b, g.epoch, p.timeout_ns, p.status, kTimeoutAgChunk)) {
      ok = false;
      break;
    }
    fence_proxy_async_global();
    const int64_t off = int64_t(c) * g.chunk_bytes + int64_t(b) * block_bytes;
    ok = stream_block(g.gather[c] + off, local + off, c * blocks + b, j == last_of_step[step] ? g.pulled[c] : nullptr);
  }
  if (ok) ok = bs.finish();
  if (!ok) bs.drain();
}

}  // namespace gemm
}  // namespace tn5b
