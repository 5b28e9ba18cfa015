"""CPU models of kernel index arithmetic and protocols (no GPU).

Each test restates one formula or loop of a CUDA kernel and checks the property
the kernel relies on:

* GEMM grouped raster (`tile_coords` in csrc/gemm/gemm_kernel.cuh): a bijection
  from linear tile ids to (tile_m, tile_n) for every tile kind's tile counts.
* Attention packed probabilities (`packed_col` for the forward softmax,
  `bwd_packed_col` / `softmax_grad_row` for the backward, in
  csrc/kernels/attention_tc.cu): the MMA's K-chunk kk finds exactly the BF16
  pairs the elementwise warp of its half (forward) or column quarter (backward)
  wrote, and each warp writes only inside the score columns it alone reads.
* Pull GemmRS buffer reuse (`GemmRS` parity buffers, `rs_reducer`): with ranks
  at arbitrary relative speeds, no reducer reads a source's partial buffer
  after that source overwrote it with a later call's partial.
* AG gatherer job schedule (`ag_gatherer` in csrc/gemm/comm_roles.cuh): with
  own blocks published before a CTA's first wait on a peer's block, every
  rank's CTAs finish for every shape; with the publication lagging behind later
  stores only, the eight-blocks-per-rank shape of the bench deadlocks.
* Arrival-first receiver (`rs_reduce_kernel` in csrc/comm/comm.cu): with tiles
  becoming ready in any order, the per-lane claim loop (low-water mark, scan
  window, spread offsets, cyclic nearest ready tile, CAS) claims every tile
  exactly once and every CTA exits.
"""
import random

import pytest


def tile_coords(t, tiles_m, tiles_n, group_m):
    group_size = group_m * tiles_n
    group = t // group_size
    first_m = group * group_m
    size_m = min(tiles_m - first_m, group_m)
    r = t % group_size
    return first_m + r % size_m, r // size_m


@pytest.mark.parametrize("M,N", [(8192, 4096), (8192, 12288), (1000, 520), (50304, 4096), (256, 256)])
@pytest.mark.parametrize("kind", ["single", "pair", "wide"])
@pytest.mark.parametrize("group_m", [1, 8, 16])
def test_grouped_raster_is_a_bijection(M, N, kind, group_m):
    tile_m = 128 if kind == "single" else 256
    tile_n = 512 if kind == "wide" else 256
    tiles_m, tiles_n = -(-M // tile_m), -(-N // tile_n)
    seen = {tile_coords(t, tiles_m, tiles_n, group_m) for t in range(tiles_m * tiles_n)}
    assert seen == {(i, j) for i in range(tiles_m) for j in range(tiles_n)}
    # Every output element is covered once by the CTA(s) of its tile.
    ctas = 1 if kind == "single" else 2
    rows = set()
    for tm in range(tiles_m):
        for rank in range(ctas):
            start = tm * tile_m + rank * 128
            rows.update(range(start, min(start + 128, M)))
    assert rows == set(range(M))


def packed_col(kk):
    return (kk >> 2) * 64 + (kk & 3) * 8


def test_attention_packed_probability_columns():
    # Where softmax_grad_row / the forward softmax put the BF16 pair of score
    # columns (2i, 2i+1): warp half h handles score columns [64h, 64h+64) in two
    # 32-column quarters q2 and packs quarter q2's pair p at 64h + 16*q2 + p.
    location = {}
    for half in range(2):
        for q2 in range(2):
            for p in range(16):
                c = 64 * half + 32 * q2 + 2 * p
                location[c] = 64 * half + 16 * q2 + p
        own = set(range(64 * half, 64 * half + 64))
        written = {64 * half + 16 * q2 + p for q2 in range(2) for p in range(16)}
        assert written <= own  # writes stay inside the columns this warp alone reads
    # The MMA reads K-chunk kk (score columns 16kk..16kk+15) as 8 packed columns.
    for kk in range(8):
        want = [location[16 * kk + 2 * j] for j in range(8)]
        assert want == list(range(packed_col(kk), packed_col(kk) + 8))


def bwd_packed_col(kk):
    return (kk >> 1) * 32 + (kk & 1) * 8


def test_attention_backward_packed_columns_per_quarter():
    # Backward: one warp per 32-column quarter q of a lane quarter; it reads
    # score columns [32q, 32q+32) and packs pair p (columns 32q+2p, +1) at 32q+p.
    location = {}
    for q in range(4):
        for p in range(16):
            location[32 * q + 2 * p] = 32 * q + p
        written = {32 * q + p for p in range(16)}
        assert written <= set(range(32 * q, 32 * q + 32))
    for kk in range(8):
        want = [location[16 * kk + 2 * j] for j in range(8)]
        assert want == list(range(bwd_packed_col(kk), bwd_packed_col(kk) + 8))


def test_attention_dq_ds_columns_of_their_own():
    # dQ kernel: warp of column quarter q packs dS pair p (keys 32q+2p, +1) at
    # 384 + 16q + p; the dQ MMA reads key chunk kk at [384 + 8kk, +8), outside
    # the S / dP / dQ columns [0, 384).
    location = {32 * q + 2 * p: 384 + 16 * q + p for q in range(4) for p in range(16)}
    for kk in range(8):
        want = [location[16 * kk + 2 * j] for j in range(8)]
        assert want == list(range(384 + 8 * kk, 384 + 8 * kk + 8))
    assert min(location.values()) >= 384 and max(location.values()) < 448


def _gatherer_finishes(world, blocks, ctas, pieces, lag=24, publish_before_peer_wait=True):
    """Every rank's gatherer CTAs run their jobs (own blocks first, then peer
    blocks in rank+1.. order, job j on CTA j % ctas).  An own block becomes
    visible to peers once `lag` later pieces were stored by its CTA, when the
    CTA finishes, or -- with the fix -- before the CTA's first wait on a peer.
    Returns False if every unfinished CTA waits for a block nobody can publish."""
    total = blocks + (world - 1) * blocks
    published = set()           # (rank, block)
    state = {}
    for r in range(world):
        for c in range(ctas):
            jobs = list(range(c, total, ctas))
            state[(r, c)] = dict(jobs=jobs, i=0, stored=0, pending=[], flushed=False)

    def retire(r, st, everything=False):
        keep = []
        for blk, last in st["pending"]:
            if everything or last + lag < st["stored"]:
                published.add((r, blk))
            else:
                keep.append((blk, last))
        st["pending"] = keep

    while True:
        progress, left = False, False
        for (r, c), st in state.items():
            while st["i"] < len(st["jobs"]):
                j = st["jobs"][st["i"]]
                if j < blocks:
                    st["stored"] += pieces
                    st["pending"].append((j, st["stored"] - 1))
                    retire(r, st)
                else:
                    if publish_before_peer_wait and not st["flushed"]:
                        retire(r, st, everything=True)
                        st["flushed"] = True
                    step, b = 1 + (j - blocks) // blocks, (j - blocks) % blocks
                    if ((r + step) % world, b) not in published:
                        break
                    for _ in range(pieces):  # the stream retires after every store
                        st["stored"] += 1
                        retire(r, st)
                st["i"] += 1
                progress = True
            if st["i"] == len(st["jobs"]):
                if st["pending"]:
                    retire(r, st, everything=True)
                    progress = True
            else:
                left = True
        if not left:
            return True
        if not progress:
            return False


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("blocks", [1, 2, 8, 32])
@pytest.mark.parametrize("ctas", [3, 16, 20, 32])
@pytest.mark.parametrize("pieces", [4, 64])
def test_gatherer_schedule_always_finishes(world, blocks, ctas, pieces):
    assert _gatherer_finishes(world, blocks, ctas, pieces)


def test_lagged_own_block_publication_deadlocks_at_the_bench_shape():
    # M=8192 at TP8: eight 128-row blocks per rank, 20 communication CTAs,
    # K=4096 (64 pieces of 16 KB per block): the schedule without the fix.
    assert not _gatherer_finishes(8, 8, 20, 64, publish_before_peer_wait=False)
    assert not _gatherer_finishes(4, 16, 20, 64, publish_before_peer_wait=False)
    assert _gatherer_finishes(2, 32, 20, 64, publish_before_peer_wait=False)


def _simulate_arrival(tiles, chunk_tiles, ctas, ready_order, rng, window=128):
    """One epoch of the windowed claim protocol of rs_reduce_kernel (arrival
    arm); returns {tile: claiming CTA}.  Each CTA keeps a low-water mark (all
    earlier positions of its lane claimed), scans `window` positions from it
    and claims the first ready unclaimed tile of its lane found from its own
    offset in the window, cyclically."""
    claims = {}
    ready = set()
    pending = list(ready_order)
    lwm = [0] * ctas
    offsets = [((c >> 1) * 37) % window for c in range(ctas)]
    lane_of = lambda i: (i // chunk_tiles) % 2
    active = set(range(ctas))
    steps = 0
    while active:
        steps += 1
        assert steps < 100000, "claim loop does not terminate"
        if pending and rng.random() < 0.5:
            ready.add(pending.pop(0))
        c = rng.choice(sorted(active))  # any CTA may run next
        lane = c & 1
        while lwm[c] < tiles and (lane_of(lwm[c]) != lane or lwm[c] in claims):
            lwm[c] += 1
        if lwm[c] >= tiles:
            active.discard(c)  # lane drained: the CTA exits
            continue
        span = min(window, tiles - lwm[c])
        off = offsets[c] % span
        cands = [((w - off) % span, lwm[c] + w) for w in range(span)
                 if lane_of(lwm[c] + w) == lane and lwm[c] + w not in claims and lwm[c] + w in ready]
        if not cands:
            continue  # nothing ready: back off and rescan
        pos = min(cands)[1]
        if pos not in claims:  # the CAS
            claims[pos] = c
    return claims


@pytest.mark.parametrize("tiles,chunk_tiles,ctas", [(32, 2, 8), (64, 4, 20), (48, 1, 96), (16, 2, 2), (512, 2, 40)])
def test_arrival_claims_every_tile_once_and_terminates(tiles, chunk_tiles, ctas):
    rng = random.Random(tiles * 131 + ctas)
    for trial in range(5):
        order = list(range(tiles))
        rng.shuffle(order)
        claims = _simulate_arrival(tiles, chunk_tiles, ctas, order, rng)
        assert sorted(claims) == list(range(tiles))
        for tile, cta in claims.items():
            assert (tile // chunk_tiles) % 2 == cta & 1  # claimed by a CTA of its lane


def _pull_rs_reuse_is_safe(world, calls, rng):
    """Pull GemmRS across calls with ranks at arbitrary relative speeds.  Each
    rank's call t runs as one launch: its GEMM writes partial buffer t % 2 and
    publishes the flag (epoch t) to every owner; its reducer waits for every
    source's epoch-t flag and reads that source's buffer t % 2.  A rank's call
    t+1 starts only after its call t ended (stream order).  Returns False if a
    reader ever finds a buffer already overwritten by a later call."""
    buf = [[0, 0] for _ in range(world)]          # call id held by each rank's two buffers
    flags = [0] * world                           # latest epoch each rank published
    # per rank: (call, stage) with stage 0 = GEMM pending, 1.. = reading source stage-1
    state = [[1, 0] for _ in range(world)]
    done = 0
    while done < world:
        r = rng.randrange(world)
        call, stage = state[r]
        if call > calls:
            continue
        if stage == 0:
            buf[r][call % 2] = call
            flags[r] = call
            state[r][1] = 1
            continue
        s = stage - 1
        if flags[s] < call:
            # wait: is anyone able to move?  (no deadlock: every rank's flags only rise)
            if all(state[q][0] > calls or (state[q][1] >= 1 and flags[state[q][1] - 1] < state[q][0])
                   for q in range(world)):
                return False  # everyone waits
            continue
        if buf[s][call % 2] != call:
            return False      # the source already overwrote the data of this call
        if s == world - 1:
            state[r] = [call + 1, 0]
            if call + 1 > calls:
                done += 1
        else:
            state[r][1] = stage + 1
    return True


@pytest.mark.parametrize("world", [2, 4, 8])
def test_pull_rs_parity_buffers_are_never_overwritten_while_read(world):
    rng = random.Random(world)
    for _ in range(200):
        assert _pull_rs_reuse_is_safe(world, 6, rng)
