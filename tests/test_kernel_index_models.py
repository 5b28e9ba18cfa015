"""CPU models of kernel index arithmetic and protocols (no GPU).

Each test restates one formula or loop of a CUDA kernel and checks the property
the kernel relies on:

* GEMM grouped raster (`tile_coords` in csrc/gemm/gemm_kernel.cuh): a bijection
  from linear tile ids to (tile_m, tile_n) for every tile kind's tile counts.
* Attention packed probabilities (`packed_col` / `softmax_grad_row` in
  csrc/kernels/attention_tc.cu): the MMA's K-chunk kk finds exactly the BF16
  pairs the elementwise warp of its half wrote, and each warp writes only inside
  the 64 score columns it alone reads.
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
