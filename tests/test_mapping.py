"""Schedules and tile orders of the four arms against an independent spec."""
import pytest

from tempname_5090_b200.parallel import mapping as mp
from tempname_5090_b200.parallel import planning as pl


def spec_map(m, n, world, chunk_rows, order, interleaved):
    """Independent statement of the reference CTA map (native.py mapping_reference)."""
    tiles_per_macro = (chunk_rows // 128) * (n // 128)
    out = []
    for logical in range((m // 128) * (n // 128)):
        if interleaved:
            within_dest, dest = divmod(logical, world)
            rnd, within = divmod(within_dest, tiles_per_macro)
            slot = rnd * world + dest
        else:
            slot, within = divmod(logical, tiles_per_macro)
        row, col = divmod(within, n // 128)
        out.append((order[slot] * (chunk_rows // 128) + row, col))
    return out


@pytest.mark.parametrize("arm", mp.ARMS)
@pytest.mark.parametrize("m,n,world,chunk", [(2048, 4096, 8, 128), (1024, 512, 2, 256),
                                             (4096, 1024, 4, 128)])
def test_cta_map_matches_spec(arm, m, n, world, chunk):
    plan = pl.make_role(m, n, 64, world, chunk) if arm in mp.ARRIVAL_ARMS else None
    order = mp.slot_order(m, n, 64, world, chunk, arm, plan)
    expect = spec_map(m, n, world, chunk, order, arm in mp.INTERLEAVED_ARMS)
    assert mp.cta_mapping(m, n, 64, world, chunk, arm, plan) == expect


def test_interleave_spacing_and_lanes():
    items = mp.schedule(2048, 4096, 512, 8, 128, "flux_taco_interleaved")
    assert [it["destination"] for it in items[:8]] == list(range(8))
    assert all(it["lane"] == it["within"] % 2 for it in items)
    assert sorted(it["physical"] for it in items) == list(range(16))


def test_wire_bytes_budget():
    assert mp.wire_bytes(2048, 4096, 8, False) == 14680064
    assert mp.wire_bytes(2048, 4096, 8, True) == 7798784


def test_split_sizes_pairwise():
    for world in (2, 4, 8):
        for dest in range(world):
            recv = None
            for rank in range(world):
                sends, receives = mp.split_sizes(world, rank, dest, 10)
                if rank == dest:
                    assert sum(sends) == 0 and receives[rank] == 0
                    assert sum(receives) == 10 * (world - 1)
                else:
                    assert sends[dest] == 10 and sum(receives) == 0


@pytest.mark.parametrize("bad", [(1000, 4096, 64, 8, 128), (2048, 4000, 64, 8, 128),
                                 (2048, 4096, 63, 8, 128), (2048, 4096, 64, 1, 128),
                                 (2048, 4096, 64, 8, 100)])
def test_invalid_shapes(bad):
    with pytest.raises(ValueError):
        mp.validate_shape(*bad)


def test_tile_order_256_is_bijection_and_consumer_order():
    m, n, world, chunk = 8192, 4096, 8, 128
    for arm in mp.ARMS:
        plan = pl.make_role(m, n, 2048, world, chunk) if arm in mp.ARRIVAL_ARMS else None
        ids = mp.linear_tile_ids(m, n, 2048, world, chunk, arm, plan, tile_n=256)
        assert sorted(ids) == list(range((m // 128) * (n // 256)))
        for rank in (0, 7):
            local = mp.consumer_tile_order(m, n, 2048, world, chunk, arm, rank, plan, 256)
            assert sorted(local) == list(range((m // world // 128) * (n // 256)))


def test_plan_only_for_arrival_arm():
    plan = pl.make_role(2048, 4096, 512, 8, 128)
    with pytest.raises(ValueError):
        mp.schedule(2048, 4096, 512, 8, 128, "flux", plan)
    mutated = dict(plan)
    mutated["arrival_order"] = list(reversed(plan["arrival_order"]))
    with pytest.raises(ValueError):
        mp.schedule(2048, 4096, 512, 8, 128, "flux_taco_interleaved_arrival", mutated)


@pytest.mark.parametrize("arm", ["flux", "flux_taco_interleaved"])
def test_rotated_push_order_is_a_permutation_keeping_within_destination_order(arm):
    from tempname_5090_b200.parallel import mapping
    m, n, k, world, chunk = 8192, 4096, 512, 8, 128
    base = mapping.linear_tile_ids(m, n, k, world, chunk, arm, tile_n=256)
    per_dest = m // world // 128
    cols = n // 256
    firsts = set()
    for rank in range(world):
        rot = mapping.linear_tile_ids(m, n, k, world, chunk, arm, tile_n=256, shift=rank + 1)
        assert sorted(rot) == sorted(base)
        # position i keeps its within-destination tile; only the destination rotates
        for a, b in zip(base, rot):
            ta, tb = a // cols, b // cols
            assert ta % per_dest == tb % per_dest and a % cols == b % cols
            assert tb // per_dest == (ta // per_dest + rank + 1) % world
        firsts.add(rot[0] // cols // per_dest)
        if arm == "flux":
            assert rot[-1] // cols // per_dest == rank  # own rows last
    assert len(firsts) == world  # every rank starts on a different destination


@pytest.mark.parametrize("rows,n,chunk,world", [(256, 512, 128, 2), (384, 512, 128, 2), (1024, 4096, 256, 8),
                                                (640, 768, 128, 4), (128, 256, 128, 8)])
def test_push_lanes_layout(rows, n, chunk, world):
    """Block b of a destination travels on lane b % 2; each lane's flag array
    holds its own tiles only, every (source, tile) has its own word, and lane
    rows pack the lane's blocks in block order."""
    lanes = mp.PushLanes(rows, n, chunk, world)
    tiles_n = n // 256
    tiles = (rows // 128) * tiles_n
    idx = lanes.flag_indices()
    assert len(set(idx)) == world * tiles and max(idx) < lanes.flag_words
    for s in range(world):
        for t in range(tiles):
            row = (t // tiles_n) * 128
            lane = (row // chunk) % 2
            word = lanes.flag_index(s, t)
            assert (lane * world + s) * lanes.lane_tiles <= word < (lane * world + s + 1) * lanes.lane_tiles
    seen = {0: [], 1: []}
    for row in range(0, rows, 128):
        seen[lanes.lane_of(row)].append(lanes.lane_row(row))
    for lane in (0, 1):
        assert seen[lane] == list(range(0, 128 * len(seen[lane]), 128))
        assert len(seen[lane]) * 128 * n * 2 <= lanes.lane_slot_bytes
    assert lanes.recv_bytes == 2 * world * lanes.lane_slot_bytes >= world * rows * n * 2


@pytest.mark.parametrize("rows,n,chunk,world", [(256, 512, 128, 2), (384, 512, 128, 2), (1024, 4096, 256, 8),
                                                (640, 768, 128, 4)])
def test_push_lanes_host_statement_matches_kernel_arithmetic(rows, n, chunk, world):
    """The host's PushLanes and the header the kernels compile (push_lanes.h,
    evaluated on the host through the extension) agree word for word."""
    from tempname_5090_b200 import _native
    if not _native.available():
        pytest.skip("native extension not built")
    slot, recv, words, idx = _native.lib().push_lanes_layout(rows, n, chunk, world, 256)
    lanes = mp.PushLanes(rows, n, chunk, world)
    assert (slot, recv, words) == (lanes.lane_slot_bytes, lanes.recv_bytes, lanes.flag_words)
    assert idx.flatten().tolist() == lanes.flag_indices()
