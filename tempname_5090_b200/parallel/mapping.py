"""Physical-block schedules and GEMM tile orders of the four GemmRS arms.

Semantics follow TempName-5090 (python/flux_5090/mapping.py:1-55,
src/gemm/native.cu:33-82):

* The M rows of a row-parallel projection are cut into physical blocks of
  `chunk_rows`; block p belongs to destination p // per (per = M/W/chunk_rows),
  `within` = p % per and its transport lane is within % 2.
* Slot order: `flux` / `flux_taco` emit blocks 0..B-1 (destination-major);
  `flux_taco_interleaved` rotates destinations, slot s -> (s % W)*per + s // W;
  `flux_taco_interleaved_arrival` takes a calibrated plan that keeps slot s's
  destination equal to s % W.
* Tile order: destination-major visits each slot's block row-tile by row-tile,
  all column tiles per row-tile; the interleaved arms visit rounds of W slots
  and rotate the destination at column-tile granularity.

`tile_order(..., tile_n)` expresses the order in tiles of 128 rows x tile_n
columns.  At tile_n=128 it is exactly the reference's CTA map; the sm_100a
GEMM uses tile_n=256 tiles with the same traversal.
"""
from __future__ import annotations

ARMS = ("flux", "flux_taco", "flux_taco_interleaved", "flux_taco_interleaved_arrival")
ARRIVAL_ARMS = ARMS[3:]
INTERLEAVED_ARMS = ARMS[2:]
QUANTIZED_ARMS = ARMS[1:]
BACKEND = "b200-tcgen05-nvlink-push-v1"
TILE_M = 128


def validate_shape(m, n, k, world, chunk_rows):
    if any(type(x) is not int or x <= 0 for x in (m, n, k, world, chunk_rows)):
        raise ValueError("positive integer dimensions required")
    if world < 2 or m % (world * chunk_rows) or chunk_rows % 128 or n % 128 or k % 8:
        raise ValueError("require world >= 2, M divisible by world*chunk_rows, "
                         "chunk_rows and N by 128, K by 8")


def blocks_per_destination(m, world, chunk_rows):
    return m // world // chunk_rows


def slot_order(m, n, k, world, chunk_rows, arm, plan=None):
    """Physical block emitted at each slot."""
    validate_shape(m, n, k, world, chunk_rows)
    if arm not in ARMS:
        raise ValueError(f"unknown arm: {arm}")
    count = m // chunk_rows
    per = count // world
    if arm in ARRIVAL_ARMS:
        from .planning import validate_role_plan
        validate_role_plan(plan, m, n, k, world, chunk_rows)
        return list(plan["arrival_order"])
    if plan is not None:
        raise ValueError("only the arrival arm accepts a role plan")
    if arm == "flux_taco_interleaved":
        return [(s % world) * per + s // world for s in range(count)]
    return list(range(count))


def schedule(m, n, k, world, chunk_rows, arm, plan=None):
    per = blocks_per_destination(m, world, chunk_rows)
    order = slot_order(m, n, k, world, chunk_rows, arm, plan)
    result = []
    for slot, physical in enumerate(order):
        within = physical % per
        result.append(dict(slot=slot, physical=physical, destination=physical // per,
                           within=within, row=physical * chunk_rows, rows=chunk_rows,
                           lane=within % 2))
    return result


def tile_order(m, n, k, world, chunk_rows, arm, plan=None, tile_n=128):
    """(row_tile, col_tile) pairs in production order, tiles of 128 x tile_n."""
    if n % tile_n and tile_n != 128:
        raise ValueError("N must be a multiple of the tile width")
    items = schedule(m, n, k, world, chunk_rows, arm, plan)
    row_tiles = chunk_rows // TILE_M
    col_tiles = n // tile_n
    if arm in INTERLEAVED_ARMS:
        out = []
        for round_ in range(len(items) // world):
            for r in range(row_tiles):
                for c in range(col_tiles):
                    for d in range(world):
                        out.append((items[round_ * world + d]["physical"] * row_tiles + r, c))
        return out
    return [(it["physical"] * row_tiles + r, c) for it in items
            for r in range(row_tiles) for c in range(col_tiles)]


def cta_mapping(m, n, k, world, chunk_rows, arm, plan=None):
    """The reference's 128x128 CTA map (mapping.py:34-41)."""
    return tile_order(m, n, k, world, chunk_rows, arm, plan, tile_n=128)


def linear_tile_ids(m, n, k, world, chunk_rows, arm, plan=None, tile_n=256, shift=0):
    """Tile order as linear ids tm * tiles_n + tn (the GEMM kernel's table).

    `shift` rotates destinations: a tile of destination d is replaced by the tile
    at the same position inside destination (d + shift) % W.  The arm's slot
    structure is kept; with shift = rank + 1 the ranks of an in-kernel push start
    on different destinations (and end on their own rows) instead of all pushing
    into the same GPU at once.  Results do not depend on the order: the owner
    reduces sources in index order."""
    cols = n // tile_n
    per_dest = m // world // TILE_M
    out = []
    for tm, tn in tile_order(m, n, k, world, chunk_rows, arm, plan, tile_n):
        if shift:
            tm = ((tm // per_dest + shift) % world) * per_dest + tm % per_dest
        out.append(tm * cols + tn)
    return out


def destination_tile_ids(m, n, k, world, chunk_rows, arm, plan=None, tile_n=256):
    """Per destination, its tiles (global linear ids) in the arm's production order."""
    cols = n // tile_n
    per_dest = m // world // TILE_M
    lists = [[] for _ in range(world)]
    for tm, tn in tile_order(m, n, k, world, chunk_rows, arm, plan, tile_n):
        lists[tm // per_dest].append(tm * cols + tn)
    return lists


def pull_production_ids(m, n, k, world, chunk_rows, arm, rank, plan=None, tile_n=256, tile_m=TILE_M):
    """Production order of the pull transport on `rank`: the arm's
    per-destination tile sequences interleaved across destinations one tile at
    a time, starting with destination rank+1 and ending each round with the
    rank's own rows.  A pulled tile can be reduced only when every source has
    produced it, so every source advances through every destination's tiles at
    the same pace (balanced all-to-all traffic, reduction overlapping the GEMM);
    the within-destination order is the arm's.  With CTA-pair tiles
    (tile_m = 256) ids count 256-row tiles; the BF16 arm's destination-major
    order is row-major inside each destination."""
    if tile_m == TILE_M:
        lists = destination_tile_ids(m, n, k, world, chunk_rows, arm, plan, tile_n)
    else:
        if arm != "flux":
            raise ValueError("CTA-pair tiles serve the BF16 arm's pull transport")
        per_dest, cols = m // world // tile_m, n // tile_n
        lists = [[(d * per_dest + i) * cols + j for i in range(per_dest) for j in range(cols)]
                 for d in range(world)]
    out = []
    for i in range(len(lists[0])):
        for j in range(world):
            out.append(lists[(rank + 1 + j) % world][i])
    return out


def pull_consumer_ids(m, n, k, world, chunk_rows, arm, rank, plan=None, tile_n=256, tile_m=TILE_M):
    """Flag tiles (128 rows x tile_n of `rank`'s rows, local ids) in the order
    `rank`'s tiles are produced: each producer tile covers tile_m / 128 of them."""
    if tile_m == TILE_M:
        return consumer_tile_order(m, n, k, world, chunk_rows, arm, rank, plan, tile_n)
    rows, cols = m // world, n // tile_n
    halves = tile_m // TILE_M
    out = []
    for tid in destination_tile_ids_pairs(m, n, world, rank, tile_n, tile_m):
        tm, tn = tid // cols, tid % cols
        for h in range(halves):
            out.append(((tm * tile_m - rank * rows) // TILE_M + h) * cols + tn)
    return out


def destination_tile_ids_pairs(m, n, world, dest, tile_n, tile_m):
    """Row-major tiles (global ids in tile_m x tile_n units) of one destination."""
    per_dest, cols = m // world // tile_m, n // tile_n
    return [(dest * per_dest + i) * cols + j for i in range(per_dest) for j in range(cols)]


def consumer_tile_order(m, n, k, world, chunk_rows, arm, rank, plan=None, tile_n=256):
    """Order in which `rank` consumes its own tiles: production order restricted
    to tiles destined to `rank`, as local tile ids (row tile within the
    destination) * tiles_n + col tile."""
    rows_per_dest = m // world
    tiles_per_dest_m = rows_per_dest // TILE_M
    cols = n // tile_n
    out = []
    for tm, tn in tile_order(m, n, k, world, chunk_rows, arm, plan, tile_n):
        if tm // tiles_per_dest_m == rank:
            out.append((tm - rank * tiles_per_dest_m) * cols + tn)
    return out


class PushLanes:
    """Lane layout of the push transport on each owner (the host statement of
    `csrc/common/push_lanes.h`).  Block b of a destination (chunk_rows rows)
    travels on lane b % 2, as the reference's per-block exchange alternates
    between two lane communicators (python/flux_5090/runtime.py:50-56).  Every
    lane has its own receive region [source][lane block] and flag array
    [source][lane tile]; both lanes are sized for ceil(blocks / 2) blocks."""

    def __init__(self, rows_per_dest: int, n: int, chunk_rows: int, world: int, tile_n: int = 256):
        if chunk_rows % TILE_M or rows_per_dest % chunk_rows or n % tile_n:
            raise ValueError("push lanes need 128 | chunk_rows, chunk_rows | rows, tile_n | N")
        self.rows, self.n, self.chunk_rows, self.world, self.tile_n = rows_per_dest, n, chunk_rows, world, tile_n
        self.blocks = rows_per_dest // chunk_rows
        self.lane_blocks = (self.blocks + 1) // 2
        self.tiles_n = n // tile_n
        self.lane_tiles = self.lane_blocks * (chunk_rows // TILE_M) * self.tiles_n
        self.lane_slot_bytes = self.lane_blocks * chunk_rows * n * 2
        self.recv_bytes = 2 * world * self.lane_slot_bytes
        self.flag_words = 2 * world * self.lane_tiles

    def lane_of(self, row_local: int) -> int:
        return (row_local // self.chunk_rows) % 2

    def lane_row(self, row_local: int) -> int:
        return (row_local // self.chunk_rows // 2) * self.chunk_rows + row_local % self.chunk_rows

    def slot_offset(self, lane: int, source: int) -> int:
        """Byte offset of `source`'s region of `lane` in a receive buffer."""
        return (lane * self.world + source) * self.lane_slot_bytes

    def flag_index(self, source: int, local_tile: int) -> int:
        """Word of `source`'s flag for local tile (row tile * tiles_n + column tile)."""
        row_local, tn = (local_tile // self.tiles_n) * TILE_M, local_tile % self.tiles_n
        lane = self.lane_of(row_local)
        return (lane * self.world + source) * self.lane_tiles + (self.lane_row(row_local) // TILE_M) * self.tiles_n + tn

    def flag_indices(self) -> list:
        """Every flag word a complete exchange sets (sources x local tiles)."""
        tiles = (self.rows // TILE_M) * self.tiles_n
        return [self.flag_index(s, t) for s in range(self.world) for t in range(tiles)]


def wire_bytes(m, n, world, quantized):
    """Bytes each source sends to remote owners per projection."""
    elements = (world - 1) * (m // world) * n
    return elements // 128 * 136 if quantized else elements * 2


def split_sizes(world, rank, destination, elements):
    """Sparse all-to-all splits of one block (only the owner receives)."""
    if not 0 <= rank < world or not 0 <= destination < world or elements <= 0:
        raise ValueError("invalid collective dimensions")
    sends, receives = [0] * world, [0] * world
    if rank != destination:
        sends[destination] = elements
    else:
        receives = [elements if source != rank else 0 for source in range(world)]
    return sends, receives
