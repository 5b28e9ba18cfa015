"""Fused row-parallel GEMM -> reduce-scatter ("GemmRS"), the four arms.

    out[M/W, N] (rank r) = sum_s  A_s[M, K] @ B_s[N, K]^T  restricted to rows of r

Transport `nvlink` (default): ONE persistent tcgen05 GEMM launch whose
epilogue pushes every finished 128x256 tile straight into its owner's receive
region over NVLink (BF16, or a TACO H128/E4M3 packet for remote tiles in the
quantized arms) and release-stores a per-(source, tile) epoch flag on the
owner.  Each owner has two lanes (block-within-destination parity, as the
reference's two lane communicators), each with its own receive region and
flag array (`mapping.PushLanes`, csrc/common/push_lanes.h).  Then the owner's
receiver kernel waits (bounded) on each tile's W flags
and reduces in source order 0..W-1 with BF16 rounding after every source,
fusing the TACO decode and an optional residual + bias epilogue.
Arms A/B produce tiles destination-major, C/D interleave destinations at
column-tile granularity (D in a calibrated arrival order); the arrival arm's
receiver consumes whichever tile of its lane is fully ready first.  All arms
share the arithmetic order, so the three TACO arms are bitwise equal.

Transport `nccl` keeps the reference mechanism (TempName-5090
python/flux_5090/runtime.py:161-241) as the baseline: the same GEMM writes the
full partial, each physical block is exchanged with a sparse all_to_all on one
of two lane communicators, and the owner runs the ordered (decode+)reduce.

The BF16 arm on NVLink uses the pull transport (`pull=True`, the default
there): ONE launch whose GEMM CTAs TMA-store every partial tile into this
rank's own partial buffer and release-store the tile's flag on its owner,
while `comm_ctas` reducer CTAs of the same launch wait for their own tiles'
flags, pull the tiles from every source with bulk loads (no multicast) and
reduce them in source order into the output, fusing residual + bias.  Sources
produce destinations interleaved one tile at a time (rank+1 first), so every
destination's tiles complete on all sources at the same pace and the
reduction overlaps the GEMM.  The quantized arms keep the push transport
(epilogue-encoded packets pushed into the owner's slots, separate receiver).

Receive slots (push) and partial buffers (pull) are double-buffered by call
parity.  Safety of reuse: rank s overwrites a parity buffer at call t+2 only
after its call t+1 finished; that call waited for every peer r's call t+1
tiles, which r produced after its own call t (stream order), so no peer still
reads (pull) or is yet to read (push) call t's data when it is overwritten.
"""
from __future__ import annotations

import contextlib
import os
import threading

import torch
import torch.distributed as dist

from .._native import count_launch, lib, register_operator, status_tensor
from . import mapping
from .symmetric import SymmetricBuffer
from ..utils import tracing

TILE_N = 256
DEFAULT_TIMEOUT_NS = 10_000_000_000
# Reducer CTAs of the pull transport (the rest of the SMs run the GEMM): chosen
# per shape by parallel/tuning.py unless TN5B_COMM_CTAS fixes a count.
DEFAULT_COMM_CTAS = int(os.environ.get("TN5B_COMM_CTAS", "0"))


class _Lanes:
    """Two extra NCCL communicators + streams for the NCCL transport (per group)."""
    _cache: dict = {}

    @classmethod
    def get(cls, group):
        key = id(group)
        if key not in cls._cache:
            ranks = dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))
            # Same backend as the parent group (NCCL on GPUs; Gloo for CPU ranks in tests).
            backend = dist.get_backend(group)
            lanes = tuple(dist.new_group(ranks=ranks, backend=backend) for _ in range(2))
            streams = tuple(torch.cuda.Stream() for _ in range(2)) if backend == "nccl" else (None, None)
            cls._cache[key] = (lanes, streams)
        return cls._cache[key]


class RSWorkspace:
    """Exchange buffers shared by every GemmRS operator of one (M, N) on one
    group: the tile flags and the epoch sequence, plus (allocated on first use)
    the push transport's receive regions (2 parities x 2 lanes x W sources,
    `mapping.PushLanes`) and the pull transport's partial buffers (2 parities x
    [M, N]).  Any number of operators may share it: each call is a full
    exchange, so the parity chain argument holds across operators.  The flag
    array serves both transports: the pull transport's [source][flag tile] and
    the push transport's [lane][source][lane tile] views."""

    def __init__(self, m: int, n: int, world: int, group=None, *, recv=None, flags=None, partial=None,
                 device=None, chunk_rows: int = 128):
        self.m, self.n, self.world, self.group = m, n, world, group
        self.rows = m // world
        self.chunk_rows = chunk_rows
        self.lanes = mapping.PushLanes(self.rows, n, chunk_rows, world, TILE_N)
        self.slot_bytes = self.lanes.lane_slot_bytes
        self.tiles_per_dest = (self.rows // 128) * (n // TILE_N)
        self.flag_words = max(world * self.tiles_per_dest, self.lanes.flag_words)
        if flags is None:
            flags = SymmetricBuffer(self.flag_words * 4, group)
        self.recv, self.flags, self.partial = recv, flags, partial
        # A failed exchange leaves slots and flags of an unfinished epoch: every
        # operator sharing this workspace refuses further calls.  The lock keeps
        # each call's epoch, push and reduce together when threads share operators.
        self.failed = False
        self.lock = threading.Lock()
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        self.claims = torch.zeros(self.tiles_per_dest, dtype=torch.int32, device=device)
        self.epoch = 0
        register_operator(self)

    def slots(self):
        """Receive slots of the push transport (allocated on first use, collectively)."""
        if self.recv is None:
            self.recv = [SymmetricBuffer(self.lanes.recv_bytes, self.group) for _ in range(2)]
        return self.recv

    def partials(self):
        """Partial buffers of the pull transport (allocated on first use, collectively)."""
        if self.partial is None:
            self.partial = [SymmetricBuffer(self.m * self.n * 2, self.group) for _ in range(2)]
        return self.partial

    def close(self):
        for b in (self.recv or []) + (self.partial or []):
            if isinstance(b, SymmetricBuffer) and b._owned:
                b.close()
        if isinstance(self.flags, SymmetricBuffer) and self.flags._owned:
            self.flags.close()


class GemmRS:
    def __init__(self, m: int, n: int, k: int, group=None, arm: str = "flux", chunk_rows: int = 128,
                 plan=None, transport: str = "nvlink", timeout_ns: int = DEFAULT_TIMEOUT_NS,
                 b_mn: bool = False, workspace: RSWorkspace | None = None,
                 _emulate: tuple | None = None, device: torch.device | None = None,
                 pull: bool | None = None, comm_ctas: int | None = None, tile_kind: int | None = None):
        if arm not in mapping.ARMS:
            raise ValueError(f"unknown arm {arm}")
        if transport not in ("nvlink", "nccl"):
            raise ValueError("transport must be 'nvlink' or 'nccl'")
        if _emulate is not None:
            self.rank, self.world = _emulate[0], _emulate[1]
        else:
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        mapping.validate_shape(m, n, k, self.world, chunk_rows)
        if n % TILE_N:
            raise ValueError("N must be a multiple of 256 for the fused GemmRS")
        self.m, self.n, self.k, self.chunk_rows = m, n, k, chunk_rows
        self.group, self.arm, self.transport, self.b_mn = group, arm, transport, b_mn
        self.plan = plan
        self.quantized = arm in mapping.QUANTIZED_ARMS
        self.arrival = arm in mapping.ARRIVAL_ARMS
        self.rows = m // self.world
        self.timeout_ns = int(timeout_ns)
        # Pull transport: the BF16 arm on NVLink (the quantized arms push packets).
        self.pull = (transport == "nvlink" and not self.quantized) if pull is None else bool(pull)
        if self.pull and (transport != "nvlink" or self.quantized):
            raise ValueError("the pull transport serves the BF16 arm on NVLink")
        if comm_ctas is None:
            from .tuning import gemm_rs_comm_ctas
            comm_ctas = DEFAULT_COMM_CTAS if DEFAULT_COMM_CTAS else gemm_rs_comm_ctas(m, n, k, self.world)
        self.comm_ctas = int(comm_ctas)
        if self.pull and not 1 <= self.comm_ctas <= 64:
            raise ValueError("comm_ctas must be in [1, 64]")
        self._last_operands = None
        self._scatter_order = None
        # `device` defaults to the current CUDA device; CPU is for host-logic tests
        # (NCCL transport on Gloo ranks, or a recording stand-in for the kernels).
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        # GEMM tile kind of the pull transport: 0 single CTA 128 x 256, 2 wide CTA
        # pair 256 x 512 (flags stay per 128-row slice of a tile).
        if not self.pull:
            self.tile_kind = 0
        elif tile_kind is None:
            self.tile_kind = 0 if self.device.type != "cuda" else int(lib().fused_tile_kind(m, n, k, self.comm_ctas))
        else:
            self.tile_kind = int(tile_kind)
        if self.tile_kind not in (0, 2) or (self.tile_kind and (self.rows % 256 or n % 512)):
            raise ValueError(f"tile kind {self.tile_kind} does not fit rows {self.rows} / N {n}")
        self.tile_m = 256 if self.tile_kind else 128
        self.tile_n = 512 if self.tile_kind == 2 else TILE_N
        self.order = mapping.schedule(m, n, k, self.world, chunk_rows, arm, plan)
        ids = self.production_ids(self.rank)
        self.tile_order = torch.tensor(ids, dtype=torch.int32, device=self.device)
        local = mapping.pull_consumer_ids(m, n, k, self.world, chunk_rows, arm, self.rank, plan, self.tile_n,
                                          self.tile_m)
        self.consumer_order = torch.tensor(local, dtype=torch.int32, device=self.device)
        self.tiles_per_dest = (self.rows // 128) * (n // TILE_N)
        self.lanes = mapping.PushLanes(self.rows, n, chunk_rows, self.world, TILE_N)
        self.slot_bytes = self.lanes.lane_slot_bytes
        self._nccl_epoch = 0
        self.calls = 0
        self.failed = False
        self.status = status_tensor(self.device)
        register_operator(self)
        self.workspace = None
        if transport == "nvlink":
            if _emulate is not None:
                # (rank, world, receive slots or partial buffers [2 parities], flags)
                bufs = dict(partial=_emulate[2]) if self.pull else dict(recv=_emulate[2])
                workspace = RSWorkspace(m, n, self.world, flags=_emulate[3], device=self.device,
                                        chunk_rows=chunk_rows, **bufs)
            if workspace is not None and workspace.chunk_rows != chunk_rows:
                raise ValueError("a shared RSWorkspace serves one chunk_rows (its push lanes are cut in blocks)")
            self.workspace = workspace if workspace is not None else RSWorkspace(m, n, self.world, group,
                                                                                 chunk_rows=chunk_rows)
        else:
            self.lanes, self.lane_streams = _Lanes.get(group)
            self.partial = torch.empty((m, n), dtype=torch.bfloat16, device=self.device)
            pbytes = chunk_rows * n // 128 * 136
            self.packet_bytes = pbytes
            # Quantized arms send and receive packets only: no BF16-sized remote storage.
            self.send_packets = torch.empty((m // chunk_rows, pbytes) if self.quantized else (0, pbytes),
                                            dtype=torch.uint8, device=self.device)
            block_bytes = pbytes if self.quantized else chunk_rows * n * 2
            self.recv_blocks = torch.empty((m // chunk_rows // self.world, self.world - 1, block_bytes),
                                           dtype=torch.uint8, device=self.device)

    def production_ids(self, rank: int) -> list:
        """Tile order of `rank`'s producer GEMM.  In-kernel pushes start on
        destination rank+1 (no incast); the NCCL transport keeps the reference
        CTA map."""
        if self.pull:
            return mapping.pull_production_ids(self.m, self.n, self.k, self.world, self.chunk_rows, self.arm,
                                               rank, self.plan, tile_n=self.tile_n, tile_m=self.tile_m)
        shift = rank + 1 if self.transport == "nvlink" else 0
        return mapping.linear_tile_ids(self.m, self.n, self.k, self.world, self.chunk_rows, self.arm, self.plan,
                                       tile_n=TILE_N, shift=shift)

    @property
    def epoch(self) -> int:
        return self.workspace.epoch if self.workspace is not None else self._nccl_epoch

    @epoch.setter
    def epoch(self, value: int) -> None:
        if self.workspace is not None:
            self.workspace.epoch = value
        else:
            self._nccl_epoch = value

    @property
    def flag_tiles(self) -> int:
        """Flag tiles per destination: 128 rows x tile_n columns of its rows."""
        return (self.rows // 128) * (self.n // self.tile_n)

    def published_flags(self) -> torch.Tensor:
        """This rank's flag words that a complete exchange sets, as int32: the
        pull transport's [source][flag tile], or the push transport's two lane
        arrays at `PushLanes.flag_indices` (padding words of a shorter lane excluded)."""
        words = self.flags.local_view((self.workspace.flag_words,), torch.int32)
        if self.pull:
            return words[: self.world * self.flag_tiles]
        idx = torch.tensor(self.lanes.flag_indices(), dtype=torch.long, device=words.device)
        return words[idx]

    def device_tile_map(self) -> list:
        """Mapping probe: the (row tile, column tile) pairs this operator's GEMM
        CTAs decode from the uploaded production table, read back from the
        device (the counterpart of the reference's mapping_probe,
        src/gemm/native.cu:230-236)."""
        mode = 3 if self.pull else (2 if self.quantized else 1)
        got = lib().gemm_tile_map(self.m, self.n, self.k, mode, self.tile_kind, self.tile_order,
                                  self.device.index if self.device.index is not None else 0)
        return [tuple(r) for r in got.cpu().tolist()]

    def host_tile_map(self) -> list:
        """The production order as (row tile, column tile) pairs, from the host spec."""
        cols = self.n // self.tile_n
        return [(t // cols, t % cols) for t in self.production_ids(self.rank)]

    @property
    def recv(self):
        return self.workspace.slots()

    @property
    def flags(self):
        return self.workspace.flags

    @property
    def claims(self):
        return self.workspace.claims

    # ------------------------------------------------------------------ API
    def forward(self, x: torch.Tensor, w: torch.Tensor, *, b_mn: bool | None = None, residual=None,
                bias=None, out=None) -> torch.Tensor:
        """x [M, K] bf16; w [N, K] (or [K, N] when b_mn); returns [M/W, N] bf16."""
        b_mn = self.b_mn if b_mn is None else b_mn
        ws = self.workspace
        if self.failed or (ws is not None and ws.failed):
            raise RuntimeError("this GemmRS operator (or one sharing its receive workspace) previously failed")
        self._check_operands(x, w, b_mn, residual, bias, out)
        out = torch.empty((self.rows, self.n), dtype=torch.bfloat16, device=self.device) if out is None else out
        with (ws.lock if ws is not None else contextlib.nullcontext()):
            if self.epoch + 2 >= 2 ** 31:
                raise RuntimeError("epoch exhausted; create a new operator")
            self.epoch += 1
            try:
                if self.pull:
                    with tracing.scope("gemm_rs.pull"):
                        self._launch_pull(x, w, b_mn, out, residual, bias, phase=6)
                elif self.transport == "nvlink":
                    with tracing.scope("gemm_rs.push"):
                        self.push(x, w, b_mn)
                    with tracing.scope("gemm_rs.reduce"):
                        self.reduce(out, residual, bias)
                else:
                    with tracing.scope("gemm_rs.nccl"):
                        self._forward_nccl(x, w, b_mn, residual, bias, out)
            except BaseException:
                self.failed = True
                if ws is not None:
                    ws.failed = True
                raise
            self.calls += 1
        return out

    def scatter(self, x: torch.Tensor, out=None, phase: int = 3) -> torch.Tensor:
        """Reduce-scatter of an existing [M, N] BF16 tensor over the pull
        transport (no GEMM): the tensor is packed into this rank's partial
        buffer, its tiles are released to their owners, and a launch of the
        reducer CTAs alone pulls and sums every source's rows of this rank in
        source order (BF16 after every source).  Used for the vocab-parallel
        embedding's SumScatter (TempName-5090 python/flux_5090/model.py:100-108).
        phase 3: the whole call; single-GPU emulation of several ranks runs
        phase 1 (pack + publish, opens the epoch) on every rank, then phase 2."""
        if not self.pull:
            raise RuntimeError("scatter needs the pull transport")
        if x.dtype != torch.bfloat16 or tuple(x.shape) != (self.m, self.n) or x.stride(-1) != 1 \
                or x.device != self.device:
            raise ValueError(f"x must be a bf16 [{self.m}, {self.n}] tensor on {self.device}")
        ws = self.workspace
        if self.failed or ws.failed:
            raise RuntimeError("this GemmRS operator (or one sharing its receive workspace) previously failed")
        out = torch.empty((self.rows, self.n), dtype=torch.bfloat16, device=self.device) if out is None else out
        per_dest = (self.rows // 128) * (self.n // TILE_N)
        if self._scatter_order is None:
            self._scatter_order = torch.arange(per_dest, dtype=torch.int32, device=self.device)
        if phase not in (1, 2, 3):
            raise ValueError("phase is 3 (one call) or 1 then 2 (emulation)")
        with ws.lock:
            if phase & 1:
                if self.epoch + 2 >= 2 ** 31:
                    raise RuntimeError("epoch exhausted; create a new operator")
                self.epoch += 1
            try:
                part = ws.partials()[self.epoch & 1]
                dev = self.device.index if self.device.index is not None else 0
                with tracing.scope("gemm_rs.scatter"):
                    if phase & 1:
                        lib().pack_pieces(x, part.local)
                        lib().publish_tiles(self.flags.ptrs.data_ptr(), self.rank, self.world, per_dest,
                                            self.epoch, dev)
                        count_launch(2)
                    if phase & 2:
                        lib().rs_pull_reduce_only(part.local, part.ptrs.data_ptr(), self.flags.ptrs.data_ptr(),
                                                  self.flags.local, self.m, self.n, self.rank, self.world,
                                                  self.epoch, self._scatter_order, out, self.status,
                                                  self.timeout_ns, self.comm_ctas)
                        count_launch()
            except BaseException:
                self.failed = ws.failed = True
                raise
            if phase & 2:
                self.calls += 1
        return out

    def _check_operands(self, x, w, b_mn, residual=None, bias=None, out=None):
        """Operands must match the shape this operator's tile table, slots and flags
        were built for: a mismatch would address tiles outside them."""
        def need(t, shape, name):
            if t.dtype != torch.bfloat16 or tuple(t.shape) != shape or t.stride(-1) != 1 \
                    or t.device != self.device:
                raise ValueError(f"{name} must be a bf16 tensor of shape {list(shape)} with unit inner "
                                 f"stride on {self.device} (got {t.dtype} {list(t.shape)} on {t.device})")
        need(x, (self.m, self.k), "x")
        need(w, (self.k, self.n) if b_mn else (self.n, self.k), "w")
        if residual is not None:
            need(residual, (self.rows, self.n), "residual")
        if bias is not None:
            need(bias, (self.n,), "bias")
        if out is not None:
            need(out, (self.rows, self.n), "out")

    def _launch_pull(self, x, w, b_mn, out, residual=None, bias=None, phase=6, stamps=None, produced=None,
                     delay_tile=-1, delay_ns=0, cta_stamps=None):
        """Pull transport: one launch running the GEMM (phase bit2) and/or the
        reducer CTAs (phase bit1) of this call's epoch."""
        parity = self.epoch & 1
        part = self.workspace.partials()[parity]
        lib().gemm_rs_pull(x, False, w, b_mn, part.local, part.ptrs.data_ptr(), self.flags.ptrs.data_ptr(),
                           self.flags.local, self.rank, self.world, self.epoch, self.tile_order,
                           self.consumer_order, out, residual, bias, self.status, self.timeout_ns,
                           self.comm_ctas, phase, stamps, produced, delay_tile, delay_ns, 0, cta_stamps,
                           self.tile_kind)
        count_launch()

    def push(self, x, w, b_mn: bool | None = None, delay_tile: int = -1, delay_ns: int = 0):
        """Producer phase: the GEMM whose epilogue pushes tiles to their owners
        (pull transport: the GEMM that stores and publishes its partial tiles)."""
        b_mn = self.b_mn if b_mn is None else b_mn
        self._check_operands(x, w, b_mn)
        if self.pull:
            self._last_operands = (x, w, b_mn)
            dummy = torch.empty((self.rows, self.n), dtype=torch.bfloat16, device=self.device)
            self._launch_pull(x, w, b_mn, dummy, phase=4, delay_tile=delay_tile, delay_ns=delay_ns)
            return
        parity = self.epoch & 1
        mode = 2 if self.quantized else 1
        lib().gemm_rs_push(x, False, w, b_mn, mode, self.recv[parity].ptrs.data_ptr(),
                           self.flags.ptrs.data_ptr(), self.rank, self.world, self.chunk_rows,
                           self.epoch, self.slot_bytes, self.tile_order, self.status, self.timeout_ns, 0,
                           delay_tile, delay_ns)
        count_launch()

    def begin(self):
        """Emulation only: start a call (epoch + 1) whose phases are launched separately."""
        self.epoch += 1

    def reduce(self, out, residual=None, bias=None, stamps=None):
        """Receiver phase: bounded waits on tile flags, ordered (decode +) reduce.
        Pull transport: a launch of the reducer CTAs only (operands of the last push)."""
        if self.pull:
            if self._last_operands is None:
                raise RuntimeError("reduce() of the pull transport follows a push() of the same call")
            x, w, b_mn = self._last_operands
            self._launch_pull(x, w, b_mn, out, residual, bias, phase=2, stamps=stamps)
            return
        parity = self.epoch & 1
        count_launch()
        lib().rs_reduce(self.recv[parity].local, self.flags.local, self.slot_bytes, self.rank, self.world,
                        self.rows, self.n, TILE_N, self.chunk_rows, self.quantized, self.epoch, out,
                        residual, bias, self.consumer_order, self.arrival,
                        self.claims if self.arrival else None, self.status, self.timeout_ns, 0, stamps)

    def stage_profile(self, x, w, residual=None, bias=None) -> dict:
        """Untimed diagnostic call of the pull transport with device timestamps
        (%globaltimer, this GPU's clock): when each tile this rank produced was
        published, and when each of this rank's output tiles was reduced.  Reports
        how many output tiles were complete before this rank's GEMM published its
        last tile -- the reduction that overlapped the GEMM (the counterpart of
        the reference's per-block consumer intervals, runtime.py:243-257)."""
        if not self.pull:
            raise RuntimeError("stage_profile needs the pull transport")
        ws = self.workspace
        if self.failed or ws.failed:
            raise RuntimeError("this GemmRS operator (or one sharing its receive workspace) previously failed")
        out = torch.empty((self.rows, self.n), dtype=torch.bfloat16, device=self.device)
        flag_tiles = (self.rows // 128) * (self.n // self.tile_n)
        stamps = torch.zeros(flag_tiles, dtype=torch.int64, device=self.device)
        produced = torch.zeros((self.m // 128) * (self.n // self.tile_n), dtype=torch.int64, device=self.device)
        grid = lib().fused_grid(self.m, self.n, self.k, 3, 0, 256, self.comm_ctas, 6, self.tile_kind)
        ctas = torch.zeros(2 * grid, dtype=torch.int64, device=self.device)
        with ws.lock:
            try:
                self._profiled_call(x, w, out, stamps, 0, 0, produced=produced, cta_stamps=ctas,
                                    residual=residual, bias=bias)
            except BaseException:
                self.failed = ws.failed = True
                raise
        torch.cuda.synchronize()
        p, c, k = produced.cpu(), stamps.cpu(), ctas.cpu().view(grid, 2)
        t0 = int(k[:, 0].min())
        gemm_end = int(p.max())
        comm = k[:self.comm_ctas]
        gemm = k[self.comm_ctas:]
        return dict(out=out, kernel_ns=int(k[:, 1].max()) - t0,
                    gemm_ctas_end_ns=int(gemm[:, 1].max()) - t0, reducer_ctas_end_ns=int(comm[:, 1].max()) - t0,
                    producer_first_ns=int(p.min()) - t0, producer_last_ns=gemm_end - t0,
                    consumer_first_ns=int(c.min()) - t0, consumer_last_ns=int(c.max()) - t0,
                    consumer_tiles=int(c.numel()),
                    consumer_tiles_completed_before_producer_end=int((c < gemm_end).sum()),
                    produced_ns=(p - t0).tolist(), consumed_ns=(c - t0).tolist())

    def profile_call(self, x, w, *, delay_ns: int = 0, delay_rank: int = 0):
        """Untimed diagnostic call: optionally delays (bounded, <= 100 ms) the flag
        publication of the first lane-0 tile that `delay_rank` produces, and
        returns (output, per-local-tile completion times in ns since the first
        completion, the delayed tile's local id on its owner or None)."""
        if self.transport != "nvlink":
            raise RuntimeError("profile_call needs the NVLink transport")
        if not 0 <= delay_ns <= 100_000_000:
            raise ValueError("diagnostic delay must be within 100 ms")
        ws = self.workspace
        if self.failed or ws.failed:
            raise RuntimeError("this GemmRS operator (or one sharing its receive workspace) previously failed")
        out = torch.empty((self.rows, self.n), dtype=torch.bfloat16, device=self.device)
        stamps = torch.zeros((self.rows // 128) * (self.n // self.tile_n), dtype=torch.int64, device=self.device)
        with ws.lock:
            try:
                delayed_local = self._profiled_call(x, w, out, stamps, delay_ns, delay_rank)
            except BaseException:
                self.failed = ws.failed = True
                raise
        torch.cuda.synchronize()
        s = stamps.cpu()
        rel = (s - s.min()).tolist()
        return out, rel, delayed_local

    def _profiled_call(self, x, w, out, stamps, delay_ns, delay_rank, produced=None, cta_stamps=None,
                       residual=None, bias=None):
        self.epoch += 1
        delay_tile, delayed_local = -1, None
        if delay_ns:
            # Every rank identifies the same tile: the first lane-0 tile of
            # `delay_rank`'s own production order (orders differ per rank).
            # Local ids count flag tiles (128 rows x tile_n of the owner's rows).
            tiles_n = self.n // self.tile_n
            per_dest_m = self.rows // self.tile_m
            for tid in self.production_ids(delay_rank):
                tm = tid // tiles_n
                block = (tm * self.tile_m % self.rows) // self.chunk_rows
                if block % 2 == 0:
                    delay_tile = tid
                    dest = tm // per_dest_m
                    first_row = (tm - dest * per_dest_m) * self.tile_m
                    delayed_local = (dest, (first_row // 128) * tiles_n + tid % tiles_n)
                    break
        mine = self.rank == delay_rank
        if self.pull:
            self._launch_pull(x, w, self.b_mn, out, residual, bias, phase=6, stamps=stamps, produced=produced,
                              delay_tile=delay_tile if mine else -1, delay_ns=delay_ns if mine else 0,
                              cta_stamps=cta_stamps)
        else:
            self.push(x, w, delay_tile=delay_tile if mine else -1, delay_ns=delay_ns if mine else 0)
            self.reduce(out, stamps=stamps)
        self.calls += 1
        return delayed_local

    def _forward_nccl(self, x, w, b_mn, residual, bias, out):
        from ..ops import gemm as G, taco
        G.matmul(x, w, b_t=b_mn, out=self.partial, tile_order=None)
        per = self.rows // self.chunk_rows
        elements = self.chunk_rows * self.n
        for item in self.order:
            p, dest, within, lane = item["physical"], item["destination"], item["within"], item["lane"]
            block = self.partial.narrow(0, p * self.chunk_rows, self.chunk_rows)
            local = dest == self.rank
            if self.quantized:
                send = self.send_packets[p] if not local else self.send_packets[p][:0]
                if not local:
                    taco.encode(block, send)
                count = self.packet_bytes
            else:
                send = block.reshape(-1).view(torch.uint8) if not local else block.reshape(-1).view(torch.uint8)[:0]
                count = elements * 2
            recv = self.recv_blocks[within].reshape(-1)[: (self.world - 1) * count] if local else \
                self.recv_blocks[0].reshape(-1)[:0]
            sends, receives = mapping.split_sizes(self.world, self.rank, dest, count)
            dist.all_to_all_single(recv, send, output_split_sizes=receives, input_split_sizes=sends,
                                   group=self.lanes[lane])
            if local:
                target = out.narrow(0, within * self.chunk_rows, self.chunk_rows)
                if self.quantized:
                    taco.decode_reduce(block, recv.view(self.world - 1, count), self.rank, self.world, out=target)
                else:
                    taco.ordered_reduce(block, recv.view(torch.bfloat16), self.rank, self.world, out=target)
        if residual is not None or bias is not None:
            y = out.float()
            if residual is not None:
                y = (residual.float() + y).to(torch.bfloat16).float()
            if bias is not None:
                y = y + bias.float()
            out.copy_(y.to(torch.bfloat16))

    def state(self) -> dict:
        return dict(backend=mapping.BACKEND, transport=self.transport, arm=self.arm, rank=self.rank,
                    world=self.world, calls=self.calls, epoch=self.epoch,
                    shape=[self.m, self.n, self.k], chunk_rows=self.chunk_rows,
                    production_schedule=self.order, tile_n=self.tile_n, tile_m=self.tile_m,
                    pull_transport=self.pull, comm_ctas=self.comm_ctas if self.pull else 0,
                    push_destination_rotation=(self.rank + 1) % self.world if self.transport == "nvlink" else 0,
                    quantization="all_remote_h128_e4m3" if self.quantized else "none",
                    remote_wire_bytes_per_source=mapping.wire_bytes(self.m, self.n, self.world, self.quantized),
                    reduction_order=list(range(self.world)), rounding="bf16_after_each_source",
                    consumer_policy="per_lane_ready" if self.arrival else "ordered",
                    transport_lanes=2, producer_launches_per_call=1,
                    publication="system-release-per-tile-epoch")

    def close(self):
        if self.workspace is not None:
            self.workspace.close()
