"""Fused sequence-parallel all-gather -> GEMM (column-parallel linears).

    out[M, N] = gather_rows(x_shard)[M, K] @ B[N, K]^T   (+ bias, GeLU, GeLU-backward)

ONE persistent launch per call with two kinds of CTAs:

* `comm_ctas` gatherer CTAs copy this rank's shard into its own chunk of its
  symmetric gather buffer, publishing each 128-row block as soon as it is
  complete (a system-scope release of `published[rank][block] = epoch` on
  every peer), and pull every peer's published blocks (rank+1 first) from the
  peer's gather buffer with bulk loads -- no multicast -- into the local gather
  buffer, flagging each 128-row block with the call's epoch once it is stored;
* the other CTAs run the tcgen05 GEMM: tiles of the own chunk first, read
  straight from the shard, then each peer chunk's tiles once their block count
  flag is set (bounded wait), with TMA loads of LOCAL memory only.

Buffer reuse: peers only read this rank's own chunk; every gatherer CTA of a
peer adds 1 to this rank's `pulled` counter after its last load from it, and
this rank overwrites its own chunk at call t+1 only once the counter shows
that every peer finished reading call t's -- a bounded wait inside the kernel,
so back-to-back calls of one operator are safe without any host barrier.  No
peer ever writes into this rank's buffer, so `gathered` stays valid until this
rank's own next call.

The gather buffer doubles as the saved full input of the layer (the
reference's ColumnLinear saves `gather_rows(x)` for dW, model.py:110-117).
Cumulative counter targets (pieces per block, gatherer CTAs per call) are kept
on the host; every rank issues the same sequence of calls per operator.
"""
from __future__ import annotations

import os
import threading

import torch
import torch.distributed as dist

from .._native import count_launch, lib, register_operator, status_tensor
from ..ops import gemm as G
from .symmetric import SymmetricBuffer
from ..utils import tracing

DEFAULT_TIMEOUT_NS = 10_000_000_000
# Gatherer CTAs: chosen per shape by parallel/tuning.py (needs the GEMM's N,
# given at construction) unless TN5B_AG_COMM_CTAS fixes a count.
DEFAULT_COMM_CTAS = int(os.environ.get("TN5B_AG_COMM_CTAS", "0"))
PIECE_BYTES = 16384
READY_STRIDE = 32         # u32 words between two block counters (one 128-byte line)


def control_layout(m: int) -> tuple:
    """Byte layout of a rank's control block: published[world][M/W/128] u32 block
    flags at 0, the pulled counter at the next 256-byte boundary.
    Returns (pulled offset, total bytes)."""
    flags = (m // 128) * 4
    pulled = (flags + 255) // 256 * 256
    return pulled, pulled + 256


def ag_tile_order(m: int, n: int, world: int, rank: int, bn: int, tile_m: int = 128) -> list:
    """Own chunk first, then rank+1, ... (the order chunks arrive in); inside a
    chunk, column tiles outer so a weight panel is reused by all row tiles of
    the chunk.  Tiles are tile_m x bn (256 x 512 for the wide CTA pair)."""
    rows = m // world
    tm_per = rows // tile_m
    tn = (n + bn - 1) // bn
    out = []
    for step in range(world):
        c = (rank + step) % world
        for j in range(tn):
            for i in range(tm_per):
                out.append((c * tm_per + i) * tn + j)
    return out


class AGGemm:
    def __init__(self, m: int, k: int, group=None, timeout_ns: int = DEFAULT_TIMEOUT_NS,
                 comm_ctas: int | None = None, _emulate: tuple | None = None,
                 device: torch.device | None = None, tile_kind: int | None = None, n: int | None = None):
        if _emulate is not None:
            self.rank, self.world, self.gather, self.ctrl = _emulate
        else:
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world < 2 or self.world > 64:
            raise ValueError("the fused all-gather needs 2..64 ranks")
        if m % self.world or (m // self.world) % 128:
            raise ValueError("rows per rank must be a multiple of 128")
        if k % 8:
            raise ValueError("K must be a multiple of 8")
        self.m, self.k, self.group = m, k, group
        if tile_kind not in (None, 0, 2) or (tile_kind == 2 and (m // self.world) % 256):
            raise ValueError("tile_kind is 0 (single CTA) or 2 (wide CTA pair, rows per rank % 256 == 0)")
        self._kind = tile_kind
        if comm_ctas is None:
            from .tuning import ag_gemm_comm_ctas
            comm_ctas = DEFAULT_COMM_CTAS or (ag_gemm_comm_ctas(m, n, k, self.world) if n else 20)
        self.comm_ctas = int(comm_ctas)
        if not 1 <= self.comm_ctas <= 64:
            raise ValueError("comm_ctas must be in [1, 64]")
        # `device` defaults to the current CUDA device; CPU serves host-logic tests.
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.timeout_ns = int(timeout_ns)
        self.pulled_offset, ctrl_bytes = control_layout(m)
        if _emulate is None:
            self.gather = SymmetricBuffer(m * k * 2, group)
            self.ctrl = SymmetricBuffer(ctrl_bytes, group)
        self.blocks = (m // self.world) // 128
        self.pieces_per_block = -(-(128 * k * 2) // PIECE_BYTES)
        # arrived-piece counter per (source, 128-row block), one 128-byte line each
        self.ready = torch.zeros(self.world * self.blocks * READY_STRIDE, dtype=torch.int32, device=self.device)
        self._published_ptrs = torch.tensor([p for p in self.ctrl.peers], dtype=torch.int64, device=self.device)
        self._pulled_ptrs = torch.tensor([p + self.pulled_offset for p in self.ctrl.peers], dtype=torch.int64,
                                         device=self.device)
        self.calls = 0            # completed epochs
        self.failed = False
        self._lock = threading.Lock()
        self._orders: dict = {}
        self.status = status_tensor(self.device)
        register_operator(self)

    @property
    def gathered(self) -> torch.Tensor:
        """This rank's gathered [M, K] input of the most recent call."""
        return self.gather.local_view((self.m, self.k), torch.bfloat16)

    def input_buffer(self) -> torch.Tensor:
        """This rank's chunk of the gather buffer as a [M/W, K] tensor, ready to
        be written with the NEXT call's shard (e.g. by the kernel producing it):
        a bounded device wait, launched here on the current stream, holds the
        writer back until every peer has finished reading the previous call's
        contents.  Passing this view as `shard` skips the own-chunk copy: its
        blocks are published to the peers as soon as the call starts."""
        rows = self.m // self.world
        if self.device.type == "cuda":
            target = self.targets(self.calls + 1)["pulled_target"]
            lib().wait_probe(self.ctrl.local + self.pulled_offset, target, self.timeout_ns, self.status)
            count_launch()
        return self.gather.local_view((rows, self.k), torch.bfloat16, offset=self.rank * rows * self.k * 2)

    def _order(self, n: int, bn: int, kind: int) -> torch.Tensor:
        key = (n, bn, kind)
        if key not in self._orders:
            tile_n = 2 * bn if kind == 2 else bn
            ids = ag_tile_order(self.m, n, self.world, self.rank, tile_n, 256 if kind else 128)
            self._orders[key] = torch.tensor(ids, dtype=torch.int32, device=self.device)
        return self._orders[key]

    def tile_kind(self, n: int, bn: int) -> int:
        """0 single CTA 128 x bn, 2 wide CTA pair 256 x 512 (wave model, cached)."""
        key = ("kind", n, bn)
        if key not in self._orders:
            kind = 0
            if self._kind is not None:
                kind = self._kind if bn == 256 else 0
            elif bn == 256 and self.device.type == "cuda" and (self.m // self.world) % 256 == 0:
                kind = int(lib().fused_tile_kind(self.m, n, self.k, self.comm_ctas))
            self._orders[key] = kind
        return self._orders[key]

    def targets(self, epoch: int) -> dict:
        """Targets of call `epoch` (1-based): the peers' gatherer CTAs that
        finished reading the previous call's own chunk (cumulative counter),
        and the per-block arrival flag (the epoch)."""
        return dict(pulled_target=(self.world - 1) * self.comm_ctas * (epoch - 1), ready_target=epoch)

    def _check(self, shard, w, b_mn, bias, gelu_aux, gelu_grad_of, out):
        n = w.shape[1] if b_mn else w.shape[0]
        if tuple(shard.shape) != (self.m // self.world, self.k):
            raise ValueError(f"shard must be [{self.m // self.world}, {self.k}]")
        if w.dim() != 2 or (w.shape[0] if b_mn else w.shape[1]) != self.k or w.stride(-1) != 1:
            raise ValueError(f"w must be 2-D with K={self.k} ({'[K, N]' if b_mn else '[N, K]'}) and unit inner stride")
        for t, name in ((shard, "shard"), (w, "w")):
            if t.dtype != torch.bfloat16 or t.device != self.device:
                raise ValueError(f"{name} must be bf16 on {self.device}")
        if bias is not None and (tuple(bias.shape) != (n,) or bias.dtype != torch.bfloat16
                                 or not bias.is_contiguous() or bias.device != self.device):
            raise ValueError(f"bias must be a contiguous bf16 [{n}] on {self.device}")
        for t, name in ((gelu_aux, "gelu_aux"), (gelu_grad_of, "gelu_grad_of"), (out, "out")):
            if t is None:
                continue
            if tuple(t.shape) != (self.m, n) or t.dtype != torch.bfloat16 or t.stride(-1) != 1 \
                    or t.device != self.device:
                raise ValueError(f"{name} must be a bf16 [{self.m}, {n}] with unit inner stride on {self.device}")
        return n

    def forward(self, shard: torch.Tensor, w: torch.Tensor, *, b_mn: bool = False, bias=None,
                gelu_aux=None, gelu_grad_of=None, out=None, bn: int = 0, phase: int = 7,
                _stamps: tuple | None = None) -> torch.Tensor:
        """One call (phase 7).  Single-GPU emulation of several ranks runs each
        call as three launches per rank -- phase 1 (own chunk), 2 (pull peers),
        4 (GEMM) -- over all ranks in turn, so no launch waits on a later one.
        Phase 3 then 4 runs the gather and the GEMM of one call as two launches
        (to time them apart)."""
        if self.failed:
            raise RuntimeError("this AG->GEMM operator previously failed (its counters are out of step)")
        n = self._check(shard, w, b_mn, bias, gelu_aux, gelu_grad_of, out)
        if phase not in (1, 2, 3, 4, 7):
            raise ValueError("phase must be 7 (one launch), 1, 2, 4 (emulation) or 3 then 4 (gather, then GEMM)")
        out = torch.empty((self.m, n), dtype=torch.bfloat16, device=self.device) if out is None else out
        if bn == 0:
            bn = 256 if n >= 256 and (self.m // 128) * ((n + 255) // 256) >= 148 else 128
        epi = 0
        aux = None
        if bias is not None:
            epi |= G.EPI_BIAS
        if gelu_aux is not None:
            epi |= G.EPI_GELU
            aux = gelu_aux
        if gelu_grad_of is not None:
            epi |= G.EPI_GELU_BWD
            aux = gelu_grad_of
        # Counter targets are cumulative over calls: a launch that fails leaves
        # them out of step, so the operator refuses further calls; the lock keeps
        # targets and launch paired when threads share the operator.
        with self._lock:
            epoch = self.calls + 1 if phase & 1 else self.calls
            try:
                t = self.targets(epoch)
                kind = self.tile_kind(n, bn)
                with tracing.scope("ag_gemm"):
                    lib().ag_gemm(shard.contiguous(), self.gathered, w, b_mn, out, epi, bias, aux,
                                  self.gather.ptrs.data_ptr(), self._published_ptrs.data_ptr(),
                                  self._pulled_ptrs.data_ptr(), self.ctrl.local,
                                  self.ctrl.local + self.pulled_offset, self.ready, self.rank, self.world, epoch,
                                  t["pulled_target"], t["ready_target"], self._order(n, bn, kind), self.status,
                                  self.timeout_ns, bn, self.comm_ctas, phase, *(_stamps or (None, None)), kind)
            except BaseException:
                self.failed = True
                raise
            if phase & 1:
                self.calls = epoch
            count_launch()
        return out

    def stage_profile(self, shard, w, **kw) -> dict:
        """Untimed diagnostic call with device timestamps (%globaltimer of this
        GPU): start / end of every gatherer and GEMM CTA, and the time each
        peer block had fully arrived.  Tells whether the GEMM waited for data
        (blocks arriving after the GEMM CTAs became free) or the reverse."""
        n = w.shape[1] if kw.get("b_mn") else w.shape[0]
        bn = kw.get("bn", 0) or (256 if n >= 256 and (self.m // 128) * ((n + 255) // 256) >= 148 else 128)
        grid = lib().fused_grid(self.m, n, self.k, 0, 1, bn, self.comm_ctas, 7, self.tile_kind(n, bn))
        ctas = torch.zeros(2 * grid, dtype=torch.int64, device=self.device)
        blocks = torch.zeros(self.world * self.blocks, dtype=torch.int64, device=self.device)
        out = self.forward(shard, w, _stamps=(ctas, blocks), **kw)
        torch.cuda.synchronize()
        k = ctas.cpu().view(grid, 2)
        b = blocks.cpu().view(self.world, self.blocks)
        t0 = int(k[:, 0].min())
        comm, gemm = k[:self.comm_ctas], k[self.comm_ctas:]
        peers = [c for c in range(self.world) if c != self.rank]
        return dict(out=out, kernel_ns=int(k[:, 1].max()) - t0, gemm_ctas=int(gemm.shape[0]),
                    gather_end_ns=int(comm[:, 1].max()) - t0, gemm_end_ns=int(gemm[:, 1].max()) - t0,
                    gemm_first_end_ns=int(gemm[:, 1].min()) - t0,
                    own_chunk_ready_ns=int(b[self.rank].max()) - t0,
                    peer_chunk_ready_ns={c: int(b[c].max()) - t0 for c in peers},
                    first_peer_block_ns=min(int(b[c].min()) - t0 for c in peers))

    def close(self):
        if isinstance(self.gather, SymmetricBuffer) and self.gather._owned:
            self.gather.close()
            self.ctrl.close()
