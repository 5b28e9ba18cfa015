"""Fused sequence-parallel all-gather -> GEMM (column-parallel linears).

    out[M, N] = gather_rows(x_shard)[M, K] @ B[N, K]^T   (+ bias, GeLU, GeLU-backward)

ONE persistent tcgen05 launch per call.  An extra warp in every CTA copies
that CTA's slice of the local shard into every rank's symmetric gather buffer
over NVLink (peers first) and bumps the owner's per-source counter with a
system-scope release; the TMA producer of each CTA waits (bounded) until the
row chunk of its next tile has fully arrived in LOCAL memory, then loads it
with TMA -- no TMA load ever reads another GPU's memory.  Tiles of the local
shard come first, then rank+1, rank+2, ... so the math starts immediately.

The gather buffer doubles as the saved full input of the layer (the
reference's ColumnLinear saves `gather_rows(x)` for dW, model.py:110-117).
Counter targets accumulate the sender grid sizes of every call, identical on
all ranks because every rank issues the same sequence of shapes.
Buffer reuse across calls follows the same chain argument as GemmRS: a peer
can overwrite rank r's gather buffer for call t+1 only after r's own call t+1
push, which r issues after every stream-ordered reader of call t.
"""
from __future__ import annotations

import threading

import torch
import torch.distributed as dist

from .._native import count_launch, lib, status_tensor
from ..ops import gemm as G
from .symmetric import SymmetricBuffer
from ..utils import tracing

DEFAULT_TIMEOUT_NS = 10_000_000_000


def ag_tile_order(m: int, n: int, world: int, rank: int, bn: int) -> list:
    """Own chunk first, then rank+1, ...; inside a chunk, column tiles outer so a
    weight panel is reused by all row tiles of the chunk."""
    rows = m // world
    tm_per = rows // 128
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
                 _emulate: tuple | None = None, device: torch.device | None = None):
        if _emulate is not None:
            self.rank, self.world, self.gather, self.flags = _emulate
        else:
            self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if m % self.world or (m // self.world) % 128:
            raise ValueError("rows per rank must be a multiple of 128")
        if k % 8:
            raise ValueError("K must be a multiple of 8")
        self.m, self.k, self.group = m, k, group
        # `device` defaults to the current CUDA device; CPU serves host-logic tests.
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.timeout_ns = int(timeout_ns)
        if _emulate is None:
            self.gather = SymmetricBuffer(m * k * 2, group)
            self.flags = SymmetricBuffer(self.world * 4, group)
        self.flag_total = 0
        self.calls = 0
        self.failed = False
        self._lock = threading.Lock()
        self._orders: dict = {}
        self.status = status_tensor(self.device)

    @property
    def gathered(self) -> torch.Tensor:
        """This rank's gathered [M, K] input of the most recent call."""
        return self.gather.local_view((self.m, self.k), torch.bfloat16)

    def _order(self, n: int, bn: int) -> torch.Tensor:
        key = (n, bn)
        if key not in self._orders:
            ids = ag_tile_order(self.m, n, self.world, self.rank, bn)
            self._orders[key] = torch.tensor(ids, dtype=torch.int32, device=self.device)
        return self._orders[key]

    def forward(self, shard: torch.Tensor, w: torch.Tensor, *, b_mn: bool = False, bias=None,
                gelu_aux=None, gelu_grad_of=None, out=None, bn: int = 0) -> torch.Tensor:
        if self.failed:
            raise RuntimeError("this AG->GEMM operator previously failed (its chunk counters are out of step)")
        n = w.shape[1] if b_mn else w.shape[0]
        if shard.shape != (self.m // self.world, self.k):
            raise ValueError(f"shard must be [{self.m // self.world}, {self.k}]")
        if w.dim() != 2 or (w.shape[0] if b_mn else w.shape[1]) != self.k or w.stride(-1) != 1:
            raise ValueError(f"w must be 2-D with K={self.k} ({'[K, N]' if b_mn else '[N, K]'}) and unit inner stride")
        for t, name in ((shard, "shard"), (w, "w")):
            if t.dtype != torch.bfloat16 or t.device != self.device:
                raise ValueError(f"{name} must be bf16 on {self.device}")
        if bias is not None and tuple(bias.shape) != (n,):
            raise ValueError(f"bias must have shape [{n}]")
        for t, name in ((gelu_aux, "gelu_aux"), (gelu_grad_of, "gelu_grad_of"), (out, "out")):
            if t is not None and tuple(t.shape) != (self.m, n):
                raise ValueError(f"{name} must have shape [{self.m}, {n}]")
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
        # The counter target is cumulative over calls (every CTA of every call bumps
        # each owner's counter once): a launch that fails leaves it out of step, so
        # the operator refuses further calls; the lock keeps target and launch paired.
        with self._lock:
            try:
                grid = lib().gemm_grid(self.m, n, bn, 0)
                target = self.flag_total + grid
                with tracing.scope("ag_gemm"):
                    lib().ag_gemm(shard.contiguous(), self.gathered, w, b_mn, out, epi, bias, aux,
                                  self.gather.ptrs.data_ptr(), self.flags.ptrs.data_ptr(), self.flags.local,
                                  self.rank, self.world, target, self._order(n, bn), self.status,
                                  self.timeout_ns, bn)
                self.flag_total = target
            except BaseException:
                self.failed = True
                raise
            count_launch()
            self.calls += 1
        return out

    def close(self):
        if isinstance(self.gather, SymmetricBuffer) and self.gather._owned:
            self.gather.close()
            self.flags.close()
