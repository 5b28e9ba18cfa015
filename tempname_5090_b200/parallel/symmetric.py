"""Symmetric device buffers over NVLink: one allocation per rank, mapped into
every peer through CUDA IPC, with a device-resident table of peer base
pointers for kernels.

Every rank creates the same buffers in the same order (SPMD).  The IPC handles
are exchanged with `all_gather_object` on the process group; each rank opens
its peers' handles once.  Kernels receive `ptrs` (int64 device tensor [world])
and address peer r's copy at ptrs[r] + offset.

`SymmetricBuffer.emulated(nbytes, world)` builds the same object for W
emulated ranks on a single GPU (W local allocations), used by single-GPU tests
of the multi-rank kernels where no launch ever waits on another launch.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._native import lib


class SymmetricBuffer:
    def __init__(self, nbytes: int, group=None, *, _emulate_world: int | None = None):
        self.nbytes = int(nbytes)
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._owned = []      # pointers we allocated (freed on close)
        self._opened = []     # peer pointers we mapped (closed on close)
        if _emulate_world is not None:
            self.world, self.rank = _emulate_world, 0
            self.peers = [lib().symm_alloc(self.nbytes) for _ in range(self.world)]
            self._owned = list(self.peers)
        else:
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
            base = lib().symm_alloc(self.nbytes)
            self._owned = [base]
            handle = lib().ipc_handle(base)
            handles = [None] * self.world
            dist.all_gather_object(handles, (handle, self.nbytes), group=group)
            peers = []
            for r, (h, size) in enumerate(handles):
                if size != self.nbytes:
                    raise RuntimeError("symmetric buffer sizes differ across ranks")
                if r == self.rank:
                    peers.append(base)
                else:
                    p = lib().ipc_open(h)
                    self._opened.append(p)
                    peers.append(p)
            self.peers = peers
        self.ptrs = torch.tensor(self.peers, dtype=torch.int64, device=self.device)
        self.local = self.peers[self.rank]

    @classmethod
    def emulated(cls, nbytes: int, world: int) -> "SymmetricBuffer":
        return cls(nbytes, _emulate_world=world)

    def as_rank(self, rank: int) -> "SymmetricBuffer":
        """Emulation only: the same allocations seen from emulated rank `rank`."""
        clone = object.__new__(SymmetricBuffer)
        clone.__dict__.update(self.__dict__)
        clone._owned, clone._opened = [], []
        clone.rank, clone.local = rank, self.peers[rank]
        return clone

    def view(self, rank: int, shape, dtype, offset: int = 0) -> torch.Tensor:
        """Non-owning tensor view of rank `rank`'s copy (peer memory for r != self)."""
        elem = torch.empty((), dtype=dtype).element_size()
        numel = 1
        for s in shape:
            numel *= s
        if offset + numel * elem > self.nbytes:
            raise ValueError("view exceeds the symmetric buffer")
        return lib().view_ptr(self.peers[rank] + offset, list(shape), dtype, self.device.index)

    def local_view(self, shape, dtype, offset: int = 0) -> torch.Tensor:
        return self.view(self.rank, shape, dtype, offset)

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            lib().ipc_close(p)
        for p in self._owned:
            lib().symm_free(p)
        self._opened, self._owned = [], []

    def __del__(self):  # pragma: no cover - best effort at interpreter exit
        try:
            if self._owned or self._opened:
                self.close()
        except Exception:
            pass
