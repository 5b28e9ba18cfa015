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

Guard regions (race/overrun detection, off by default): with `guard_bytes`
(or the environment variable TN5B_GUARD_BYTES) every rank's allocation gets a
pattern-filled guard before and after its `nbytes`; pointers and views address
the inner region, and `check_guards()` reports whether this rank's guards (all
ranks' guards when emulated) still hold the pattern -- a kernel that wrote past
either end of a peer's region shows up on that peer.  Only this GPU's own
memory is read.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .._native import lib


GUARD_PATTERN = 0xA5


def default_guard_bytes() -> int:
    g = int(os.environ.get("TN5B_GUARD_BYTES", "0"))
    if g < 0 or g % 256:
        raise ValueError("TN5B_GUARD_BYTES must be a non-negative multiple of 256")
    return g


class SymmetricBuffer:
    def __init__(self, nbytes: int, group=None, *, guard_bytes: int | None = None,
                 _emulate_world: int | None = None):
        self.nbytes = int(nbytes)
        self.guard = default_guard_bytes() if guard_bytes is None else int(guard_bytes)
        if self.guard < 0 or self.guard % 256:
            raise ValueError("guard_bytes must be a non-negative multiple of 256 (keeps 256-byte alignment)")
        total = self.nbytes + 2 * self.guard
        self.device = torch.device("cuda", torch.cuda.current_device())
        self._owned = []      # allocation bases we own (freed on close)
        self._opened = []     # peer allocation bases we mapped (closed on close)
        if _emulate_world is not None:
            self.world, self.rank = _emulate_world, 0
            raw = [lib().symm_alloc(total) for _ in range(self.world)]
            self._owned = list(raw)
            self._guarded = list(raw)  # every emulated rank's guards live on this GPU
        else:
            self.world = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
            base = lib().symm_alloc(total)
            self._owned = [base]
            self._guarded = [base]
            handle = lib().ipc_handle(base)
            handles = [None] * self.world
            dist.all_gather_object(handles, (handle, total), group=group)
            raw = []
            for r, (h, size) in enumerate(handles):
                if size != total:
                    raise RuntimeError("symmetric buffer sizes differ across ranks")
                if r == self.rank:
                    raw.append(base)
                else:
                    p = lib().ipc_open(h)
                    self._opened.append(p)
                    raw.append(p)
        if self.guard:
            for b in self._guarded:
                for off in (0, self.guard + self.nbytes):
                    lib().view_ptr(b + off, [self.guard], torch.uint8, self.device.index).fill_(GUARD_PATTERN)
        self.peers = [b + self.guard for b in raw]
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

    def check_guards(self) -> list:
        """Ranks whose guard regions (on this GPU) no longer hold the pattern.
        Synchronises the device; empty when guards are off or intact."""
        if not self.guard:
            return []
        torch.cuda.synchronize(self.device)
        bad = []
        for b in self._guarded:
            for off in (0, self.guard + self.nbytes):
                v = lib().view_ptr(b + off, [self.guard], torch.uint8, self.device.index)
                if not bool((v == GUARD_PATTERN).all()):
                    rank = self.peers.index(b + self.guard) if len(self._guarded) > 1 else self.rank
                    bad.append(rank)
                    break
        return bad

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
