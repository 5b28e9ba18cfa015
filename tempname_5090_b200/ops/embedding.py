"""Vocab-parallel embedding lookup/backward and position embedding.

Forward: masked lookup of this rank's vocabulary shard (zeros elsewhere); the
caller reduce-scatters the contributions and adds position rows to its
sequence shard.  Backward is deterministic (stable bucketing, no float atomics).
Semantics: TempName-5090 model.py:240-249.
"""
from __future__ import annotations

import torch

from .._native import count_launch, lib


def lookup(tokens, table, start, out=None):
    M, H = tokens.numel(), table.shape[1]
    out = torch.empty((M, H), dtype=table.dtype, device=table.device) if out is None else out
    if table.is_cuda:
        lib().embed_fwd(tokens, table, out, start)
        count_launch()
        return out
    local = tokens - start
    mask = (local >= 0) & (local < table.shape[0])
    out.copy_(table[local.clamp(0, table.shape[0] - 1)] * mask[:, None].to(table.dtype))
    return out


def positions(rows, row0, S, device):
    return (torch.arange(rows, device=device) + row0) % S


def add_position(x, table, row0):
    if x.is_cuda:
        lib().add_position(x, table, row0)
        count_launch()
        return x
    x.copy_((x.float() + table[positions(x.shape[0], row0, table.shape[0], x.device)].float()).to(x.dtype))
    return x


def position_grad(g, S, row0, out=None):
    rows, H = g.shape
    out = torch.empty((S, H), dtype=g.dtype, device=g.device) if out is None else out
    if g.is_cuda:
        lib().position_bwd(g, out, row0)
        count_launch()
        return out
    acc = torch.zeros((S, H), dtype=torch.float32)
    acc.index_add_(0, positions(rows, row0, S, g.device), g.float())
    out.copy_(acc.to(g.dtype))
    return out


def lookup_grad(tokens, g, dtable, start, accumulate=True, workspace=None):
    """dtable[v] (+)= sum of g rows whose token maps to local row v (position order)."""
    V, H = dtable.shape
    if g.is_cuda:
        need = lib().embed_bwd_workspace(tokens.numel(), V)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(need, dtype=torch.int32, device=g.device)
        lib().embed_bwd(tokens, g, dtable, start, workspace, accumulate)
        count_launch(5)
        return dtable
    local = tokens - start
    mask = (local >= 0) & (local < V)
    acc = torch.zeros((V, H), dtype=torch.float32)
    acc.index_add_(0, local[mask], g[mask].float())
    touched = torch.zeros(V, dtype=torch.bool)
    touched[local[mask]] = True
    if accumulate:
        new = (dtable.float() + acc.to(dtable.dtype).float()).to(dtable.dtype)
        dtable.copy_(torch.where(touched[:, None], new, dtable))
    else:
        dtable.copy_(torch.where(touched[:, None], acc.to(dtable.dtype), dtable))
    return dtable
