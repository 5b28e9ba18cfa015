"""Vocab-parallel cross-entropy (FP32 statistics over BF16 logits).

Forward per row: max over the local vocabulary shard -> all-reduce MAX;
sum exp(x - max) and the target logit (if local) -> one all-reduce SUM of both;
loss = log(sum) + max - target.  Backward writes dlogits = (softmax - onehot) *
scale in place over the logits (they are dead after the loss).
Semantics: VocabCrossEntropy, TempName-5090 python/flux_5090/model.py:143-176.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._native import count_launch, lib


class CEState:
    __slots__ = ("gmax", "sumexp", "start", "rows")

    def __init__(self, gmax, sumexp, start, rows):
        self.gmax, self.sumexp, self.start, self.rows = gmax, sumexp, start, rows


def forward(logits: torch.Tensor, targets: torch.Tensor, group=None, rank: int = 0, world: int = 1,
            scale: float | None = None):
    """Return (mean loss scalar tensor [fp32], state).  `scale` defaults to 1/rows."""
    M, V = logits.shape
    start = rank * V
    scale = 1.0 / M if scale is None else scale
    if logits.is_cuda:
        dev = logits.device
        stats = torch.empty((3, M), dtype=torch.float32, device=dev)
        rowmax, both = stats[0], stats[1:]
        lib().ce_stats(logits, targets, start, rowmax, both[1])
        count_launch()
        if world > 1:
            dist.all_reduce(rowmax, op=dist.ReduceOp.MAX, group=group)
        lib().ce_sumexp(logits, rowmax, both[0])
        count_launch()
        if world > 1:
            dist.all_reduce(both, group=group)
        loss = torch.empty(1, dtype=torch.float32, device=dev)
        lib().ce_loss(rowmax, both[0], both[1], None, loss, scale)
        count_launch()
        return loss, CEState(rowmax, both[0], start, M)
    work = logits.float()
    gmax = work.max(-1).values
    if world > 1:
        dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    exps = (work - gmax[:, None]).exp()
    denom = exps.sum(-1)
    local = targets - start
    mask = (local >= 0) & (local < V)
    picked = work.gather(1, local.clamp(0, V - 1)[:, None]).squeeze(1) * mask
    if world > 1:
        both = torch.stack([denom, picked])
        dist.all_reduce(both, group=group)
        denom, picked = both[0], both[1]
    loss = ((denom.log() + gmax - picked).sum() * scale).reshape(1)
    return loss, CEState(gmax, denom, start, M)


def backward(logits: torch.Tensor, targets: torch.Tensor, state: CEState, scale: float):
    """In place: logits <- (softmax - onehot) * scale (BF16)."""
    M, V = logits.shape
    if logits.is_cuda:
        lib().ce_bwd(logits, targets, state.start, state.gmax, state.sumexp, scale, None)
        count_launch()
        return logits
    p = (logits.float() - state.gmax[:, None]).exp() / state.sumexp[:, None]
    local = targets - state.start
    mask = (local >= 0) & (local < V)
    rows = torch.arange(M)
    p[rows[mask], local[mask]] -= 1.0
    logits.copy_((p * scale).to(logits.dtype))
    return logits
