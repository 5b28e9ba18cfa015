"""Causal attention over a fused QKV buffer [tokens, 3*heads*128] (per-token
layout [3][heads][head_dim], TempName-5090 model.py:254); output
[tokens, heads*128].  CUDA: hand-written sm_100a tcgen05 kernels (TMA-fed,
scores/probabilities/accumulators in tensor memory; forward saves the row
LSE; the backward is two deterministic kernels, dK/dV per key block and dQ per
query block).  CPU: torch math reference (test oracle).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .._native import count_launch, lib, status_tensor

TIMEOUT_NS = 10_000_000_000

HEAD_DIM = 128


def _split(qkv, B, S, H, d):
    q, k, v = qkv.float().reshape(B, S, 3, H, d).permute(2, 0, 3, 1, 4).unbind(0)
    return q, k, v


def forward(qkv: torch.Tensor, B: int, S: int, H: int, out: torch.Tensor | None = None):
    """Return (out [B*S, H*128] bf16, lse [B*H, S] fp32)."""
    d = qkv.shape[1] // (3 * H)
    scale = 1.0 / math.sqrt(d)
    if qkv.is_cuda:
        if d != HEAD_DIM:
            raise ValueError("the CUDA attention kernel is specialised for head_dim 128")
        out = torch.empty((B * S, H * d), dtype=torch.bfloat16, device=qkv.device) if out is None else out
        lse = torch.empty((B * H, S), dtype=torch.float32, device=qkv.device)
        lib().attention_fwd_tc(qkv, out, lse, B, S, H, scale, status_tensor(qkv.device), TIMEOUT_NS)
        count_launch()
        return out, lse
    q, k, v = _split(qkv, B, S, H, d)
    s = (q @ k.transpose(-1, -2)) * scale
    mask = torch.ones(S, S, dtype=torch.bool).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, -1)
    o = torch.softmax(s, -1) @ v
    o = o.transpose(1, 2).reshape(B * S, H * d).to(qkv.dtype)
    if out is not None:
        out.copy_(o)
        o = out
    return o, lse.reshape(B * H, S)


def backward(qkv, out, dout, lse, B: int, S: int, H: int, dqkv: torch.Tensor | None = None,
             debug: torch.Tensor | None = None):
    """`debug`: optional zeroed int64 [2, B*H*S/128, 8] CUDA tensor that receives
    the dK/dV and dQ kernels' per-CTA cycle counters (MMA thread waiting for
    tiles / for the elementwise warps / for the previous block's MMAs, MMA total;
    one elementwise warp waiting for S and dP / working; blocks)."""
    d = qkv.shape[1] // (3 * H)
    scale = 1.0 / math.sqrt(d)
    if qkv.is_cuda:
        dqkv = torch.empty_like(qkv) if dqkv is None else dqkv
        Dvec = torch.empty((B * H, S), dtype=torch.float32, device=qkv.device)
        lib().attention_bwd_tc(qkv, out, dout, lse, Dvec, dqkv, B, S, H, scale, status_tensor(qkv.device),
                               TIMEOUT_NS, debug)
        count_launch(3)
        return dqkv
    q, k, v = _split(qkv, B, S, H, d)
    do = dout.float().reshape(B, S, H, d).transpose(1, 2)
    s = (q @ k.transpose(-1, -2)) * scale
    mask = torch.ones(S, S, dtype=torch.bool).triu(1)
    p = torch.exp(s.masked_fill(mask, float("-inf")) - lse.reshape(B, H, S, 1))
    dv = p.transpose(-1, -2) @ do
    dp = do @ v.transpose(-1, -2)
    Dq = (do * out.float().reshape(B, S, H, d).transpose(1, 2)).sum(-1, keepdim=True)
    ds = p * (dp - Dq)
    dq = ds @ k * scale
    dk = ds.transpose(-1, -2) @ q * scale
    g = torch.stack([dq, dk, dv], 0).permute(1, 3, 0, 2, 4).reshape(B * S, 3 * H * d)
    if dqkv is None:
        return g.to(qkv.dtype)
    dqkv.copy_(g)
    return dqkv
