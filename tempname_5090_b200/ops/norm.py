"""LayerNorm forward/backward, GeLU backward and column sums.

CUDA tensors: native sm_100a kernels.  CPU tensors: the same math in torch
(test oracle path).  Semantics: F.layer_norm in FP32 on BF16 storage.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .._native import count_launch, lib


def layer_norm_fwd(x, weight, bias, eps, out=None):
    """Returns (y, mean, rstd); y may be written into `out` (row-strided view allowed)."""
    rows, H = x.shape
    if x.is_cuda:
        y = torch.empty((rows, H), dtype=torch.bfloat16, device=x.device) if out is None else out
        mean = torch.empty(rows, dtype=torch.float32, device=x.device)
        rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
        lib().layernorm_fwd(x, weight, bias, y, mean, rstd, float(eps))
        count_launch()
        return y, mean, rstd
    xf = x.float()
    mean = xf.mean(1)
    var = xf.var(1, unbiased=False)
    rstd = torch.rsqrt(var + eps)
    y = ((xf - mean[:, None]) * rstd[:, None] * weight.float() + bias.float()).to(x.dtype)
    if out is not None:
        out.copy_(y)
        y = out
    return y, mean, rstd


def layer_norm_bwd(dy, x, weight, mean, rstd, dres=None, workspace=None, out=None):
    """Returns (dx, dweight, dbias); dx = bf16(bf16(ln_dx) + dres) when dres is given,
    written into `out` (contiguous [rows, H]) when given."""
    rows, H = x.shape
    if x.is_cuda:
        dx = torch.empty_like(x) if out is None else out
        dw = torch.empty(H, dtype=torch.bfloat16, device=x.device)
        db = torch.empty(H, dtype=torch.bfloat16, device=x.device)
        need = lib().layernorm_bwd_workspace(rows, H)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(need, dtype=torch.float32, device=x.device)
        lib().layernorm_bwd(dy.contiguous(), x.contiguous(), weight, mean, rstd, dx, dw, db, workspace, dres)
        count_launch(4)
        return dx, dw, db
    xf, g = x.float(), dy.float()
    xhat = (xf - mean[:, None]) * rstd[:, None]
    gw = g * weight.float()
    s1 = gw.mean(1, keepdim=True)
    s2 = (gw * xhat).mean(1, keepdim=True)
    dx = rstd[:, None] * (gw - s1 - xhat * s2)
    if dres is not None:
        dx = dx.to(torch.bfloat16).float() + dres.float()
    dx = dx.to(x.dtype)
    if out is not None:
        out.copy_(dx)
        dx = out
    return (dx, (g * xhat).sum(0).to(x.dtype), g.sum(0).to(x.dtype))


def gelu_bwd(dy, pre):
    if dy.is_cuda:
        dx = torch.empty_like(dy)
        lib().gelu_bwd(dy.contiguous(), pre.contiguous(), dx)
        count_launch()
        return dx
    z = pre.float()
    cdf = 0.5 * (1 + torch.erf(z * 0.7071067811865476))
    pdf = 0.3989422804014327 * torch.exp(-0.5 * z * z)
    return (dy.float() * (cdf + z * pdf)).to(dy.dtype)


def column_sum(g, out=None, workspace=None):
    """bf16 column sums of a [rows, cols] bf16 matrix (bias gradients), deterministic."""
    rows, cols = g.shape
    if g.is_cuda:
        out = torch.empty(cols, dtype=torch.bfloat16, device=g.device) if out is None else out
        parts = 64 if rows >= 4096 else (32 if rows >= 512 else 1)
        if workspace is None or workspace.numel() < parts * cols:
            workspace = torch.empty(parts * cols, dtype=torch.float32, device=g.device)
        lib().column_sum(g, out, workspace)
        count_launch(2)
        return out
    s = g.float().sum(0).to(g.dtype)
    if out is not None:
        out.copy_(s)
        return out
    return s
