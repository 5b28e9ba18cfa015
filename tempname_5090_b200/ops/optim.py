"""Global gradient norm and fused AdamW over flat FP32 master buffers.

The clip coefficient min(max_norm / (norm + 1e-6), 1) is computed on the
device from the all-reduced FP64 squared norm, so a step never waits on the
host.  Update rule and ordering: torch.optim.AdamW (single-tensor) as used by
TempName-5090 (model.py:382-420): decoupled decay on matrices only,
betas (0.9, 0.95), eps 1e-8, BF16 copy-out of the FP32 master.
"""
from __future__ import annotations

import math

import torch

from .._native import count_launch, lib, status_tensor


def sqsum(grad: torch.Tensor, out: torch.Tensor, accumulate: bool = False, partial=None):
    """out (fp64 scalar) (+)= sum(float(grad)^2), deterministic."""
    if grad.is_cuda:
        parts = lib().grad_sqsum_parts(grad.numel())
        if partial is None or partial.numel() < parts:
            partial = torch.empty(parts, dtype=torch.float64, device=grad.device)
        lib().grad_sqsum(grad, partial, out, accumulate)
        count_launch(2)
        return out
    s = grad.float().square().sum(dtype=torch.float64)
    if accumulate:
        out += s
    else:
        out.copy_(s)
    return out


def adamw(master, m, v, grad, param, n_decay, norm2, *, max_norm, lr, weight_decay, beta1, beta2,
          eps, step):
    """One AdamW step on a flat region; the first n_decay elements are decayed."""
    if master.is_cuda:
        lib().adamw_step(master, m, v, grad, param, n_decay, norm2, max_norm, lr, weight_decay,
                         beta1, beta2, eps, step, status_tensor(master.device))
        count_launch()
        return
    total = float(norm2.item())
    coef = min(max_norm / (math.sqrt(total) + 1e-6), 1.0) if max_norm > 0 else 1.0
    g = grad.float() * coef
    p = master.clone()
    p[:n_decay] *= 1 - lr * weight_decay
    m.lerp_(g, 1 - beta1)
    v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
    p.addcdiv_(m, denom, value=-lr / bc1)
    master.copy_(p)
    param.copy_(p.to(param.dtype))
