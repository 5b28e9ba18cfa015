"""tcgen05 BF16 GEMM entry points.

`matmul(a, b)` computes a @ b.T for a [M,K], b [N,K] (the F.linear layout).
Transposed operands are expressed without copies: `a_t=True` means `a` is
stored [K, M] (MN-major), `b_t=True` means `b` is stored [K, N].  Epilogues:
bias, exact GeLU with the pre-activation written to `aux`, residual add
(out = bf16(bf16(res + bf16(acc)) + bias)), accumulate (out += acc) and GeLU
backward (out = bf16(bf16(acc) * gelu'(pre)) with the saved pre-activation).
`pair` selects the tile kind: -1 auto (default), 0 single CTA 128x256 with
double-buffered accumulators, 1 CTA pair 256x256 (tcgen05 cta_group::2), 2 wide
CTA pair 256x512 (two N=256 MMAs per K step, for long K loops).
"""
from __future__ import annotations

import torch

from .._native import count_launch, lib, status_tensor

EPI_BIAS, EPI_GELU, EPI_RESIDUAL, EPI_ACCUMULATE, EPI_GELU_BWD = 1, 2, 4, 8, 16


def matmul(a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = False,
           out: torch.Tensor | None = None, bias: torch.Tensor | None = None,
           gelu_aux: torch.Tensor | None = None, residual: torch.Tensor | None = None,
           accumulate: bool = False, gelu_grad_of: torch.Tensor | None = None, bn: int = 0,
           max_ctas: int = 0, tile_order: torch.Tensor | None = None, pair: int = -1,
           group_m: int = 0, debug: torch.Tensor | None = None) -> torch.Tensor:
    M = a.shape[1] if a_t else a.shape[0]
    N = b.shape[1] if b_t else b.shape[0]
    if not a.is_cuda:
        return _matmul_cpu(a, b, a_t, b_t, out, bias, gelu_aux, residual, accumulate, gelu_grad_of)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    epi = 0
    if bias is not None:
        epi |= EPI_BIAS
    if gelu_aux is not None:
        epi |= EPI_GELU
    if residual is not None:
        epi |= EPI_RESIDUAL
    if accumulate:
        epi |= EPI_ACCUMULATE
    aux = gelu_aux
    if gelu_grad_of is not None:
        epi |= EPI_GELU_BWD
        aux = gelu_grad_of
    lib().gemm(a, a_t, b, b_t, out, epi, bias, aux, residual, status_tensor(a.device),
               bn, max_ctas, tile_order, pair, group_m, debug)
    count_launch()
    return out


def _gelu_grad(z):
    cdf = 0.5 * (1 + torch.erf(z * 0.7071067811865476))
    return cdf + z * 0.3989422804014327 * torch.exp(-0.5 * z * z)


def _matmul_cpu(a, b, a_t, b_t, out, bias, gelu_aux, residual, accumulate, gelu_grad_of):
    """Reference math of every epilogue (FP32 accumulate, BF16 rounding points as on the GPU)."""
    af = a.float().t() if a_t else a.float()
    bf = b.float().t() if b_t else b.float()
    acc = af @ bf.t()
    bf16 = torch.bfloat16
    if residual is not None:
        y = (residual.float() + acc.to(bf16).float()).to(bf16).float()
        if bias is not None:
            y = y + bias.float()
        res = y
    else:
        if bias is not None:
            acc = acc + bias.float()
        res = acc
        if gelu_aux is not None:
            pre = acc.to(bf16)
            gelu_aux.copy_(pre)
            res = torch.nn.functional.gelu(pre.float())
        if gelu_grad_of is not None:
            res = acc.to(bf16).float() * _gelu_grad(gelu_grad_of.float())
    if accumulate:
        res = out.float() + res
    if out is None:
        return res.to(bf16)
    out.copy_(res.to(bf16))
    return out
