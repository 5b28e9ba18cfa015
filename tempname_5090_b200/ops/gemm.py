"""tcgen05 BF16 GEMM entry points.

`matmul(a, b)` computes a @ b.T for a [M,K], b [N,K] (the F.linear layout).
Transposed operands are expressed without copies: `a_t=True` means `a` is
stored [K, M] (MN-major), `b_t=True` means `b` is stored [K, N].  Epilogues:
bias, exact GeLU with the pre-activation written to `aux`, residual add
(out = bf16(bf16(res + bf16(acc)) + bias)) and accumulate (out += acc).
"""
from __future__ import annotations

import torch

from .._native import count_launch, lib, status_tensor

EPI_BIAS, EPI_GELU, EPI_RESIDUAL, EPI_ACCUMULATE = 1, 2, 4, 8


def matmul(a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = False,
           out: torch.Tensor | None = None, bias: torch.Tensor | None = None,
           gelu_aux: torch.Tensor | None = None, residual: torch.Tensor | None = None,
           accumulate: bool = False, bn: int = 0, max_ctas: int = 0,
           tile_order: torch.Tensor | None = None) -> torch.Tensor:
    M = a.shape[1] if a_t else a.shape[0]
    N = b.shape[1] if b_t else b.shape[0]
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
    lib().gemm(a, a_t, b, b_t, out, epi, bias, gelu_aux, residual, status_tensor(a.device),
               bn, max_ctas, tile_order)
    count_launch()
    return out
