"""How many SMs a fused NVLink operator gives to its communication CTAs.

A fused launch splits the GPU: `c` CTAs move data (reducer / gatherer roles),
the other SMs run the GEMM.  The launch ends when the slower side ends, so
`comm_ctas` balances an estimate of the two:

    gemm(c) = FLOPs / ((SMs - c) * per-SM GEMM rate)
    comm(c) = remote bytes / min(NVLink rate, c * per-CTA bulk rate)

The rates are B200 measurements of this framework's kernels: ~8 TFLOP/s per
SM for the tcgen05 GEMM at these shapes (about 1.1-1.2 PFLOP/s over 132-148
SMs), ~580 GB/s per GPU for bulk pulls over NVLink 5 with both directions
busy, and ~22 GB/s per communication CTA when it pulls from all peers in turn.
A projection with a short K (attention out-projection, K = h/W) is
NVLink-bound and gets more communication CTAs; a long-K one keeps its SMs for
the GEMM.  The choice depends only on shapes, so every rank picks the same.
"""
from __future__ import annotations

SMS = 148
GEMM_TFLOPS_PER_SM = 8.0
NVLINK_GBS = 580.0
CTA_GBS = 22.0
CANDIDATES = (16, 20, 24, 32, 40, 48)


def estimate_us(flops: float, remote_bytes: float, comm: int, sms: int = SMS) -> float:
    gemm = flops / ((sms - comm) * GEMM_TFLOPS_PER_SM * 1e6)
    comm_t = remote_bytes / (min(NVLINK_GBS, comm * CTA_GBS) * 1e3)
    return max(gemm, comm_t)


def comm_ctas(flops: float, remote_bytes: float, sms: int = SMS) -> int:
    """The candidate with the smallest estimated launch time (ties: fewer CTAs)."""
    return min(CANDIDATES, key=lambda c: (round(estimate_us(flops, remote_bytes, c, sms), 1), c))


def gemm_rs_comm_ctas(m: int, n: int, k: int, world: int) -> int:
    """GEMM -> reduce-scatter: each rank pulls (W-1)/W of an [M, N] BF16 partial."""
    return comm_ctas(2.0 * m * n * k, (world - 1) / world * m * n * 2)


def ag_gemm_comm_ctas(m: int, n: int, k: int, world: int) -> int:
    """All-gather -> GEMM: each rank pulls (W-1)/W of the gathered [M, K] BF16 input."""
    return comm_ctas(2.0 * m * n * k, (world - 1) / world * m * k * 2)
