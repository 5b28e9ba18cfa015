"""CPU reference check of the reduce-scatter numerics (no GPU).

8 virtual TP ranks each compute A_r[1024, 512] (bf16, N(0,1)) @ W_r[512, 1024]
(bf16, N(0, 0.02)); the BF16 [1024, 1024] partials are reduce-scattered by rows
into 8 x [128, 1024] with the ordered BF16 sum, once plain and once with every
remote source through the TACO H128/E4M3 codec; both are compared with the
FP32 sum of the exact products.  Seed 0.

    python -m tempname_5090_b200.runner.cpu_check
"""
from __future__ import annotations

import json


def run(seed: int = 0, world: int = 8, m: int = 1024, k: int = 512, n: int = 1024) -> dict:
    import torch
    from ..ops import taco
    g = torch.Generator().manual_seed(seed)
    a = [torch.randn((m, k), generator=g).to(torch.bfloat16) for _ in range(world)]
    w = [(0.02 * torch.randn((k, n), generator=g)).to(torch.bfloat16) for _ in range(world)]
    exact = [a[r].float() @ w[r].float() for r in range(world)]
    partial = [e.to(torch.bfloat16) for e in exact]
    fp32_sum = sum(exact)
    rows = m // world
    plain_err, taco_err = [], []
    plain_out, taco_out = [], []
    for d in range(world):
        sl = slice(d * rows, (d + 1) * rows)
        srcs = [partial[s][sl].contiguous() for s in range(world)]
        plain = taco.ordered_sum_cpu(srcs)
        coded = taco.ordered_sum_cpu([s_ if s == d else taco.decode_cpu(taco.encode_cpu(s_), s_.numel()).reshape(s_.shape)
                                      for s, s_ in enumerate(srcs)])
        ref = fp32_sum[sl]
        plain_err.append(((plain.float() - ref).norm() / ref.norm()).item())
        taco_err.append(((coded.float() - ref).norm() / ref.norm()).item())
        plain_out.append(plain)
        taco_out.append(coded)
    return dict(world=world, shape=[m, k, n], seed=seed,
                plain_rel_l2_max=max(plain_err), taco_rel_l2_max=max(taco_err),
                plain_rel_l2=plain_err, taco_rel_l2=taco_err,
                wire_bytes_per_source_bf16=(world - 1) * rows * n * 2,
                wire_bytes_per_source_taco=(world - 1) * rows * n // 128 * 136)


if __name__ == "__main__":
    print(json.dumps(run(), indent=1))
