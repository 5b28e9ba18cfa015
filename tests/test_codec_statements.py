"""The torch CPU statement of the TACO codec (ops.taco, FP32) against the
stdlib FP64 oracle (utils.reference), and the reduction-placement rules the
receivers rely on.  Follows the reference's worker-math checks
(tests/test_worker_math.py:14-59 of TempName-5090)."""
import random

import torch

from tempname_5090_b200.ops import taco
from tempname_5090_b200.utils import reference as ref


def _groups(seed, count=6):
    rng = random.Random(seed)
    out = []
    for g in range(count):
        scale = 10.0 ** rng.uniform(-3, 3)
        vals = [ref.bf16_round(rng.gauss(0.0, scale)) for _ in range(128)]
        if g == 1:
            vals[5] = ref.bf16_round(vals[5] * 300.0)   # one outlier in the group
        if g == 2:
            vals = [0.0] * 128                          # an all-zero group
        out.append(vals)
    return out


def test_fp32_statement_tracks_fp64_oracle():
    for seed in range(4):
        groups = _groups(seed)
        flat = [v for g in groups for v in g]
        x = torch.tensor(flat, dtype=torch.float32).to(torch.bfloat16)
        pkt_torch = taco.encode_cpu(x)
        pkt_ref = ref.encode(flat)
        assert pkt_torch.numel() == len(pkt_ref) == taco.packet_bytes(len(flat)) == ref.packet_bytes(len(flat))
        dec_torch = taco.decode_cpu(pkt_torch, len(flat)).float()
        dec_ref = torch.tensor(ref.decode(pkt_ref), dtype=torch.float32)
        # Both decode to (almost) the same values; codes may differ only on FP32-vs-FP64 ties.
        for g in range(len(groups)):
            sl = slice(128 * g, 128 * (g + 1))
            norm = max(dec_ref[sl].norm().item(), 1e-30)
            assert (dec_torch[sl] - dec_ref[sl]).norm().item() <= 0.02 * norm + 1e-30, (seed, g)
        codes_equal = (pkt_torch[:len(flat)].numpy().tobytes() == bytes(pkt_ref[:len(flat)]))
        mismatches = sum(a != b for a, b in zip(pkt_torch[:len(flat)].tolist(), pkt_ref[:len(flat)]))
        assert codes_equal or mismatches <= len(flat) // 100, mismatches


def test_local_source_is_never_quantized():
    """decode_reduce adds the owner's own partial in BF16; only remote sources pass the codec."""
    g = torch.Generator().manual_seed(3)
    local = torch.randn(512, generator=g).to(torch.bfloat16)
    zeros = torch.zeros(512, dtype=torch.bfloat16)
    for world, rank in ((2, 0), (2, 1), (4, 2)):
        packets = torch.cat([taco.encode_cpu(zeros) for _ in range(world - 1)])
        out = taco.decode_reduce(local, packets, rank, world)
        assert torch.equal(out, local)


def test_bf16_order_semantics():
    """Rounding after each source in index order: 256 + 1 - 256 + 1 = 1 (not 2)."""
    srcs = [torch.tensor([v], dtype=torch.bfloat16) for v in (256.0, 1.0, -256.0, 1.0)]
    assert taco.ordered_sum_cpu(srcs).item() == 1.0
    assert ref.reduce_sources([256.0], [[1.0], [-256.0], [1.0]], 0, 4) == [1.0]
