"""8 virtual ranks, plain and TACO reduce-scatter vs the FP32 sum."""
from tempname_5090_b200.runner import cpu_check


def test_cpu_reference_check_seed0():
    r = cpu_check.run(seed=0)
    assert r["plain_rel_l2_max"] < 0.01
    assert r["taco_rel_l2_max"] < 0.05
    assert r["taco_rel_l2_max"] > r["plain_rel_l2_max"]
    assert r["wire_bytes_per_source_taco"] * 256 == r["wire_bytes_per_source_bf16"] * 136
