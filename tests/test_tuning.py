"""Communication-CTA choice of the fused operators (`parallel/tuning.py`):
the launch time estimate is the slower of the GEMM on the remaining SMs and
the transfer at min(NVLink rate, CTAs x per-CTA rate)."""
import pytest

from tempname_5090_b200.parallel import tuning


def test_estimate_is_the_slower_side():
    # 100 GFLOP on 148 - 20 SMs vs 40 MB over min(580, 20 * 22) GB/s
    gemm = 100e9 / ((148 - 20) * tuning.GEMM_TFLOPS_PER_SM * 1e6)
    comm = 40e6 / (min(tuning.NVLINK_GBS, 20 * tuning.CTA_GBS) * 1e3)
    assert tuning.estimate_us(100e9, 40e6, 20) == pytest.approx(max(gemm, comm))


def test_choice_is_a_candidate_and_minimises_the_estimate():
    for flops, remote in ((137e9, 58.7e6), (34e9, 58.7e6), (275e9, 33e6), (1e9, 1e6)):
        c = tuning.comm_ctas(flops, remote)
        assert c in tuning.CANDIDATES
        best = min(round(tuning.estimate_us(flops, remote, x), 1) for x in tuning.CANDIDATES)
        assert round(tuning.estimate_us(flops, remote, c), 1) == best
        # ties go to fewer communication CTAs (more SMs for the GEMM)
        assert all(x >= c for x in tuning.CANDIDATES if round(tuning.estimate_us(flops, remote, x), 1) == best)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_short_k_projection_gets_at_least_as_many_comm_ctas(world):
    # The attention out-projection (K = h/W) is NVLink-bound; the FC2 shape (K = f/W) less so.
    m, h, f = 8192, 4096, 16384
    assert tuning.gemm_rs_comm_ctas(m, h, h // world, world) >= tuning.gemm_rs_comm_ctas(m, h, f // world, world)


def test_the_choice_depends_only_on_shapes():
    # every rank computes the same count (no device query, no randomness)
    assert tuning.ag_gemm_comm_ctas(8192, 1536, 4096, 8) == tuning.ag_gemm_comm_ctas(8192, 1536, 4096, 8)
