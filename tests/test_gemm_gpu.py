"""tcgen05 GEMM numerics against a plain PyTorch fp32 reference of the same op."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(a, b, a_t, b_t):
    af = a.float().t() if a_t else a.float()
    bf = b.float().t() if b_t else b.float()
    return af @ bf.t()


def _rel(x, y):
    return ((x.float() - y.float()).norm() / y.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 320), (384, 128, 1024),
                                   (1000, 520, 200), (2048, 6288, 4096)])
@pytest.mark.parametrize("a_t,b_t", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("kind", [0, 1, 2])
def test_gemm_matches_fp32(M, N, K, a_t, b_t, kind):
    from tempname_5090_b200.ops.gemm import matmul
    from tempname_5090_b200._native import check_status
    if (a_t and M % 8) or (b_t and N % 8):
        pytest.skip("MN-major storage needs 16-byte rows")
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    a = torch.randn((K, M) if a_t else (M, K), generator=g, device="cuda").to(torch.bfloat16)
    b = torch.randn((K, N) if b_t else (N, K), generator=g, device="cuda").to(torch.bfloat16)
    out = matmul(a, b, a_t=a_t, b_t=b_t, bn=256 if kind else 0, pair=kind)
    torch.cuda.synchronize()
    check_status()
    ref = _ref(a, b, a_t, b_t)
    assert _rel(out, ref) < 1e-2


@pytest.mark.parametrize("bn,kind", [(128, 0), (256, 0), (256, 1), (256, 2)])
def test_gemm_epilogues(bn, kind):
    from tempname_5090_b200.ops.gemm import matmul
    M, N, K = 512, 768, 256
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn((N, K), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bias = torch.randn((N,), generator=g, device="cuda").to(torch.bfloat16)
    ref = a.float() @ b.float().t()
    out = matmul(a, b, bias=bias, bn=bn, pair=kind)
    assert _rel(out, ref + bias.float()) < 1e-2
    aux = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    out = matmul(a, b, bias=bias, gelu_aux=aux, bn=bn, pair=kind)
    pre = (ref + bias.float()).to(torch.bfloat16)
    assert _rel(aux, pre) < 1e-2
    assert _rel(out, torch.nn.functional.gelu(pre.float())) < 1e-2
    res = torch.randn((M, N), generator=g, device="cuda").to(torch.bfloat16)
    out = matmul(a, b, bias=bias, residual=res, bn=bn, pair=kind)
    expect = ((res.float() + ref.to(torch.bfloat16).float()).to(torch.bfloat16).float() + bias.float())
    assert _rel(out, expect) < 1e-2
    base = torch.randn((M, N), generator=g, device="cuda").to(torch.bfloat16)
    acc = base.clone()
    matmul(a, b, out=acc, accumulate=True, bn=bn, pair=kind)
    assert _rel(acc, base.float() + ref) < 1e-2


def test_gemm_strided_output_and_tile_order():
    from tempname_5090_b200.ops.gemm import matmul
    M, N, K = 256, 512, 128
    a = torch.randn((M, K), device="cuda").to(torch.bfloat16)
    b = torch.randn((N, K), device="cuda").to(torch.bfloat16)
    big = torch.zeros((M, 2 * N), dtype=torch.bfloat16, device="cuda")
    view = big[:, N:]
    tiles = (M // 128) * (N // 256)
    order = torch.arange(tiles - 1, -1, -1, dtype=torch.int32, device="cuda")
    matmul(a, b, out=view, bn=256, tile_order=order)
    assert _rel(view, a.float() @ b.float().t()) < 1e-2
    assert big[:, :N].abs().sum().item() == 0


@pytest.mark.parametrize("kind", [1, 2])
def test_pair_tiles_bitwise_equal_single_cta(kind):
    """Same K loop order in every tile kind: identical FP32 accumulators."""
    from tempname_5090_b200.ops.gemm import matmul
    a = torch.randn((1024, 768), device="cuda").to(torch.bfloat16)
    b = torch.randn((1536, 768), device="cuda").to(torch.bfloat16)
    x = matmul(a, b, bn=256, pair=0)
    y = matmul(a, b, bn=256, pair=kind)
    assert torch.equal(x, y)


@pytest.mark.parametrize("M,N,K", [(8192, 4096, 8192), (12288, 4096, 8192)])
def test_split_wide_gemm_tail_runs_as_pair_tiles(M, N, K):
    """A long-K wide-tile GEMM whose last wave is at most half full runs that
    wave as CTA-pair 256 x 256 tiles in a second launch (8192 x 4096: 3 wide
    waves + a pair wave instead of 4 wide waves); every tile kind accumulates K
    in the same order, so the result is bitwise the single-CTA one, with epilogues."""
    from tempname_5090_b200.ops.gemm import matmul
    from tempname_5090_b200._native import check_status
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    b = (0.05 * torch.randn((N, K), generator=g, device="cuda")).to(torch.bfloat16)
    bias = torch.randn((N,), generator=g, device="cuda").to(torch.bfloat16)
    single = matmul(a, b, bn=256, pair=0)
    split = matmul(a, b, bn=256, pair=2)
    torch.cuda.synchronize()
    check_status()
    assert torch.equal(single, split)
    assert _rel(split, a.float() @ b.float().t()) < 1e-2
    aux_s = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    aux_w = torch.empty_like(aux_s)
    assert torch.equal(matmul(a, b, bias=bias, gelu_aux=aux_s, bn=256, pair=0),
                       matmul(a, b, bias=bias, gelu_aux=aux_w, bn=256, pair=2))
    assert torch.equal(aux_s, aux_w)
