"""Byte/bit parity of this framework's TACO codec and ordered reductions with the
reference's OWN kernels (TempName-5090 src/taco/codec.cu, compiled unmodified
for sm_100a by baseline/build_reference_codec.py), on the same GPU and inputs."""
import ctypes
import os

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "baseline", "_ref", "libref_taco_codec.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(LIB):
        # Build the reference's own codec (unmodified) with nvcc from its staged
        # source or the reference checkout; skip only when neither exists.
        import importlib.util
        spec = importlib.util.spec_from_file_location("build_reference_codec",
                                                      os.path.join(ROOT, "baseline", "build_reference_codec.py"))
        builder = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(builder)
        if builder.find_source() is None:
            pytest.skip("reference codec source not available (baseline/_ref or the reference checkout)")
        builder.build()
    lib = ctypes.CDLL(LIB)
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.flux_5090_encode.argtypes = [vp, vp, i64, vp]
    lib.flux_5090_decode.argtypes = [vp, vp, i64, vp]
    lib.flux_5090_reduce.argtypes = [vp, vp, vp, i64, i32, i32, vp]
    lib.flux_5090_decode_reduce.argtypes = [vp, vp, vp, i64, i32, i32, vp]
    for f in (lib.flux_5090_encode, lib.flux_5090_decode, lib.flux_5090_reduce, lib.flux_5090_decode_reduce):
        f.restype = i32
    return lib


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _inputs(n, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(n, generator=g, device="cuda")
    x[::97] *= 40.0          # outliers
    x[128:256] = 0.0         # an all-zero group
    x[256:384] *= 1e-4       # a tiny-variance group
    return x.to(torch.bfloat16)


def test_encode_decode_byte_identical(ref):
    from tempname_5090_b200.ops import taco
    for seed in range(3):
        x = _inputs(128 * 512, seed)
        ours = taco.encode(x)
        theirs = torch.empty_like(ours)
        assert ref.flux_5090_encode(x.data_ptr(), theirs.data_ptr(), x.numel(), _stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(ours, theirs)
        d_ours = taco.decode(ours, x.numel())
        d_theirs = torch.empty_like(x)
        assert ref.flux_5090_decode(ours.data_ptr(), d_theirs.data_ptr(), x.numel(), _stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(d_ours, d_theirs)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ordered_reductions_bit_identical(ref, world):
    from tempname_5090_b200.ops import taco
    n = 128 * 256
    local = _inputs(n, 10)
    remote = torch.cat([_inputs(n, 20 + s) for s in range(world - 1)])
    packets = torch.cat([taco.encode(remote[s * n:(s + 1) * n]) for s in range(world - 1)])
    for rank in range(world):
        ours = taco.ordered_reduce(local, remote, rank, world)
        theirs = torch.empty_like(local)
        assert ref.flux_5090_reduce(local.data_ptr(), remote.data_ptr(), theirs.data_ptr(), n, rank, world, _stream()) == 0
        ours_q = taco.decode_reduce(local, packets, rank, world)
        theirs_q = torch.empty_like(local)
        assert ref.flux_5090_decode_reduce(local.data_ptr(), packets.data_ptr(), theirs_q.data_ptr(), n, rank, world,
                                           _stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(ours, theirs)
        assert torch.equal(ours_q, theirs_q)


def test_fused_gemm_epilogue_packets_match_reference_encoder(ref):
    """The TACO encoder inside the GemmRS epilogue vs the reference encoder of the
    same BF16 partial: emulated 2-rank push, then compare the received packet bytes."""
    from tempname_5090_b200.parallel.gemm_rs import GemmRS
    from tempname_5090_b200.parallel.symmetric import SymmetricBuffer
    from tempname_5090_b200.ops import gemm as G
    from tempname_5090_b200.parallel.mapping import PushLanes
    world, m, n, k, chunk = 2, 768, 512, 384, 128
    rows = m // world
    lanes = PushLanes(rows, n, chunk, world)
    recv = [SymmetricBuffer.emulated(lanes.recv_bytes, world) for _ in range(2)]
    flags = SymmetricBuffer.emulated(lanes.flag_words * 4, world)
    op = GemmRS(m, n, k, arm="flux_taco", chunk_rows=chunk,
                _emulate=(0, world, [b.as_rank(0) for b in recv], flags.as_rank(0)))
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (0.05 * torch.randn((n, k), generator=g, device="cuda")).to(torch.bfloat16)
    op.begin()
    op.push(x, w)  # rank 0 pushes the rows of rank 1 as packets into rank 1's slot 0
    torch.cuda.synchronize()
    partial = G.matmul(x, w, bn=256)
    pbytes = chunk * n // 128 * 136
    parity = op.epoch & 1
    region = recv[parity].view(1, (lanes.recv_bytes,), torch.uint8)  # rank 1's receive regions
    for blk in range(rows // chunk):
        # block blk of source 0 sits in lane blk % 2, packet blk // 2 of that lane
        start = lanes.slot_offset(blk % 2, 0) + (blk // 2) * pbytes
        block = partial[rows + blk * chunk: rows + (blk + 1) * chunk].contiguous()
        theirs = torch.empty(pbytes, dtype=torch.uint8, device="cuda")
        assert ref.flux_5090_encode(block.data_ptr(), theirs.data_ptr(), block.numel(), _stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(region[start:start + pbytes], theirs)
