"""The allocation-free sum-of-squares entry point, called through its exported
C symbol, against the regular (workspace-taking) entry point.

It serves callers that cannot allocate device memory: code hosted by a
framework that owns all device memory, or loops that cannot afford the
device-wide synchronisation of cudaMalloc.  This file is collected last so a
run that stops at the first failure has already run every other test.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    from tempname_5090_b200 import _C  # loads libtorch and the extension first
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.tn5b_grad_sqsum_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_regular_entry_point_twice(dtype):
    from tempname_5090_b200.ops import optim
    fn = _entry()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row share the scratch array
        g = torch.Generator(device="cuda").manual_seed(10 + call)
        n = 3_000_000 + 8 * call
        x = (torch.randn(n, generator=g, device="cuda") * (call + 1)).to(dtype)
        out = torch.full((), float("nan"), dtype=torch.float64, device="cuda")
        rc = fn(x.data_ptr(), int(dtype == torch.float32), n, out.data_ptr(), stream)
        assert rc == 0
        ref = torch.zeros((), dtype=torch.float64, device="cuda")
        optim.sqsum(x, ref)
        torch.cuda.synchronize()
        assert abs(out.item() - ref.item()) <= 1e-6 * ref.item()


def test_noalloc_rejects_sizes_beyond_the_maximum():
    fn = _entry()
    x = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((), dtype=torch.float64, device="cuda")
    too_many = 16384 * 16384 + 8
    assert fn(x.data_ptr(), 0, too_many, out.data_ptr(), None) == -2
    assert fn(x.data_ptr(), 0, 12, out.data_ptr(), None) == -1  # not a multiple of 8
