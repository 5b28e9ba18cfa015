"""CPU oracle of the TACO codec (stdlib only) and the ordered BF16 reduction."""
import math
import random
import struct
import subprocess
import sys

import pytest

from tempname_5090_b200.utils import reference as ref


def test_every_finite_code_round_trips():
    for code in range(256):
        value = ref.e4m3_decode(code)
        if math.isnan(value):
            assert code & 127 == 127
            continue
        assert ref.e4m3_encode(value) == code or (value == 0 and ref.e4m3_encode(value) in (0, 128))


def test_signed_zero_and_saturation():
    assert ref.e4m3_encode(0.0) == 0
    assert ref.e4m3_encode(-0.0) == 128
    assert ref.e4m3_encode(1e9) == 126
    assert ref.e4m3_encode(-1e9) == 128 | 126
    assert ref.e4m3_decode(126) == 448.0


def test_midpoints_tie_to_even_code():
    for code in range(126):
        lo, hi = ref.e4m3_decode(code), ref.e4m3_decode(code + 1)
        mid = (lo + hi) / 2
        if ref.fp32(mid) != mid:
            continue
        expected = code if code % 2 == 0 else code + 1
        assert ref.e4m3_encode(mid) == expected, (code, mid)


def test_hadamard_is_orthonormal():
    rnd = random.Random(1)
    x = [rnd.uniform(-1, 1) for _ in range(128)]
    y = ref.hadamard_fp64(ref.hadamard_fp64(x))
    assert max(abs(a - b) for a, b in zip(x, y)) < 1e-12
    impulse = ref.hadamard_fp64([1.0] + [0.0] * 127)
    assert all(abs(v - 1 / math.sqrt(128)) < 1e-15 for v in impulse)


def test_packet_layout_is_soa():
    rnd = random.Random(2)
    values = [rnd.gauss(0, 1) for _ in range(256)]
    packet = ref.encode(values)
    assert len(packet) == 2 * 136 == ref.packet_bytes(256)
    g0 = ref.encode_group(values[:128])
    g1 = ref.encode_group(values[128:])
    assert packet[:128] == g0[0] and packet[128:256] == g1[0]
    assert struct.unpack_from("<2f", packet, 256) == (g0[1], g1[1])
    assert struct.unpack_from("<2f", packet, 264) == (g0[2], g1[2])


def test_round_trip_error_bound():
    rnd = random.Random(3)
    values = [ref.bf16_round(rnd.gauss(0, 1)) for _ in range(128 * 4)]
    decoded = ref.decode(ref.encode(values))
    assert ref.relative_l2(decoded, values) < 0.05


def test_ordered_reduction_rounds_after_each_source():
    # 256 + 1 = 257 is not representable in bf16 (rounds to 256): order matters.
    local = [1.0]
    remote = [[256.0], [-256.0], [1.0]]
    assert ref.reduce_sources(local, remote, 0, 4) == [1.0]   # ((1+256)-256)+1 = 1
    assert ref.reduce_sources(local, remote, 3, 4) == [2.0]   # ((256-256)+1)+1 = 2


def test_bf16_rounding_rne_and_nan():
    assert ref.bf16_round(1.0 + 2 ** -8) == 1.0           # tie -> even
    assert ref.bf16_round(1.0 + 3 * 2 ** -9) == 1.0 + 2 ** -7
    assert math.isnan(ref.bf16_round(float("nan")))


def test_oracle_imports_no_torch():
    code = ("import sys; import tempname_5090_b200.utils.reference; "
            "assert 'torch' not in sys.modules")
    subprocess.run([sys.executable, "-c", code], check=True)


def test_rejects_bad_packets():
    with pytest.raises(ValueError):
        ref.decode(b"\x00" * 135)
    with pytest.raises(ValueError):
        ref.decode_group(b"\x7f" * 128, 1.0, 1.0)
    with pytest.raises(ValueError):
        ref.encode([1.0] * 100)
