"""Standard-library CPU oracle for the TACO H128/E4M3FN codec and ordered BF16 sums.

This module imports no torch.  It is the independent arithmetic the device
codec is checked against (TempName-5090 python/flux_5090/reference.py:1-161):

* BF16 rounding is round-to-nearest-even on the FP32 value, NaN kept quiet.
* E4M3FN encoding saturates to +-448 and picks the nearest finite code, ties
  resolved towards the even code (low mantissa bit 0); signed zero is kept.
* The Hadamard transform is an explicit FP64 Walsh matrix product scaled by
  1/sqrt(128), independent of any butterfly ordering.
* A packet for E elements (E multiple of 128) is SoA:
  payload[E] u8 | quant[E/128] f32 | adaptive[E/128] f32  (136 bytes / group).
* The ordered reduction visits sources 0..W-1, the local partial at its own
  rank, and rounds to BF16 after every addition.
"""
from __future__ import annotations

import bisect
import math
import struct

GROUP_SIZE = 128
GROUP_BYTES = 136
E4M3_MAX = 448.0


def fp32(value: float) -> float:
    """Round a Python float to the nearest FP32 value (overflow -> inf)."""
    try:
        return struct.unpack("<f", struct.pack("<f", float(value)))[0]
    except OverflowError:
        return math.copysign(math.inf, value)


def bf16_bits(value: float) -> int:
    bits = struct.unpack("<I", struct.pack("<f", fp32(value)))[0]
    if (bits & 0x7FFFFFFF) > 0x7F800000:  # NaN: keep it quiet
        return ((bits >> 16) | 0x40) & 0xFFFF
    rounding = 0x7FFF + ((bits >> 16) & 1)
    return ((bits + rounding) >> 16) & 0xFFFF


def bf16_round(value: float) -> float:
    return struct.unpack("<f", struct.pack("<I", bf16_bits(value) << 16))[0]


def e4m3_decode(code: int) -> float:
    if type(code) is not int or not 0 <= code <= 255:
        raise ValueError("an E4M3FN code must be an integer byte")
    sign = -1.0 if code & 0x80 else 1.0
    exponent = (code >> 3) & 0xF
    mantissa = code & 0x7
    if exponent == 0xF and mantissa == 0x7:
        return math.nan
    if exponent == 0:
        return sign * mantissa * 2.0 ** -9  # subnormal: m/8 * 2^-6
    return sign * (1.0 + mantissa / 8.0) * 2.0 ** (exponent - 7)


# Positive finite codes 0..126 in increasing magnitude (the encoding is monotonic).
_POSITIVE = [e4m3_decode(c) for c in range(127)]


def e4m3_encode(value: float) -> int:
    """FP32 value -> E4M3FN code: saturating, nearest, ties to the even code."""
    value = fp32(value)
    if not math.isfinite(value):
        raise ValueError("the E4M3 oracle accepts finite values only")
    sign = 0x80 if math.copysign(1.0, value) < 0 else 0
    magnitude = min(abs(value), E4M3_MAX)
    upper = bisect.bisect_left(_POSITIVE, magnitude)
    if upper == 0:
        return sign
    if upper >= len(_POSITIVE):
        return sign | 126
    lower = upper - 1
    below, above = magnitude - _POSITIVE[lower], _POSITIVE[upper] - magnitude
    if below < above or (below == above and lower % 2 == 0):
        return sign | lower
    return sign | upper


def _walsh_sign(row: int, col: int) -> float:
    return -1.0 if bin(row & col).count("1") & 1 else 1.0


_SIGNS = [[_walsh_sign(r, c) for c in range(GROUP_SIZE)] for r in range(GROUP_SIZE)]


def hadamard_fp64(values) -> list:
    values = [float(v) for v in values]
    if len(values) != GROUP_SIZE or not all(math.isfinite(v) for v in values):
        raise ValueError("the Hadamard oracle needs exactly 128 finite values")
    scale = 1.0 / math.sqrt(GROUP_SIZE)
    return [math.fsum(s * v for s, v in zip(row, values)) * scale for row in _SIGNS]


def encode_group(values):
    """128 BF16-representable values -> (payload bytes, quant scale, adaptive scale).

    FP64 arithmetic: packet bytes next to a rounding threshold may differ from
    the device's FP32 evaluation; decoded values stay within the codec bound.
    """
    values = [bf16_round(v) for v in values]
    if len(values) != GROUP_SIZE or not all(math.isfinite(v) for v in values):
        raise ValueError("encoding needs exactly 128 finite BF16 values")
    variance = max(math.fsum(v * v for v in values) / GROUP_SIZE + 1e-6, 1e-12)
    adaptive = fp32(min(max(E4M3_MAX / math.sqrt(variance), 1e-3), 1e3))
    coefficients = hadamard_fp64([v * adaptive for v in values])
    peak = max(abs(c) for c in coefficients)
    quant = fp32(min(max(max(peak, 1e-12) / E4M3_MAX, 1e-12), 1e6))
    payload = bytes(e4m3_encode(min(max(c / quant, -E4M3_MAX), E4M3_MAX)) for c in coefficients)
    return payload, quant, adaptive


def decode_group(payload, quant: float, adaptive: float) -> list:
    payload = bytes(payload)
    if len(payload) != GROUP_SIZE:
        raise ValueError("a TACO group holds exactly 128 coefficient bytes")
    quant, adaptive = float(quant), float(adaptive)
    if not (math.isfinite(quant) and fp32(1e-12) <= quant <= 1e6 and math.isfinite(adaptive)
            and fp32(1e-3) <= adaptive <= 1e3):
        raise ValueError("corrupt TACO scales")
    coefficients = [e4m3_decode(b) for b in payload]
    if not all(math.isfinite(c) for c in coefficients):
        raise ValueError("NaN E4M3 payload is not a valid TACO packet")
    restored = hadamard_fp64([c * quant for c in coefficients])
    return [bf16_round(v / adaptive) for v in restored]


def packet_bytes(elements: int) -> int:
    if type(elements) is not int or elements <= 0 or elements % GROUP_SIZE:
        raise ValueError("element count must be a positive multiple of 128")
    return elements // GROUP_SIZE * GROUP_BYTES


def encode(values) -> bytes:
    values = list(values)
    if not values or len(values) % GROUP_SIZE:
        raise ValueError("encoding needs a positive multiple of 128 values")
    groups = [encode_group(values[i:i + GROUP_SIZE]) for i in range(0, len(values), GROUP_SIZE)]
    count = len(groups)
    return (b"".join(g[0] for g in groups) + struct.pack(f"<{count}f", *(g[1] for g in groups))
            + struct.pack(f"<{count}f", *(g[2] for g in groups)))


def decode(packet) -> list:
    packet = bytes(packet)
    if not packet or len(packet) % GROUP_BYTES:
        raise ValueError("a packet holds exactly 136 bytes per 128-element group")
    count = len(packet) // GROUP_BYTES
    elements = count * GROUP_SIZE
    quant = struct.unpack_from(f"<{count}f", packet, elements)
    adaptive = struct.unpack_from(f"<{count}f", packet, elements + 4 * count)
    out = []
    for g in range(count):
        out.extend(decode_group(packet[g * GROUP_SIZE:(g + 1) * GROUP_SIZE], quant[g], adaptive[g]))
    return out


def reduce_sources(local, remote, rank: int, world: int) -> list:
    """Ordered BF16 reduction; `remote` lists the W-1 other sources ascending."""
    if type(rank) is not int or type(world) is not int or not 2 <= world <= 128 \
            or not 0 <= rank < world:
        raise ValueError("invalid rank/world")
    local = [bf16_round(v) for v in local]
    remote = [[bf16_round(v) for v in row] for row in remote]
    if not local or len(remote) != world - 1 or any(len(r) != len(local) for r in remote):
        raise ValueError("expected world-1 remote sources of the local size")
    if not all(math.isfinite(v) for row in [local, *remote] for v in row):
        raise ValueError("the reduction oracle needs finite inputs")
    ordered = remote[:rank] + [local] + remote[rank:]
    acc = [0.0] * len(local)
    for source in ordered:
        acc = [bf16_round(fp32(a + v)) for a, v in zip(acc, source)]
    return acc


def relative_l2(actual, expected) -> float:
    actual, expected = list(actual), list(expected)
    if len(actual) != len(expected) or not actual:
        raise ValueError("expected equal non-empty vectors")
    if not all(math.isfinite(float(x)) for x in actual + expected):
        return math.inf
    num = math.fsum((a - b) ** 2 for a, b in zip(actual, expected))
    den = math.fsum(b * b for b in expected)
    if den == 0:
        return 0.0 if num == 0 else math.inf
    return math.sqrt(num / den)
