"""TACO H128/E4M3 codec operators.

CUDA tensors run the native sm_100a kernels (byte-identical to the reference
codec, TempName-5090 src/taco/codec.cu).  CPU tensors run a torch FP32
statement of the same arithmetic, used by CPU tests and oracles.
"""
from __future__ import annotations

import math

import torch

from .._native import count_launch, lib

GROUP = 128
GROUP_BYTES = 136


def packet_bytes(elements: int) -> int:
    if elements <= 0 or elements % GROUP:
        raise ValueError("element count must be a positive multiple of 128")
    return elements // GROUP * GROUP_BYTES


def _hadamard(x: torch.Tensor) -> torch.Tensor:
    """Unnormalised Walsh-Hadamard over the last dim (128), butterfly distances 1..64."""
    shape = x.shape
    for d in (1, 2, 4, 8, 16, 32, 64):
        v = x.reshape(-1, GROUP // (2 * d), 2, d)
        lo, hi = v[:, :, 0], v[:, :, 1]
        x = torch.stack((lo + hi, lo - hi), dim=2).reshape(shape)
    return x


def _e4m3_levels(device):
    from ..utils.reference import e4m3_decode
    return torch.tensor([e4m3_decode(c) for c in range(127)], dtype=torch.float32, device=device)


def _quantize_e4m3(x: torch.Tensor) -> torch.Tensor:
    """FP32 -> E4M3FN codes (saturating, nearest, ties to even code), uint8."""
    levels = _e4m3_levels(x.device)
    mag = x.abs().clamp(max=448.0).contiguous()
    upper = torch.bucketize(mag, levels).clamp(0, 126)
    lower = (upper - 1).clamp(min=0)
    below = mag - levels[lower]
    above = levels[upper] - mag
    pick_upper = (above < below) | ((above == below) & (upper % 2 == 0))
    code = torch.where(pick_upper, upper, lower)
    code = torch.where(mag == 0, torch.zeros_like(code), code)
    sign = (torch.signbit(x)).to(torch.int64) * 128
    return (code + sign).to(torch.uint8)


def _dequantize_e4m3(codes: torch.Tensor) -> torch.Tensor:
    from ..utils.reference import e4m3_decode
    table = torch.tensor([e4m3_decode(c) for c in range(256)], dtype=torch.float32, device=codes.device)
    return table[codes.long()]


def encode_cpu(x: torch.Tensor) -> torch.Tensor:
    g = x.reshape(-1, GROUP).to(torch.bfloat16).float()
    variance = (g * g).sum(1, keepdim=True) / 128.0 + 1e-6
    adaptive = (448.0 * torch.rsqrt(variance.clamp_min(1e-12))).clamp(1e-3, 1e3)
    z = _hadamard(g * adaptive) * 0.08838834764831844055
    quant = (z.abs().amax(1, keepdim=True) / 448.0).clamp(1e-12, 1e6)
    codes = _quantize_e4m3(z / quant)
    return torch.cat([codes.reshape(-1), quant.reshape(-1).view(torch.uint8),
                      adaptive.reshape(-1).view(torch.uint8)])


def decode_cpu(packet: torch.Tensor, elements: int) -> torch.Tensor:
    groups = elements // GROUP
    codes = packet[:elements].reshape(groups, GROUP)
    quant = packet[elements:elements + 4 * groups].view(torch.float32).reshape(groups, 1)
    adaptive = packet[elements + 4 * groups:].view(torch.float32).reshape(groups, 1)
    z = _hadamard(_dequantize_e4m3(codes) * quant) * 0.08838834764831844055
    return (z / adaptive).to(torch.bfloat16).reshape(-1)


def encode(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    x = x.contiguous()
    n = x.numel()
    if out is None:
        out = torch.empty(packet_bytes(n), dtype=torch.uint8, device=x.device)
    if x.is_cuda:
        lib().taco_encode(x.view(-1), out)
        count_launch()
    else:
        out.copy_(encode_cpu(x))
    return out


def decode(packet: torch.Tensor, elements: int, out: torch.Tensor | None = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(elements, dtype=torch.bfloat16, device=packet.device)
    if packet.is_cuda:
        lib().taco_decode(packet, out.view(-1))
        count_launch()
    else:
        out.view(-1).copy_(decode_cpu(packet, elements))
    return out


def ordered_sum_cpu(sources) -> torch.Tensor:
    acc = torch.zeros_like(sources[0], dtype=torch.float32)
    for s in sources:
        acc = (acc + s.float()).to(torch.bfloat16).float()
    return acc.to(torch.bfloat16)


def decode_reduce(local: torch.Tensor, packets: torch.Tensor, rank: int, world: int,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """Ordered sum over sources 0..W-1: own BF16 partial at `rank`, decoded packets elsewhere."""
    out = torch.empty_like(local) if out is None else out
    if local.is_cuda:
        lib().taco_decode_reduce(local.contiguous(), packets.contiguous(), out, rank, world)
        count_launch()
        return out
    n = local.numel()
    pb = packet_bytes(n)
    sources = []
    for s in range(world):
        if s == rank:
            sources.append(local.reshape(-1))
        else:
            slot = s - (s > rank)
            sources.append(decode_cpu(packets.reshape(-1)[slot * pb:(slot + 1) * pb], n))
    out.copy_(ordered_sum_cpu(sources).reshape(out.shape))
    return out


def ordered_reduce(local: torch.Tensor, remote: torch.Tensor, rank: int, world: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    out = torch.empty_like(local) if out is None else out
    if local.is_cuda:
        lib().ordered_reduce(local.contiguous(), remote.contiguous(), out, rank, world)
        count_launch()
        return out
    remote = remote.reshape(world - 1, -1)
    sources = [local.reshape(-1) if s == rank else remote[s - (s > rank)] for s in range(world)]
    out.copy_(ordered_sum_cpu(sources).reshape(out.shape))
    return out


def delay(cycles: int) -> None:
    """Bounded diagnostic delay kernel on the current stream (<= 1e8 cycles)."""
    if type(cycles) is not int or not 0 < cycles <= 100_000_000:
        raise ValueError("delay cycles must be in (0, 1e8]")
    lib().diagnostic_delay(cycles)
    count_launch()
