"""Untimed correctness gates (rank-coordinated) and independent references.

* `validate_packet_bytes` (stdlib) / `packet_tensor_valid` (device boolean):
  exact SoA size, finite E4M3 payload, scales in range.
* `validate_operator_buffers`: after a fused GemmRS call, every tile flag of
  every source equals the call's epoch, the device's read-back of the tile map
  equals the host's production order (mapping probe), the output is finite
  and the device status word is clear -- MIN-reduced over ranks so all ranks
  fail together.
* `projection_reference`: an independent GemmRS result built from a library
  GEMM (test oracle only), a dense all_to_all and the ordered BF16 sum, plus
  the same with an independent FP32 torch statement of the TACO codec.
Follows TempName-5090 python/flux_5090/validation.py and worker.py:153-204.
"""
from __future__ import annotations

import math
import struct


def _fp32(v):
    return struct.unpack("<f", struct.pack("<f", v))[0]


def validate_packet_bytes(packet, elements: int) -> dict:
    packet = bytes(packet)
    if type(elements) is not int or elements <= 0 or elements % 128:
        raise ValueError("packet element count must be a positive multiple of 128")
    groups = elements // 128
    if len(packet) != groups * 136:
        raise ValueError("wrong TACO packet size")
    if any(b & 127 == 127 for b in packet[:elements]):
        raise ValueError("non-finite E4M3 payload")
    quant = struct.unpack_from(f"<{groups}f", packet, elements)
    adaptive = struct.unpack_from(f"<{groups}f", packet, elements + 4 * groups)
    if not all(math.isfinite(v) and _fp32(1e-12) <= v <= _fp32(1e6) for v in quant):
        raise ValueError("invalid quantisation scales")
    if not all(math.isfinite(v) and _fp32(1e-3) <= v <= _fp32(1e3) for v in adaptive):
        raise ValueError("invalid adaptive scales")
    return dict(passed=True, elements=elements, groups=groups, bytes=len(packet))


def packet_tensor_valid(packet, elements: int):
    import torch
    groups = elements // 128
    if (packet.dtype != torch.uint8 or not packet.is_contiguous() or packet.numel() != groups * 136
            or elements % 128):
        raise ValueError("expected a contiguous uint8 TACO packet")
    flat = packet.view(-1)
    quant = flat[elements:elements + 4 * groups].view(torch.float32)
    adaptive = flat[elements + 4 * groups:].view(torch.float32)
    ok = torch.bitwise_and(flat[:elements], 127).ne(127).all()
    ok = ok & (torch.isfinite(quant) & (quant >= _fp32(1e-12)) & (quant <= _fp32(1e6))).all()
    ok = ok & (torch.isfinite(adaptive) & (adaptive >= _fp32(1e-3)) & (adaptive <= _fp32(1e3))).all()
    return ok


def require_all(ok: bool, message: str, group=None) -> None:
    import torch
    import torch.distributed as dist
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=group)
    if int(flag.item()) != 1:
        raise RuntimeError(message + " (failed on at least one rank)")


def relative_error(actual, expected) -> float:
    import torch
    if not bool(torch.isfinite(actual).all() and torch.isfinite(expected).all()):
        return float("inf")
    diff = torch.linalg.vector_norm(actual.float() - expected.float()).item()
    norm = torch.linalg.vector_norm(expected.float()).item()
    return diff / max(norm, 1e-12)


def validate_operator_buffers(op, output) -> dict:
    """Untimed, rank-coordinated gate after a fused GemmRS call."""
    import torch
    from .._native import status_tensor
    torch.cuda.synchronize()
    good = bool(torch.isfinite(output).all())
    detail = []
    if op.transport == "nvlink":
        flags = op.published_flags()
        if not bool((flags == op.epoch).all()):
            good = False
            detail.append("tile flags do not all equal the call epoch")
        # Mapping probe: the device decodes the uploaded production table into
        # exactly the host's tile order (reference validation.py:96-100).
        if op.device_tile_map() != op.host_tile_map():
            good = False
            detail.append("device tile map differs from the host production order")
    if int(status_tensor(output.device)[0].item()) != 0:
        good = False
        detail.append("device status word set")
    require_all(good, "operator buffer/publication validation failed: " + "; ".join(detail), op.group)
    return dict(passed=True, tiles_checked=op.world * (op.flag_tiles if op.pull else op.tiles_per_dest),
                mapping_probe=True,
                scope="untimed, rank-coordinated")


def projection_reference(x, w, rank: int, world: int, group, quantized: bool):
    """(plain ordered BF16 result, result with remote sources through an independent codec)."""
    import torch
    import torch.distributed as dist
    from ..ops import taco
    partial = torch.mm(x, w.t()).contiguous()  # library GEMM: test oracle only
    sources = torch.empty_like(partial)
    dist.all_to_all_single(sources.view(-1), partial.view(-1), group=group)
    sources = sources.view(world, partial.shape[0] // world, partial.shape[1])
    plain = torch.zeros_like(sources[0], dtype=torch.float32)
    indep = torch.zeros_like(plain)
    for s in range(world):
        plain = (plain + sources[s].float()).to(torch.bfloat16).float()
        contrib = sources[s]
        if quantized and s != rank:
            contrib = taco.decode_cpu(taco.encode_cpu(contrib), contrib.numel()).reshape(contrib.shape)
        indep = (indep + contrib.float()).to(torch.bfloat16).float()
    return plain.to(torch.bfloat16), indep.to(torch.bfloat16)


def fused_operator_check(m: int, hidden: int, ffn: int, group=None, seed: int = 11) -> dict:
    """Untimed bitwise check of the fused NVLink operators at a layer's shapes,
    MIN-reduced over ranks (every rank reports the same verdict):

    * AG->GEMM (FC1 shape: gather [M/W, h] shards, times W_fc1 [f/W, h]^T) against
      NCCL all_gather_into_tensor + this framework's GEMM of the same tile kind;
    * GemmRS (attention out-projection: [M, h/W] x [h, h/W]^T, residual + bias)
      against a dense all_to_all of the partials + the ordered BF16 reduction.
    """
    import torch
    import torch.distributed as dist
    from ..ops import gemm as G
    from ..ops import taco
    from .._native import check_status
    from ..parallel.ag_gemm import AGGemm
    from ..parallel.gemm_rs import GemmRS
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    rows = m // world
    g = torch.Generator(device="cuda").manual_seed(seed + 131 * rank)
    result = dict(world=world, ag_shape=[m, hidden, ffn // world], rs_shape=[m, hidden, hidden // world])
    # AG -> GEMM
    shard = torch.randn((rows, hidden), generator=g, device="cuda").to(torch.bfloat16)
    w1 = (0.02 * torch.randn((ffn // world, hidden), generator=g, device="cuda")).to(torch.bfloat16)
    ag = AGGemm(m, hidden, group)
    try:
        got = ag.forward(shard, w1)
        full = torch.empty((m, hidden), dtype=torch.bfloat16, device="cuda")
        dist.all_gather_into_tensor(full, shard, group=group)
        kind = ag.tile_kind(ffn // world, 256)
        want = G.matmul(full, w1, bn=256, pair=kind)
        torch.cuda.synchronize()
        check_status()  # a timed-out device wait raises with its code instead of reading as a mismatch
        ag_ok = bool(torch.equal(ag.gathered, full)) and bool(torch.equal(got, want))
        result["ag_tile_kind"] = kind
    finally:
        ag.close()
    # GEMM -> RS with residual + bias
    k = hidden // world
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w2 = (0.02 * torch.randn((hidden, k), generator=g, device="cuda")).to(torch.bfloat16)
    res = torch.randn((rows, hidden), generator=g, device="cuda").to(torch.bfloat16)
    bias = torch.randn((hidden,), generator=g, device="cuda").to(torch.bfloat16)
    rs = GemmRS(m, hidden, k, group)
    try:
        got = rs.forward(x, w2, residual=res, bias=bias)
        partial = G.matmul(x, w2, bn=256, pair=rs.tile_kind)
        sources = torch.empty_like(partial)
        dist.all_to_all_single(sources, partial, group=group)
        sources = sources.view(world, rows, hidden)
        remote = torch.cat([sources[s] for s in range(world) if s != rank])
        y = taco.ordered_reduce(sources[rank].contiguous(), remote, rank, world)
        want = ((res.float() + y.float()).to(torch.bfloat16).float() + bias.float()).to(torch.bfloat16)
        torch.cuda.synchronize()
        check_status()
        rs_ok = bool(torch.equal(got, want))
        result["rs_tile_kind"] = rs.tile_kind
        result["rs_transport"] = "nvlink-pull" if rs.pull else "nvlink-push"
    finally:
        rs.close()
    flags = torch.tensor([int(ag_ok), int(rs_ok)], dtype=torch.int32, device="cuda")
    dist.all_reduce(flags, op=dist.ReduceOp.MIN, group=group)
    result["ag_bitwise_all_ranks"] = bool(flags[0].item())
    result["rs_bitwise_all_ranks"] = bool(flags[1].item())
    return result
