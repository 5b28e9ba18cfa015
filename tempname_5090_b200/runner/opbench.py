"""Operator benchmarks on one node (one process per GPU; launch with torchrun).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m tempname_5090_b200.runner.opbench --op gemmrs
    ... --op attention      # AG->GEMM QKV + causal attention + GemmRS out-proj (TP8, SP)
    ... --op sweep          # GemmRS N=4096, K=16384/TP, M in 2048..32768, bf16 vs TACO
    python -m tempname_5090_b200.runner.opbench --op gemm         # 1 GPU: tile kinds vs cuBLAS
    python -m tempname_5090_b200.runner.opbench --op gemm_once --kind 2   # one GEMM (profiler case)
    python -m tempname_5090_b200.runner.opbench --op attn_kernel  # 1 GPU: attention fwd/bwd kernels
    python -m tempname_5090_b200.runner.opbench --op fused_emulated --world 8   # 1 GPU: fused-op kernels, ranks emulated
    torchrun ... -m tempname_5090_b200.runner.opbench --op nvlink   # SM-issued peer stores vs local copy

Timing: every iteration is bracketed by CUDA events on the launching stream,
the L2 is flushed (a 256 MiB write) between iterations outside the events,
and the reported time is the MAX over ranks of the per-rank median.
Baselines on the same box: `nccl+cublas` (torch.mm + NCCL reduce_scatter /
all_gather + SDPA, the path that only calls libraries) and `transport=nccl`
(this framework's GEMM + the reference's per-block sparse all_to_all mechanism).
Roofline fraction = max(FLOPs / measured bf16 peak, NVLink bytes / 770 GB/s) / time.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


def peaks() -> dict:
    try:
        d = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return dict(bf16_tflops=float(d["bf16_tflops"]), nvlink_gbs=770.0, source="measured")
    except (OSError, ValueError, KeyError):
        return dict(bf16_tflops=1590.0, nvlink_gbs=770.0, source="fallback")


class Timer:
    def __init__(self, world, group=None):
        import torch
        self.torch = torch
        self.world, self.group = world, group
        self.flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")

    def run(self, fn, warmup=5, iterations=20) -> float:
        """Median microseconds per call, max over ranks."""
        torch = self.torch
        import torch.distributed as dist
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(iterations):
            self.flush.fill_(1.0)
            if self.world > 1:
                dist.barrier(group=self.group)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e) * 1000.0)
        med = torch.tensor(statistics.median(times), dtype=torch.float64, device="cuda")
        if self.world > 1:
            dist.all_reduce(med, op=dist.ReduceOp.MAX, group=self.group)
        return float(med.item())

    def back_to_back(self, fn, calls=10) -> float:
        """Microseconds per call of `calls` consecutive calls (no flush between:
        host launch gaps hide behind the previous call), max over ranks."""
        torch = self.torch
        import torch.distributed as dist
        fn()
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(calls):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor(s.elapsed_time(e) * 1000.0 / calls, dtype=torch.float64, device="cuda")
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())


def split_phases(op, x, w, timer, iterations=10) -> dict:
    """Pull GemmRS with its two halves as separate launches: the GEMM CTAs
    alone (partial tiles stored and published), then the reducer CTAs alone
    (median device times, max over ranks)."""
    import torch
    import torch.distributed as dist
    out = torch.empty((op.rows, op.n), dtype=torch.bfloat16, device="cuda")
    gemm, red = [], []
    for _ in range(iterations + 2):
        timer.flush.fill_(1.0)
        if op.world > 1:
            dist.barrier()
        e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        op.begin()
        e[0].record()
        op.push(x, w)
        e[1].record()
        op.reduce(out)
        e[2].record()
        torch.cuda.synchronize()
        gemm.append(e[0].elapsed_time(e[1]) * 1000)
        red.append(e[1].elapsed_time(e[2]) * 1000)
    t = torch.tensor([statistics.median(gemm[2:]), statistics.median(red[2:])], dtype=torch.float64, device="cuda")
    if op.world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return dict(gemm_phase_us=float(t[0]), reduce_phase_us=float(t[1]))


def gemmrs_case(m, n, k, rank, world, timer, arms, transports, with_library=True, chunk_rows=128,
                comm_sweep=(None,), kind_sweep=(None,)):
    import torch
    import torch.distributed as dist
    from ..parallel.gemm_rs import GemmRS
    from ..parallel import planning
    from ..ops import gemm as G
    from .._native import check_status
    pk = peaks()
    g = torch.Generator(device="cuda").manual_seed(17 + rank)
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn((n, k), generator=g, device="cuda")).to(torch.bfloat16)
    flops = 2.0 * m * n * k
    rows = []
    for arm in arms:
        plan = None
        if arm.endswith("arrival"):
            plan = planning.make_role(m, n, k, world, chunk_rows)
        for transport in transports:
            pull = transport == "nvlink" and arm == "flux"
            sweep = [(c, kind) for c in comm_sweep for kind in kind_sweep] if pull else [(None, None)]
            for comm, kind in sweep:
                op = GemmRS(m, n, k, arm=arm, chunk_rows=chunk_rows, plan=plan, transport=transport,
                            comm_ctas=comm, tile_kind=kind)
                us = timer.run(lambda: op.forward(x, w))
                wire = (world - 1) * (m // world) * n * (136 / 128 if arm != "flux" else 2.0)
                roof = max(flops / (pk["bf16_tflops"] * 1e12), wire / (pk["nvlink_gbs"] * 1e9)) * 1e6
                row = dict(op="gemmrs", arm=arm, transport=transport + ("-pull" if op.pull else ""), m=m, n=n,
                           k=k, world=world, us=us, roofline_us=roof, roofline_fraction=roof / us,
                           tflops=flops / us / 1e6, nvlink_bytes_per_rank=wire, peaks=pk["source"])
                row["back_to_back_us"] = timer.back_to_back(lambda: op.forward(x, w))
                if op.pull:
                    row.update(split_phases(op, x, w, timer))
                    row["comm_ctas"] = op.comm_ctas
                    row["tile_kind"] = op.tile_kind
                    prof = op.stage_profile(x, w)
                    row["stage"] = {key: prof[key] for key in ("producer_last_ns", "consumer_first_ns",
                                                                "consumer_last_ns", "consumer_tiles",
                                                                "consumer_tiles_completed_before_producer_end")}
                check_status()
                rows.append(row)
                op.close()
    # GEMM alone (no communication) and the library-only baseline
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    rows.append(dict(op="gemm_only", m=m, n=n, k=k, us=timer.run(lambda: G.matmul(x, w, out=out))))
    if with_library and world > 1:
        rs = torch.empty((m // world, n), dtype=torch.bfloat16, device="cuda")

        def library():
            full = torch.mm(x, w.t())
            dist.reduce_scatter_tensor(rs, full)
        rows.append(dict(op="gemmrs", arm="flux", transport="nccl+cublas", m=m, n=n, k=k, world=world,
                         us=timer.run(library)))
        rows.append(dict(op="cublas_gemm_only", m=m, n=n, k=k, us=timer.run(lambda: torch.mm(x, w.t(), out=out))))
    return rows


def attention_case(rank, world, timer, heads=32, hidden=4096, seq=2048, batch=4):
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F
    from ..parallel.tp import TensorParallel
    from ..ops import attention as A
    tp = TensorParallel(None)
    m = seq * batch
    lh = heads // world
    g = torch.Generator(device="cuda").manual_seed(5 + rank)
    xs = torch.randn((m // world, hidden), generator=g, device="cuda").to(torch.bfloat16)
    wqkv = (0.02 * torch.randn((3 * hidden // world, hidden), generator=g, device="cuda")).to(torch.bfloat16)
    bqkv = torch.zeros(3 * hidden // world, dtype=torch.bfloat16, device="cuda")
    wo = (0.02 * torch.randn((hidden, hidden // world), generator=g, device="cuda")).to(torch.bfloat16)
    bo = torch.zeros(hidden, dtype=torch.bfloat16, device="cuda")

    def ours():
        qkv, _ = tp.ag_linear(("bench_qkv", 0), xs, wqkv, bias=bqkv)
        attn, _ = A.forward(qkv, batch, seq, lh)
        return tp.linear_rs(attn, wo, residual=xs, bias=bo, role="attn")

    full = torch.empty((m, hidden), dtype=torch.bfloat16, device="cuda")
    rs = torch.empty((m // world, hidden), dtype=torch.bfloat16, device="cuda")

    def library():
        dist.all_gather_into_tensor(full, xs)
        qkv = F.linear(full, wqkv, bqkv)
        q, k, v = qkv.view(batch, seq, 3, lh, 128).permute(2, 0, 3, 1, 4).unbind(0)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(m, lh * 128)
        dist.reduce_scatter_tensor(rs, torch.mm(a, wo.t()))
        return rs

    flops = 2 * m * hidden * 3 * hidden / world + 4 * batch * lh * seq * seq * 128 / 2 + 2 * m * hidden * hidden / world
    rows = [dict(op="attention_block", impl="ours", world=world, us=timer.run(ours), flops=flops)]
    if world > 1:
        rows.append(dict(op="attention_block", impl="nccl+cublas+sdpa", world=world, us=timer.run(library), flops=flops))
    # Stage breakdown (each stage timed alone on the same inputs).
    qkv, _ = tp.ag_linear(("bench_qkv", 0), xs, wqkv, bias=bqkv)
    attn, _ = A.forward(qkv, batch, seq, lh)
    q, k, v = qkv.view(batch, seq, 3, lh, 128).permute(2, 0, 3, 1, 4).unbind(0)
    stages = dict(
        ag_gemm=lambda: tp.ag_linear(("bench_qkv", 0), xs, wqkv, bias=bqkv),
        attention=lambda: A.forward(qkv, batch, seq, lh, out=attn),
        gemm_rs=lambda: tp.linear_rs(attn, wo, residual=xs, bias=bo, role="attn"),
        lib_all_gather=lambda: dist.all_gather_into_tensor(full, xs) if world > 1 else None,
        lib_qkv_gemm=lambda: F.linear(full, wqkv, bqkv),
        lib_sdpa=lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True),
        lib_out_gemm=lambda: torch.mm(attn, wo.t()),
    )
    for name, fn in stages.items():
        rows.append(dict(op="attention_stage", stage=name, world=world, us=timer.run(fn),
                         back_to_back_us=timer.back_to_back(fn)))
    if world > 1:
        prof = tp.ag_operator(("bench_qkv", 0), m, hidden, 3 * hidden // world).stage_profile(xs, wqkv, bias=bqkv)
        rows.append(dict(op="stage_profile", stage="ag_gemm", world=world,
                         **{k: v for k, v in prof.items() if k != "out"}))
        prof = tp.rs_operator(m, hidden, hidden // world, "attn").stage_profile(attn, wo, residual=xs, bias=bo)
        rows.append(dict(op="stage_profile", stage="gemm_rs", world=world,
                         **{k: v for k, v in prof.items() if k not in ("out", "produced_ns", "consumed_ns")}))
    tp.close()
    return rows


GEMM_SHAPES = ((8192, 8192, 8192), (8192, 12288, 4096), (8192, 16384, 4096), (8192, 4096, 16384),
               (8192, 4096, 4096), (8192, 4096, 2048))


def gemm_case(shapes, timer):
    """Tile kinds (0 single CTA, 1 CTA pair, 2 wide pair, -1 auto) against cuBLAS,
    with the kernel's own cycle counters (MMA-role cycles and wait fractions).
    Kind "2u" is the wide tile without the tail split (a grid cap of all SMs
    turns the split off)."""
    import torch
    from ..ops.gemm import matmul
    from .._native import check_status, lib
    rows = []
    sms = lib().sm_count()
    for (m, n, k) in shapes:
        a = torch.randn((m, k), device="cuda").to(torch.bfloat16)
        b = torch.randn((n, k), device="cuda").to(torch.bfloat16)
        out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        ref = torch.mm(a, b.t())
        flops = 2.0 * m * n * k
        for kind in (0, 1, 2, "2u", -1):
            pair, cap = (2, sms) if kind == "2u" else (kind, 0)
            fn = (lambda pair=pair, cap=cap: matmul(a, b, out=out, bn=256 if pair else 0, pair=pair, max_ctas=cap))
            fn()
            torch.cuda.synchronize()
            check_status()
            exact = bool(torch.equal(out, ref))
            us = timer.run(fn)
            dbg = torch.zeros(148 * 8, dtype=torch.int64, device="cuda")
            matmul(a, b, out=out, bn=256 if pair else 0, pair=pair, max_ctas=cap, debug=dbg)
            torch.cuda.synchronize()
            d = dbg.view(-1, 8).double()
            lead = d[d[:, 1] > 0]
            rows.append(dict(op="gemm", kind=kind, m=m, n=n, k=k, us=us, tflops=flops / us / 1e6,
                             bitwise_equal_cublas=exact, mma_cycles=lead[:, 1].mean().item(),
                             mma_wait_data=(lead[:, 0] / lead[:, 1]).mean().item(),
                             mma_wait_accumulator=(lead[:, 4] / lead[:, 1]).mean().item()))
        us = timer.run(lambda: torch.mm(a, b.t(), out=out))
        rows.append(dict(op="gemm", kind="cublas", m=m, n=n, k=k, us=us, tflops=flops / us / 1e6))
    return rows


def gemm_once(m, n, k, kind):
    """Three launches of one GEMM (a small, self-ending case for a profiler)."""
    import torch
    from ..ops.gemm import matmul
    a = torch.randn((m, k), device="cuda").to(torch.bfloat16)
    b = torch.randn((n, k), device="cuda").to(torch.bfloat16)
    out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    for _ in range(3):
        if kind == "cublas":
            torch.mm(a, b.t(), out=out)
        else:
            matmul(a, b, out=out, bn=256 if int(kind) else 0, pair=int(kind))
    torch.cuda.synchronize()
    return [dict(op="gemm_once", kind=kind, m=m, n=n, k=k)]


def attention_once(B, S, H):
    """Three forward + backward calls at one shape (a small, self-ending case for a profiler)."""
    import torch
    from ..ops import attention as A
    qkv = torch.randn((B * S, 3 * H * 128), device="cuda").to(torch.bfloat16)
    dout = torch.randn((B * S, H * 128), device="cuda").to(torch.bfloat16)
    for _ in range(3):
        out, lse = A.forward(qkv, B, S, H)
        A.backward(qkv, out, dout, lse, B, S, H)
    torch.cuda.synchronize()
    return [dict(op="attn_once", B=B, S=S, H=H)]


def attention_kernel_case(timer, shapes=((4, 2048, 4), (1, 2048, 32), (4, 2048, 32))):
    """Causal attention kernels (head_dim 128) against an fp32 torch reference."""
    import torch
    import torch.nn.functional as F
    from ..ops import attention as A
    rows = []
    for (B, S, H) in shapes:
        d = 128
        qkv = torch.randn((B * S, 3 * H * d), device="cuda").to(torch.bfloat16)
        out, lse = A.forward(qkv, B, S, H)
        dout = torch.randn((B * S, H * d), device="cuda").to(torch.bfloat16)
        dqkv = A.backward(qkv, out, dout, lse, B, S, H)
        q, k, v = qkv.float().reshape(B, S, 3, H, d).permute(2, 0, 3, 1, 4).unbind(0)
        q.requires_grad_(True); k.requires_grad_(True); v.requires_grad_(True)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2).reshape(B * S, H * d)
        o.backward(dout.float())
        g = dqkv.float().reshape(B, S, 3, H, d).permute(2, 0, 3, 1, 4)
        rel = lambda x, y: ((x - y).norm() / y.norm()).item()
        again = A.backward(qkv, out, dout, lse, B, S, H)
        dbg = torch.zeros((2, B * H * (S // 128), 8), dtype=torch.int64, device="cuda")
        A.backward(qkv, out, dout, lse, B, S, H, debug=dbg)
        torch.cuda.synchronize()
        phases = {}
        for name, c in zip(("dkdv", "dq"), dbg.double().cpu()):
            blocks = c[:, 6].sum().item()
            mma = c[:, 3].sum().item()
            phases[name] = dict(mma_wait_tiles=c[:, 0].sum().item() / mma, mma_wait_elementwise=c[:, 1].sum().item() / mma,
                                mma_wait_prev_mma=c[:, 2].sum().item() / mma,
                                ew_wait_cycles_per_block=c[:, 4].sum().item() / blocks,
                                ew_work_cycles_per_block=c[:, 5].sum().item() / blocks,
                                mma_cycles_per_block=mma / blocks)
        flops = 4.0 * B * H * S * S * d / 2
        fwd_us = timer.run(lambda: A.forward(qkv, B, S, H, out=out))
        bwd_us = timer.run(lambda: A.backward(qkv, out, dout, lse, B, S, H, dqkv=dqkv))
        rows.append(dict(op="attention_kernel", B=B, S=S, H=H, fwd_us=fwd_us, bwd_us=bwd_us,
                         fwd_tflops=flops / fwd_us / 1e6, bwd_tflops=2.5 * flops / bwd_us / 1e6,
                         out_rel_err=rel(out.float(), o.detach()), dq_rel_err=rel(g[0], q.grad),
                         dk_rel_err=rel(g[1], k.grad), dv_rel_err=rel(g[2], v.grad),
                         backward_deterministic=bool(torch.equal(again, dqkv)), backward_phases=phases))
    return rows


def nvlink_case(rank, world, timer, mib=64):
    """NVLink transfer mechanisms, ring pattern (every rank moves `mib` MiB
    between itself and rank+1 at once), swept over the number of CTAs:

    * push:       SM-issued 16-byte stores into the peer's memory (copy kernel)
    * pull:       SM-issued 16-byte loads from the peer's memory, local stores
    * bulk_pull:  untiled bulk (TMA-engine) loads from the peer's memory into a
                  shared-memory ring, bulk stores to local memory; one issuing
                  thread per CTA, `stages` x `chunk` bytes in flight per CTA
    * local_copy / bulk_local: the same kernels on this GPU's memory only.
    """
    import torch
    from .._native import lib, status_tensor
    from ..parallel.symmetric import SymmetricBuffer
    nbytes = mib << 20
    buf = SymmetricBuffer(2 * nbytes)
    def data(r):
        return torch.randn(nbytes // 4, device="cuda", generator=torch.Generator(device="cuda").manual_seed(99 + r))
    src = data(rank)
    buf.local_view((nbytes // 4,), torch.float32).copy_(src)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    local_dst = torch.empty_like(src)
    peer = (rank + 1) % world
    peer_src = buf.peers[peer]                    # the peer's first half (its data)
    peer_dst = buf.peers[peer] + nbytes           # the peer's second half (landing zone)
    status = status_tensor(torch.device("cuda", torch.cuda.current_device()))
    C = lib()
    rows = []

    def row(pattern, fn, **kw):
        us = timer.run(fn)
        rows.append(dict(op="nvlink", pattern=pattern, world=world, bytes=nbytes, us=us,
                         gbs_per_rank=nbytes / us / 1e3, **kw))

    row("local_copy", lambda: C.copy_ptr(local_dst.data_ptr(), src.data_ptr(), nbytes, 0), ctas=4 * 148)
    for ctas in (32, 64, 148, 296, 592):
        row("push", lambda c=ctas: C.copy_ptr(peer_dst, src.data_ptr(), nbytes, c), ctas=ctas)
    for ctas in (32, 64, 148, 296, 592):
        row("pull", lambda c=ctas: C.copy_ptr(local_dst.data_ptr(), peer_src, nbytes, c), ctas=ctas)
    for chunk, stages in ((16384, 8), (32768, 6), (65536, 3)):
        for ctas in (8, 16, 24, 32, 48, 64, 148):
            row("bulk_pull", lambda c=ctas, k=chunk, s=stages: C.bulk_copy(local_dst.data_ptr(), peer_src, nbytes,
                                                                          c, k, s, 10 ** 9, status),
                ctas=ctas, chunk=chunk, stages=stages)
    for ctas in (16, 32, 148):
        row("bulk_local", lambda c=ctas: C.bulk_copy(local_dst.data_ptr(), src.data_ptr(), nbytes, c, 32768, 6,
                                                     10 ** 9, status), ctas=ctas, chunk=32768, stages=6)
    # Data check: one more bulk pull and one SM pull must reproduce the peer's data.
    local_dst.zero_()
    C.bulk_copy(local_dst.data_ptr(), peer_src, nbytes, 32, 32768, 6, 10 ** 9, status)
    torch.cuda.synchronize()
    expect = data(peer)
    bulk_ok = bool(torch.equal(local_dst, expect))
    local_dst.zero_()
    C.copy_ptr(local_dst.data_ptr(), peer_src, nbytes, 148)
    torch.cuda.synchronize()
    rows.append(dict(op="nvlink_check", status=int(status[0].item()), bulk_pull_equal=bulk_ok,
                     pull_equal=bool(torch.equal(local_dst, expect))))
    buf.close()
    return rows


def ag_gemm_case(rank, world, timer, m=8192, hidden=4096, ffn=16384):
    """AG->GEMM at the model's column-parallel shapes (QKV: N = 3h/W, FC1:
    N = f/W): the fused launch, its two halves launched separately (gather
    only -- the communication CTAs alone -- then the GEMM alone on the gathered
    data), the device stage profile, and the library path (NCCL all_gather +
    cuBLAS)."""
    import torch
    import torch.distributed as dist
    from ..parallel.ag_gemm import AGGemm
    from .._native import check_status
    rows = []
    g = torch.Generator(device="cuda").manual_seed(41 + rank)
    shard = torch.randn((m // world, hidden), generator=g, device="cuda").to(torch.bfloat16)
    for name, n in (("qkv", 3 * hidden // world), ("fc1", ffn // world)):
        op = AGGemm(m, hidden, n=n)
        w = (0.02 * torch.randn((n, hidden), generator=g, device="cuda")).to(torch.bfloat16)
        out = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        fused = timer.run(lambda: op.forward(shard, w, out=out))
        b2b = timer.back_to_back(lambda: op.forward(shard, w, out=out))
        gather = timer.run(lambda: op.forward(shard, w, out=out, phase=3))
        gemm = timer.run(lambda: op.forward(shard, w, out=out, phase=4))
        prof = op.stage_profile(shard, w, out=out)
        check_status()  # a timed-out wait would make every later wait return at once: fail here instead
        full = torch.empty((m, hidden), dtype=torch.bfloat16, device="cuda")
        lib_ag = timer.run(lambda: dist.all_gather_into_tensor(full, shard))
        lib_mm = timer.run(lambda: torch.mm(full, w.t(), out=out))
        rows.append(dict(op="ag_gemm", shape=name, m=m, n=n, k=hidden, world=world, fused_us=fused,
                         back_to_back_us=b2b, gather_only_us=gather, gemm_only_us=gemm,
                         library_all_gather_us=lib_ag, library_gemm_us=lib_mm, library_us=lib_ag + lib_mm,
                         tile_kind=op.tile_kind(n, 256), comm_ctas=op.comm_ctas,
                         gather_gbs=(world - 1) * (m // world) * hidden * 2 / gather / 1e3,
                         stage={k: v for k, v in prof.items() if k != "out"}))
        op.close()
    return rows


def fused_emulated_case(m, n, k, world, timer, repeats=3):
    """The fused operators' kernels with W ranks emulated on ONE GPU (every
    rank's buffers local; phases launched so that no launch waits on another):
    the pull GemmRS GEMM phase (partial tiles TMA-stored + flags published) and
    reducer phase (W sources pulled and reduced), and the AG->GEMM gather and
    GEMM phases.  A small, self-ending case for a profiler; the times are
    single-GPU (no NVLink), the kernels and their code paths are the real ones.
    Launch sequence per repeat (for a profiler's launch skip count): W GemmRS
    GEMM phases, W reducer phases; after all repeats, per repeat W AG own-chunk
    phases, W peer-pull phases, W AG GEMM phases."""
    import torch
    from ..parallel.gemm_rs import GemmRS
    from ..parallel.ag_gemm import AGGemm, control_layout
    from ..parallel.symmetric import SymmetricBuffer
    rows = m // world
    rows_out = []
    g = torch.Generator(device="cuda").manual_seed(3)
    data = [SymmetricBuffer.emulated(m * n * 2, world) for _ in range(2)]
    flags = SymmetricBuffer.emulated(world * (rows // 128) * (n // 256) * 4, world)
    ops = [GemmRS(m, n, k, _emulate=(r, world, [b.as_rank(r) for b in data], flags.as_rank(r)))
           for r in range(world)]
    xs = [torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16) for _ in range(world)]
    w = (0.02 * torch.randn((n, k), generator=g, device="cuda")).to(torch.bfloat16)
    out = torch.empty((rows, n), dtype=torch.bfloat16, device="cuda")
    events = lambda: (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    gemm_us, red_us = [], []
    for _ in range(repeats):
        for op in ops:
            op.begin()
        s, e = events()
        s.record()
        for r, op in enumerate(ops):
            op.push(xs[r], w)
        e.record()
        torch.cuda.synchronize()
        gemm_us.append(s.elapsed_time(e) * 1000 / world)
        s, e = events()
        s.record()
        for op in ops:
            op.reduce(out)
        e.record()
        torch.cuda.synchronize()
        red_us.append(s.elapsed_time(e) * 1000 / world)
    rows_out.append(dict(op="fused_emulated", stage="gemm_rs_pull_gemm_phase", m=m, n=n, k=k, world=world,
                         tile_kind=ops[0].tile_kind, comm_ctas=ops[0].comm_ctas, us_per_rank=min(gemm_us)))
    rows_out.append(dict(op="fused_emulated", stage="gemm_rs_pull_reduce_phase", world=world,
                         us_per_rank=min(red_us), bytes_per_rank=world * rows * n * 2))
    for b in data + [flags]:
        b.close()
    # AG -> GEMM: QKV shape of the attention block (K = n, N = 3 * n / W)
    kk, nn = n, 3 * n // world
    gather = SymmetricBuffer.emulated(m * kk * 2, world)
    pulled_off, ctrl_bytes = control_layout(m)
    ctrl = SymmetricBuffer.emulated(ctrl_bytes, world)
    ags = [AGGemm(m, kk, _emulate=(r, world, gather.as_rank(r), ctrl.as_rank(r))) for r in range(world)]
    shards = [torch.randn((rows, kk), generator=g, device="cuda").to(torch.bfloat16) for _ in range(world)]
    wq = (0.02 * torch.randn((nn, kk), generator=g, device="cuda")).to(torch.bfloat16)
    outs = torch.empty((m, nn), dtype=torch.bfloat16, device="cuda")
    ag_us = []
    for _ in range(repeats):
        for phase in (1, 2):
            for r in range(world):
                ags[r].forward(shards[r], wq, phase=phase)
        s, e = events()
        s.record()
        for r in range(world):
            ags[r].forward(shards[r], wq, phase=4, out=outs)
        e.record()
        torch.cuda.synchronize()
        ag_us.append(s.elapsed_time(e) * 1000 / world)
    rows_out.append(dict(op="fused_emulated", stage="ag_gemm_gemm_phase", m=m, n=nn, k=kk, world=world,
                         tile_kind=ags[0].tile_kind(nn, 256), us_per_rank=min(ag_us)))
    gather.close()
    ctrl.close()
    return rows_out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--op", choices=("gemmrs", "attention", "sweep", "gemm", "gemm_once", "attn_kernel", "attn_once",
                                     "nvlink", "fused_emulated", "ag_gemm"),
                    default="gemmrs")
    ap.add_argument("--kind", default="2", help="gemm_once: tile kind 0/1/2/-1 or 'cublas'")
    ap.add_argument("--heads", type=int, default=32, help="attn_once: heads (batch from --batch, length from --seq)")
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--k", type=int, default=2048)
    ap.add_argument("--arms", default="all")
    ap.add_argument("--transports", default="nvlink,nccl")
    ap.add_argument("--comm-ctas", default="", help="gemmrs: comma list of reducer CTA counts (pull transport)")
    ap.add_argument("--tile-kinds", default="", help="gemmrs: comma list of pull GEMM tile kinds (0 single, 2 wide)")
    ap.add_argument("--world", type=int, default=8, help="fused_emulated: emulated ranks on one GPU")
    ap.add_argument("--repeats", type=int, default=3, help="fused_emulated: calls per stage (1 for a profiler)")
    ap.add_argument("--out", type=Path)
    args = ap.parse_args(argv)
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    timer = Timer(world)
    from ..config import ARMS
    arms = ARMS if args.arms == "all" else tuple(args.arms.split(","))
    transports = tuple(args.transports.split(","))
    rows = []
    comm_sweep = tuple(int(c) for c in args.comm_ctas.split(",")) if args.comm_ctas else (None,)
    if args.op == "gemmrs":
        kinds = tuple(int(c) for c in args.tile_kinds.split(",")) if args.tile_kinds else (None,)
        rows += gemmrs_case(args.m, args.n, args.k, rank, world, timer, arms, transports, comm_sweep=comm_sweep,
                            kind_sweep=kinds)
    elif args.op == "gemm":
        rows += gemm_case(GEMM_SHAPES, timer)
    elif args.op == "gemm_once":
        rows += gemm_once(args.m, args.n, args.k, args.kind)
    elif args.op == "attn_once":
        rows += attention_once(args.batch, args.seq, args.heads)
    elif args.op == "attn_kernel":
        rows += attention_kernel_case(timer)
    elif args.op == "nvlink":
        rows += nvlink_case(rank, world, timer)
    elif args.op == "ag_gemm":
        rows += ag_gemm_case(rank, world, timer)
    elif args.op == "fused_emulated":
        rows += fused_emulated_case(args.m, args.n, args.k, args.world, timer, repeats=args.repeats)
    elif args.op == "attention":
        rows += attention_case(rank, world, timer)
    else:
        for m in (2048, 4096, 8192, 16384, 32768):
            chunk = 128 if m // world >= 128 else None
            if chunk is None:
                continue
            rows += gemmrs_case(m, 4096, 16384 // world, rank, world, timer, ("flux", "flux_taco"), ("nvlink",),
                                with_library=(m == 8192))
    if rank == 0:
        for r in rows:
            print(json.dumps(r), flush=True)
        if args.out:
            args.out.parent.mkdir(parents=True, exist_ok=True)
            args.out.write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
