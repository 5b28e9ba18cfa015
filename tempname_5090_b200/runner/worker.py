"""One torchrun window (one process per GPU): preflight | calibrate | operator | train.

    python -m torch.distributed.run --standalone --nnodes=1 --nproc-per-node W \\
        -m tempname_5090_b200.runner.worker --config CONFIG.json --out DIR --stage S --arm A

Every rank writes `DIR/rank{r}.json` atomically (also on failure, with the
traceback).  GPU checks precede every recorded number; every time is a CUDA
event interval on the launching stream, MAX over ranks.  Stages follow
TempName-5090 python/flux_5090/worker.py:95-335.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import os
import platform
import socket
import subprocess
import time
import traceback
from pathlib import Path

from . import protocol as P


def _peaks():
    """Roofline denominators: MEASURED_PEAKS.json when present, else the pool fallback."""
    root = Path(__file__).resolve().parents[2]
    try:
        data = json.loads((root / "MEASURED_PEAKS.json").read_text())
        return dict(bf16_tflops=float(data["bf16_tflops"]), hbm_gbs=float(data["hbm_gbs"]),
                    nvlink_gbs=770.0, source="measured")
    except (OSError, ValueError, KeyError):
        return dict(bf16_tflops=1590.0, hbm_gbs=6650.0, nvlink_gbs=770.0, source="fallback")


def tensor_sha(t) -> str:
    import torch
    return hashlib.sha256(t.detach().contiguous().view(-1).view(torch.uint8).cpu().numpy().tobytes()).hexdigest()


def identity(local_rank: int) -> dict:
    import torch
    p = torch.cuda.get_device_properties(local_rank)
    return dict(host=socket.gethostname(), device_name=p.name, sm_count=p.multi_processor_count,
                total_memory=p.total_memory, capability=list(torch.cuda.get_device_capability(local_rank)),
                torch=torch.__version__, cuda=torch.version.cuda, python=platform.python_version(),
                nccl_env={k: v for k, v in sorted(os.environ.items()) if k.startswith("NCCL_")})


def _timed(fn, warmup: int, iterations: int, group) -> float:
    """Mean seconds per call of fn(), CUDA events, MAX over ranks."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier(group=group)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(iterations):
        fn()
    end.record()
    torch.cuda.synchronize()
    t = torch.tensor(start.elapsed_time(end) / 1000.0 / iterations, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


# ------------------------------------------------------------------ preflight
def preflight(config: dict, rank: int, world: int, group) -> dict:
    import torch
    import torch.distributed as dist
    from .._native import lib, status_tensor
    from ..ops import gemm as G, taco
    from ..utils import reference as ref
    from .validation import relative_error, require_all
    checks = {}
    # tcgen05 GEMM vs a float64 host product
    a = (torch.arange(128 * 64, device="cuda", dtype=torch.float32).reshape(128, 64) % 7 / 8).to(torch.bfloat16)
    b = (torch.arange(256 * 64, device="cuda", dtype=torch.float32).reshape(256, 64) % 5 / 4).to(torch.bfloat16)
    exact = (a.double().cpu() @ b.double().cpu().t()).to(torch.bfloat16).cuda()
    checks["tcgen05_gemm"] = relative_error(G.matmul(a, b), exact) < 1e-2
    # NCCL probes on the group: all_reduce, all_gather, reduce_scatter, all_to_all
    v = torch.full((world * 4,), rank + 1, dtype=torch.bfloat16, device="cuda")
    out = torch.empty(4, dtype=torch.bfloat16, device="cuda")
    dist.reduce_scatter_tensor(out, v, group=group)
    checks["nccl_reduce_scatter"] = bool(torch.equal(out, torch.full_like(out, world * (world + 1) // 2)))
    gathered = torch.empty(world, dtype=torch.int32, device="cuda")
    dist.all_gather_into_tensor(gathered, torch.tensor([rank], dtype=torch.int32, device="cuda"), group=group)
    checks["nccl_all_gather"] = gathered.cpu().tolist() == list(range(world))
    send = torch.arange(world, dtype=torch.int32, device="cuda") + 100 * rank
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    checks["nccl_all_to_all"] = recv.cpu().tolist() == [100 * s + rank for s in range(world)]
    # peer access matrix (NVLink P2P for the symmetric-memory path)
    peer = [bool(torch.cuda.can_device_access_peer(torch.cuda.current_device(), o)) if o != torch.cuda.current_device()
            else True for o in range(torch.cuda.device_count())]
    checks["peer_access"] = all(peer[:world]) if world > 1 else True
    # symmetric-memory ping: a small fused GemmRS vs the independent reference
    if world > 1:
        from ..parallel.gemm_rs import GemmRS
        from .validation import projection_reference
        m, n, k = world * 256, 512, 256
        g = torch.Generator(device="cuda").manual_seed(rank)
        x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
        w = (0.05 * torch.randn((n, k), generator=g, device="cuda")).to(torch.bfloat16)
        op = GemmRS(m, n, k, group, timeout_ns=2_000_000_000)
        y = op.forward(x, w)
        plain, _ = projection_reference(x, w, rank, world, group, quantized=False)
        checks["symmetric_gemm_rs"] = relative_error(y, plain) < 1e-2
        op.close()
    # bounded wait: a flag nothing sets must time out with status 5 and leave the context usable
    flag = torch.zeros(4, dtype=torch.int32, device="cuda")
    st = status_tensor("cuda")
    st.zero_()
    lib().wait_probe(flag.data_ptr(), 1, 100_000_000, st)
    torch.cuda.synchronize()
    checks["bounded_wait_probe"] = int(st[0].item()) == 5
    st.zero_()
    # codec vs the stdlib oracle
    gen = torch.Generator(device="cuda").manual_seed(9871)
    xs = torch.randn(256, generator=gen, device="cuda").to(torch.bfloat16)
    pk = taco.encode(xs)
    dec = taco.decode(pk, 256)
    oracle = ref.decode(bytes(pk.cpu().tolist()))
    checks["taco_codec"] = ref.relative_l2(dec.float().cpu().tolist(), oracle) <= 0.01
    smi = None
    if rank == 0:
        try:
            smi = subprocess.run(["nvidia-smi", "topo", "-m"], capture_output=True, text=True, timeout=20).stdout
        except (OSError, subprocess.TimeoutExpired) as exc:
            smi = str(exc)
    require_all(all(checks.values()), f"preflight failed: {checks}", group)
    return dict(checks=checks, peer_access=peer, nvidia_smi_topology=smi)


# ------------------------------------------------------------------- operator
def operators(config: dict, arm: str, rank: int, world: int, group) -> dict:
    import torch
    from ..ops import gemm as G
    from ..parallel.gemm_rs import GemmRS
    from .validation import projection_reference, relative_error, require_all, validate_operator_buffers
    model, timing = config["model"], config["timing"]
    m, n = model["sequence"] * model["micro_batch"], model["hidden"]
    peaks = _peaks()
    results = []
    for role, k in (("attn", model["hidden"] // world), ("mlp", model["ffn"] // world)):
        g = torch.Generator(device="cuda").manual_seed(config["seed"] + 173 * rank + k)
        x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
        w = (torch.randn((n, k), generator=g, device="cuda") / math.sqrt(k)).to(torch.bfloat16)
        plan = config["execution_plan"]["roles"][role] if arm == P.ARRIVAL else None
        op = GemmRS(m, n, k, group, arm=arm, chunk_rows=model["chunk_rows"], plan=plan,
                    transport=config.get("transport", "nvlink"))
        out = op.forward(x, w)
        validate_operator_buffers(op, out)
        plain, indep = projection_reference(x, w, rank, world, group, quantized=arm != "flux")
        e_plain, e_codec = relative_error(out, plain), relative_error(out, indep)
        require_all(e_plain <= (0.05 if arm != "flux" else 0.01) and e_codec <= 0.01,
                    f"{role}: reference gate failed (bf16 {e_plain:.4g}, codec {e_codec:.4g})", group)
        retained = out.clone()
        x2 = (x * 0.75 + 0.125).to(torch.bfloat16)
        changed = op.forward(x2, w)
        _, indep2 = projection_reference(x2, w, rank, world, group, quantized=arm != "flux")
        require_all(torch.equal(out, retained) and relative_error(changed, indep2) <= 0.01,
                    f"{role}: output lifetime / changed-input reuse failed", group)
        bitwise = None
        if arm != "flux":
            other = "flux_taco" if arm == "flux_taco_interleaved" else "flux_taco_interleaved"
            sibling = GemmRS(m, n, k, group, arm=other, chunk_rows=model["chunk_rows"],
                             transport=config.get("transport", "nvlink"))
            bitwise = bool(torch.equal(sibling.forward(x, w), retained))
            require_all(bitwise, f"{role}: order-only sibling arm output differs", group)
            sibling.close()
        diagnostic = arrival_diagnostic(op, x, w, retained, group) if arm == P.ARRIVAL else None
        seconds = _timed(lambda: op.forward(x, w), timing["operator_warmup"], timing["operator_iterations"], group)
        full = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
        gemm_only = _timed(lambda: G.matmul(x, w, out=full), 5, timing["operator_iterations"], group)
        flops = 2.0 * m * n * k
        wire = (world - 1) * (m // world) * n * (136 / 128 if arm != "flux" else 2.0)
        roof = max(flops / (peaks["bf16_tflops"] * 1e12), wire / (peaks["nvlink_gbs"] * 1e9))
        results.append(dict(role=role, us_per_call=seconds * 1e6, timed_iterations=timing["operator_iterations"],
                            correctness_passed=True, bf16_relative_l2=e_plain, codec_reference_relative_l2=e_codec,
                            order_bitwise_equal=bitwise, gemm_only_us=gemm_only * 1e6,
                            roofline_us=roof * 1e6, roofline_fraction=roof / seconds, peaks=peaks,
                            arrival_diagnostic=diagnostic, execution=op.state()))
        op.close()
    return dict(operator_results=results)


def arrival_diagnostic(op, x, w, expected, group, delay_ns: int = 20_000_000) -> dict:
    """Artificial lane skew (never timed): rank 0 delays the flag of its first
    lane-0 tile by a bounded 20 ms; each owner records per-tile completion
    times of its arrival-first receiver.  Evidence of bypass = tiles of the
    other lane, later in the consumption order, finished before the delayed tile.
    Output must stay bitwise equal (arithmetic order never depends on arrival)."""
    import torch
    import torch.distributed as dist
    from .validation import require_all
    out, stamps, delayed = op.profile_call(x, w, delay_ns=delay_ns, delay_rank=0)
    require_all(bool(torch.equal(out, expected)), "artificial lane skew changed the output", group)
    result = dict(passed=True, artificial=True, delayed_rank=0, delay_ns=delay_ns, ordinary_speedup_claim=False)
    if delayed is not None and delayed[0] == op.rank:
        tile = delayed[1]
        order = op.consumer_order.tolist()
        pos = order.index(tile)
        tiles_n = op.n // 256
        lane_of = lambda t: ((t // tiles_n) * 128 // op.chunk_rows) % 2
        overtakes = [t for t in order[pos + 1:] if lane_of(t) != lane_of(tile) and stamps[t] < stamps[tile]]
        result.update(owner=True, delayed_tile=tile, later_other_lane_tiles_completed_before=overtakes,
                      ready_bypass_observed=bool(overtakes))
    else:
        result.update(owner=False)
    return result


# ---------------------------------------------------------------------- train
def train(config: dict, arm: str, rank: int, world: int, group, out_dir=None) -> dict:
    import torch
    from ..config import parameter_counts
    from ..models.gpt import GPT
    from ..models.train import Trainer
    model_cfg, timing = config["model"], config["timing"]
    model = GPT(model_cfg, arm=arm, group=group, device="cuda", seed=config["seed"],
                transport=config.get("transport", "nvlink"), execution_plan=config.get("execution_plan"))
    trainer = Trainer(model)
    c = model.config
    gen = torch.Generator().manual_seed(config["token_seed"])
    host = []
    for _ in range(c["accumulation_steps"]):
        stream = torch.randint(0, c["vocab"], (c["micro_batch"], c["sequence"] + 1), generator=gen)
        host.append((stream[:, :-1].reshape(-1).contiguous(), stream[:, 1:].reshape(-1).contiguous()))
    input_sha = hashlib.sha256(b"".join(t.numpy().tobytes() + l.numpy().tobytes() for t, l in host)).hexdigest()
    init_sha = tensor_sha(model.store.flat)
    batches = [(t.cuda(), l.cuda()) for t, l in host]
    for _ in range(timing["warmup_steps"]):
        trainer.step_host(batches)
    torch.cuda.reset_peak_memory_stats()
    losses, norms, ms = [], [], []
    for _ in range(timing["timed_steps"]):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        loss, norm2 = trainer.step(batches)
        end.record()
        vals = torch.stack([loss.double(), norm2]).cpu()
        losses.append(float(vals[0]))
        norms.append(math.sqrt(float(vals[1])))
        ms.append(start.elapsed_time(end))
    t = torch.tensor(sum(ms) / len(ms), dtype=torch.float64, device="cuda")
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    trace = None
    if config.get("profile") and out_dir is not None:
        # One extra, untimed step under the profiler with the named scopes on.
        from ..utils import tracing
        acts = [torch.profiler.ProfilerActivity.CPU, torch.profiler.ProfilerActivity.CUDA]
        with tracing.enabled(), torch.profiler.profile(activities=acts) as prof:
            trainer.step(batches)
            torch.cuda.synchronize()
        path, sha = tracing.export(prof, Path(out_dir) / f"trace_rank{rank}.json")
        trace = dict(path=Path(path).name, sha256=sha, untimed=True)
    counts = parameter_counts(c, world)
    row = dict(trace=trace, timed_steps=timing["timed_steps"], warmup_steps=timing["warmup_steps"], step_ms=float(t.item()),
               losses=losses, grad_norms=norms, tokens_per_step=c["sequence"] * c["micro_batch"] * c["accumulation_steps"],
               initialization_sha256=init_sha, input_sha256=input_sha, final_parameters_sha256=tensor_sha(model.store.flat),
               parameters_per_rank=counts["parameters_per_rank"], parameter_counts=counts, dtype="bfloat16",
               optimizer="AdamW-fp32-master", memory=dict(peak_allocated_bytes=torch.cuda.max_memory_allocated(),
                                                          peak_reserved_bytes=torch.cuda.max_memory_reserved()))
    model.close()
    return row


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--config", type=Path, required=True)
    ap.add_argument("--out", type=Path, required=True)
    ap.add_argument("--stage", choices=("preflight", "calibrate", "operator", "train"), required=True)
    ap.add_argument("--arm", choices=P.ARMS, required=True)
    args = ap.parse_args(argv)
    config = json.loads(args.config.read_text())
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    row = dict(rank=rank, world_size=world, stage=args.stage, arm=args.arm, run_id=config["run_id"],
               completed=False, passed=False, execution_plan_sha256=config.get("execution_plan_sha256"))
    try:
        import torch
        import torch.distributed as dist
        from datetime import timedelta
        if world != config["world_size"]:
            raise ValueError("torchrun world size differs from the frozen config")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
        group = dist.group.WORLD
        row["environment_identity"] = identity(local)
        if args.stage in ("operator", "train") and world > 1:
            P.validate_execution_plan(config["execution_plan"], config)
        if args.stage == "preflight":
            row.update(preflight(config, rank, world, group))
        elif args.stage == "calibrate":
            from .calibration import calibrate
            row.update(calibrate(config, group, args.out))
        elif args.stage == "operator":
            row.update(operators(config, args.arm, rank, world, group))
        else:
            row.update(train(config, args.arm, rank, world, group, args.out))
        torch.cuda.synchronize()
        row.update(completed=True, passed=True)
        P.write(args.out / f"rank{rank}.json", row)
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:
        row.update(completed=False, passed=False, error=str(exc), traceback=traceback.format_exc())
        P.write(args.out / f"rank{rank}.json", row)
        raise


if __name__ == "__main__":
    main()
