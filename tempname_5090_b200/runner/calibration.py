"""Measured calibration of the arrival plans (one per role: attention out-proj
K=h/W and MLP down-proj K=f/W).

For every candidate plan, a fresh fused GemmRS operator is built, checked
against an independent projection reference, warmed up and timed with CUDA
events over `iterations` calls; the time is the MAX over ranks (all-reduce
outside the timed interval).  `planning.fit_role` runs the AB/BA pairs and the
confirmation on disjoint seeds; all ranks must end with the same plan digest.
Follows TempName-5090 python/flux_5090/calibration.py:23-100.
"""
from __future__ import annotations

import math
from pathlib import Path

from ..parallel.planning import SCHEMA, fit_role, role_digest, settings
from . import protocol as P


def calibrate(config: dict, group, out_dir) -> dict:
    import torch
    import torch.distributed as dist
    from ..parallel.gemm_rs import GemmRS
    from .validation import projection_reference, relative_error, require_all

    cfg = settings(config.get("calibration"))
    model = config["model"]
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    P.require(world == config["world_size"], "calibration TP size differs from the frozen config")
    m, n, chunk = model["sequence"] * model["micro_batch"], model["hidden"], model["chunk_rows"]
    samples = []
    destination = Path(out_dir) / f"calibration-rank{rank}-samples.json"
    roles = {}
    for role_index, (role, k) in enumerate((("attn", model["hidden"] // world), ("mlp", model["ffn"] // world))):
        def evaluate(plan, seed, arm, label, role=role, k=k, role_index=role_index):
            g = torch.Generator(device="cuda").manual_seed(seed + 173 * rank + 7919 * role_index)
            x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
            w = (torch.randn((n, k), generator=g, device="cuda") / math.sqrt(k)).to(torch.bfloat16)
            op = GemmRS(m, n, k, group, arm=arm, chunk_rows=chunk, plan=plan,
                        transport=config.get("transport", "nvlink"))
            actual = op.forward(x, w)
            plain, independent = projection_reference(x, w, rank, world, group, quantized=True)
            errs = torch.tensor([relative_error(actual, plain), relative_error(actual, independent)],
                                dtype=torch.float64, device="cuda")
            dist.all_reduce(errs, op=dist.ReduceOp.MAX, group=group)
            plain_err, codec_err = (float(v) for v in errs.cpu().tolist())
            require_all(math.isfinite(plain_err) and math.isfinite(codec_err) and plain_err <= 0.05
                        and codec_err <= 0.01, f"calibration {role}/{label} failed the numerical gate", group)
            for _ in range(cfg["warmup"]):
                op.forward(x, w)
            torch.cuda.synchronize()
            dist.barrier(group=group)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            for _ in range(cfg["iterations"]):
                op.forward(x, w)
            end.record()
            torch.cuda.synchronize()
            local = start.elapsed_time(end) / 1000.0
            t = torch.tensor(local, dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            elapsed = float(t.item())
            samples.append(dict(role=role, label=label, seed=seed, arm=arm, plan_digest=role_digest(plan),
                                arrival_order=plan["arrival_order"], local_elapsed_seconds=local,
                                max_rank_elapsed_seconds=elapsed, iterations=cfg["iterations"],
                                warmup=cfg["warmup"], bf16_relative_l2=plain_err,
                                codec_reference_relative_l2=codec_err, correctness_passed=True))
            P.write(destination, dict(schema="b200-calibration-samples-v1", rank=rank, samples=samples))
            op.close()
            return elapsed

        roles[role] = fit_role(m, n, k, world, chunk, evaluate, config=cfg,
                               seed=8000000 + 10000000 * role_index + int(config.get("seed", 1234)))
    bundle = dict(schema=SCHEMA, world_size=world, transport_lanes=2, roles=roles)
    digest = role_digest(bundle)
    gathered = [None] * world
    dist.all_gather_object(gathered, digest, group=group)
    if len(set(gathered)) != 1:
        raise RuntimeError("calibration produced different plans on different ranks")
    return dict(calibration_plan=bundle,
                calibration_results=dict(plan_sha256=digest, raw_samples=samples,
                                         raw_samples_file=destination.name,
                                         selection_timing="max-rank complete fused operator, CUDA events",
                                         training_and_confirmation_inputs_disjoint=True))
