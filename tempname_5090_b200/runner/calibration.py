"""Calibrate stage: measured arrival plans for the two GemmRS roles of the
model (attention out-projection, K = h/W, and MLP down-projection, K = f/W).

`OperatorTiming` is the evaluator that `planning.fit_role` drives: for each
plan it asks about, it builds a fresh fused GemmRS with that plan, checks the
first call's output against two references (the plain ordered BF16 sum and an
independent statement of the codec), warms up, and times `iterations` calls
with CUDA events.  The time of a comparison side is the slowest rank's (MAX
all-reduce outside the timed interval); every rank therefore makes the same
decisions, and the stage ends by checking that all ranks froze the same plan.
Every measurement is appended to a per-rank raw-sample file.

Counterpart of TempName-5090 python/flux_5090/calibration.py (same stage,
same kind of evidence); the structure, seeds and gates here are this module's.
"""
from __future__ import annotations

import hashlib
import math
from pathlib import Path

from ..parallel.planning import SCHEMA, Settings, fit_role, role_digest
from . import protocol as P

# Numerical gates of a calibration call (relative L2 error of the quantized
# arm's output).  Against the plain BF16 ordered sum the FP8 codec itself
# costs about 0.02 on Gaussian data (0.018 measured on 2 x B200, 0.025 in the
# CPU reference check); against an independent statement of the same codec
# only floating-point order differences remain (2.4e-5 measured).
CODEC_ERROR_GATE = 0.04
STATEMENT_ERROR_GATE = 1e-3
SAMPLES_SCHEMA = "b200-calibration-samples-v1"


def input_seed(seed: int, rank: int, role: str) -> int:
    """Per-rank, per-role input seed: every rank holds different partials, and
    the two roles never share inputs."""
    salt = int.from_bytes(hashlib.sha256(f"{role}/{rank}".encode()).digest()[:4], "little")
    return (seed * 1_000_003 + salt) % (2 ** 62)


class OperatorTiming:
    """Evaluator of one role: evaluate(plan, seed, arm, label) -> seconds."""

    def __init__(self, role: str, m: int, n: int, k: int, chunk_rows: int, settings: Settings, group, transport,
                 samples: list, sink: Path):
        import torch.distributed as dist
        self.role, self.m, self.n, self.k, self.chunk_rows = role, m, n, k, chunk_rows
        self.settings, self.group, self.transport = settings, group, transport
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.samples, self.sink = samples, sink

    def _slowest(self, values):
        import torch
        import torch.distributed as dist
        t = torch.tensor(values, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return t.cpu().tolist()

    def __call__(self, plan, seed, arm, label):
        import torch
        import torch.distributed as dist
        from ..parallel.gemm_rs import GemmRS
        from .validation import projection_reference, relative_error, require_all
        g = torch.Generator(device="cuda").manual_seed(input_seed(seed, self.rank, self.role))
        x = torch.randn((self.m, self.k), generator=g, device="cuda").to(torch.bfloat16)
        w = (torch.randn((self.n, self.k), generator=g, device="cuda") / math.sqrt(self.k)).to(torch.bfloat16)
        op = GemmRS(self.m, self.n, self.k, self.group, arm=arm, chunk_rows=self.chunk_rows, plan=plan,
                    transport=self.transport)
        try:
            got = op.forward(x, w)
            plain, statement = projection_reference(x, w, self.rank, self.world, self.group, quantized=True)
            codec_err, statement_err = self._slowest([relative_error(got, plain), relative_error(got, statement)])
            require_all(codec_err <= CODEC_ERROR_GATE and statement_err <= STATEMENT_ERROR_GATE,
                        f"calibration {self.role} {label}: output error {codec_err:.3g} vs BF16 sum, "
                        f"{statement_err:.3g} vs codec statement", self.group)
            for _ in range(self.settings.warmup):
                op.forward(x, w)
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            begin, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            begin.record()
            for _ in range(self.settings.iterations):
                op.forward(x, w)
            end.record()
            torch.cuda.synchronize()
            mine = begin.elapsed_time(end) / 1000.0
            slowest = self._slowest([mine])[0]
        finally:
            op.close()
        self.samples.append(dict(role=self.role, label=label, seed=seed, arm=arm, plan_sha256=role_digest(plan),
                                 arrival_order=plan["arrival_order"], rank_seconds=mine,
                                 slowest_rank_seconds=slowest, iterations=self.settings.iterations,
                                 warmup=self.settings.warmup, codec_relative_l2=codec_err,
                                 statement_relative_l2=statement_err, gates_passed=True))
        P.write(self.sink, dict(schema=SAMPLES_SCHEMA, rank=self.rank, samples=self.samples))
        return slowest


def calibrate(config: dict, group, out_dir) -> dict:
    import torch.distributed as dist
    model = config["model"]
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    P.require(world == config["world_size"], "calibration runs at the frozen TP size")
    cfg = Settings.parse(config.get("calibration"))
    m, n, chunk = model["sequence"] * model["micro_batch"], model["hidden"], model["chunk_rows"]
    samples: list = []
    sink = Path(out_dir) / f"calibration-rank{rank}-samples.json"
    base = int(config.get("seed", 1234))
    roles = {}
    for role, k in (("attn", model["hidden"] // world), ("mlp", model["ffn"] // world)):
        timing = OperatorTiming(role, m, n, k, chunk, cfg, group, config.get("transport", "nvlink"), samples, sink)
        role_base = (base * 7 + len(roles) + 1) * 1_000_000
        roles[role] = fit_role(m, n, k, world, chunk, timing, config=config.get("calibration"), seed=role_base)
    bundle = dict(schema=SCHEMA, world_size=world, transport_lanes=2, roles=roles)
    digest = role_digest(bundle)
    every = [None] * world
    dist.all_gather_object(every, digest, group=group)
    if len(set(every)) != 1:
        raise RuntimeError(f"ranks froze different arrival plans: {sorted(set(every))}")
    return dict(calibration_plan=bundle,
                calibration_results=dict(plan_sha256=digest, raw_samples=samples, raw_samples_file=sink.name,
                                         timing="slowest rank of the complete fused operator (CUDA events)",
                                         training_and_confirmation_inputs_disjoint=True))
