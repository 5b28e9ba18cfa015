"""CPU-only experiment protocol for the four-arm GemmRS study.

A run is a list of jobs: one `preflight`, one `calibrate` (fits the arrival
plans), then `operator` and/or `train` windows for every arm of every block.
Arm orders inside blocks are counter-balanced (each arm takes every position
equally often over 8 blocks, and every ordered pair of neighbours occurs) so
drift cancels out of the paired comparisons.  Each job gets a frozen config;
its per-rank JSON rows are validated before the next job starts.

Capabilities follow TempName-5090 tools/5090/protocol.py (jobs, orders,
frozen configs, row validation, TACO trajectory equality); the counter-balance
construction here is a Williams design and its mirror.  Nothing in this module
imports torch.
"""
from __future__ import annotations

import hashlib
import json
import math
from pathlib import Path

from ..config import ARMS, GPT_6P7B_BENCH, REFERENCE_DEFAULT, parameter_counts, validate_config

PROTOCOL = "b200-gemmrs-four-arm-v1"
ARRIVAL = "flux_taco_interleaved_arrival"
TACO_ARMS = ARMS[1:]
PLAN_SCHEMA = "rtx5090-arrival-plan-v1"
CALIBRATION = dict(warmup=2, iterations=5, training_pairs=3, confirmation_pairs=3, min_gain=0.002)
MODEL = dict(GPT_6P7B_BENCH)
REFERENCE_MODEL = dict(REFERENCE_DEFAULT)
SMALL_MODEL = dict(layers=2, hidden=512, ffn=2048, heads=4, sequence=2048, micro_batch=1,
                   accumulation_steps=1, vocab=4096, chunk_rows=128)
TIMING = dict(warmup_steps=3, timed_steps=10, operator_warmup=20, operator_iterations=50)
SCOPES = ("preflight", "operator", "train")


def require(ok, message):
    if not ok:
        raise ValueError(message)


def digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":"),
                                     allow_nan=False).encode()).hexdigest()


def sha(path) -> str:
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def read(path):
    return json.loads(Path(path).read_text())


def write(path, value) -> None:
    """Atomic JSON write (temporary file + rename)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    tmp.write_text(json.dumps(value, indent=2, ensure_ascii=False, allow_nan=False) + "\n")
    tmp.replace(path)


def finite(value, nonnegative=False) -> bool:
    return type(value) in (int, float) and math.isfinite(value) and (not nonnegative or value >= 0)


def valid_hash(value) -> bool:
    return isinstance(value, str) and len(value) == 64 and all(c in "0123456789abcdef" for c in value)


def validate_model(model: dict, world: int) -> dict:
    require(world in (1, 2, 4, 8), "world_size must be 1, 2, 4 or 8")
    require(set(model) == set(REFERENCE_MODEL), "unexpected or missing model dimensions")
    validate_config(model, world)
    require(model["hidden"] % 128 == 0, "the H128 codec needs hidden divisible by 128")
    require(model["hidden"] // model["heads"] == 128, "the attention kernel needs head_dim 128")
    return model


def williams_square(n: int) -> list:
    """Rows of a Williams design for even n: every item appears once per position
    and every ordered pair of neighbours appears exactly once."""
    require(n % 2 == 0, "a Williams design needs an even number of arms")
    first = [0]
    lo, hi = 1, n - 1
    for i in range(1, n):
        if i % 2:
            first.append(lo)
            lo += 1
        else:
            first.append(hi)
            hi -= 1
    return [[(x + r) % n for x in first] for r in range(n)]


def orders(trials: int, blocks: int) -> list:
    require(type(trials) is int and trials > 0 and type(blocks) is int and blocks > 0,
            "trials and blocks must be positive integers")
    square = williams_square(len(ARMS))
    rows = square + [row[::-1] for row in square]  # 8 rows: positions and carry-over balanced
    out = []
    for trial in range(trials):
        cycle = rows if trial % 2 == 0 else rows[::-1]
        for block in range(blocks):
            out.append(dict(trial=trial + 1, block=block,
                            arms=[ARMS[i] for i in cycle[block % len(cycle)]]))
    return out


def balanced(blocks: int) -> bool:
    return blocks >= 8 and blocks % 8 == 0


def jobs(trials: int, blocks: int, scope: str) -> list:
    require(scope in SCOPES, "invalid experiment scope")
    out = [dict(stage="preflight", arm="flux", trial=0, block=0, index=0, directory="preflight")]
    if scope == "preflight":
        return out
    out.append(dict(stage="calibrate", arm=ARRIVAL, trial=0, block=0, index=1, directory="calibrate"))
    for stage in ("operator", "train"):
        if stage == "train" and scope != "train":
            break
        for blk in orders(trials, blocks):
            for arm in blk["arms"]:
                out.append(dict(stage=stage, arm=arm, trial=blk["trial"], block=blk["block"], index=len(out),
                                directory=f"{stage}/trial{blk['trial']}/block{blk['block']:03d}-{arm}"))
    return out


def base_config(model: dict, world: int, *, run_id: str, seed: int = 1234, token_seed: int = 4321,
                timing: dict | None = None, calibration: dict | None = None, profile: bool = False,
                transport: str = "nvlink") -> dict:
    validate_model(model, world)
    return dict(protocol=PROTOCOL, run_id=run_id, world_size=world, model=dict(model), seed=seed,
                token_seed=token_seed, timing=dict(TIMING if timing is None else timing),
                calibration=dict(CALIBRATION if calibration is None else calibration), profile=profile,
                transport=transport, execution_plan=None, execution_plan_sha256=None)


def validate_execution_plan(bundle: dict, config: dict) -> dict:
    from ..parallel.planning import validate_role_plan
    model, world = config["model"], config["world_size"]
    require(isinstance(bundle, dict) and bundle.get("schema") == PLAN_SCHEMA and bundle.get("world_size") == world,
            "plan schema/topology mismatch")
    require(set(bundle.get("roles", {})) == {"attn", "mlp"}, "missing calibrated role")
    m = model["sequence"] * model["micro_batch"]
    for role, width in (("attn", model["hidden"]), ("mlp", model["ffn"])):
        validate_role_plan(bundle["roles"][role], m, model["hidden"], width // world, world, model["chunk_rows"])
    return bundle


def config_for_job(base: dict, job: dict, execution_plan: dict | None = None) -> dict:
    require(base.get("execution_plan") is None, "the base config must not carry a plan")
    cfg = json.loads(json.dumps(base))
    cfg["job"] = dict(job)
    if job["stage"] in ("operator", "train"):
        require(execution_plan is not None, "operator/train jobs need the frozen calibration plan")
        validate_execution_plan(execution_plan, base)
        cfg["execution_plan"] = execution_plan
        cfg["execution_plan_sha256"] = digest(execution_plan)
    return cfg


def calibration_from_rows(rows: list, config: dict) -> dict:
    plans = [r.get("calibration_plan") for r in rows]
    require(plans and all(p == plans[0] for p in plans), "ranks disagree on the calibrated plan")
    return validate_execution_plan(plans[0], config)


def validate_rows(rows: list, job: dict, config: dict) -> list:
    """Check every rank's row of one job; raise ValueError on the first problem."""
    world = config["world_size"]
    require(len(rows) == world and {r.get("rank") for r in rows} == set(range(world)), "missing or duplicate rank rows")
    for row in rows:
        require(row.get("world_size") == world and row.get("stage") == job["stage"] and row.get("arm") == job["arm"],
                "row identity differs from the job")
        require(row.get("completed") is True and row.get("passed") is True, f"rank {row.get('rank')} failed: "
                f"{row.get('error', 'unknown error')}")
        require(row.get("run_id") == config["run_id"], "worker run_id mismatch")
        require(row.get("execution_plan_sha256") == config.get("execution_plan_sha256"), "plan digest mismatch")
        stage = job["stage"]
        if stage == "train":
            steps = config["timing"]["timed_steps"]
            require(row.get("timed_steps") == steps and row.get("warmup_steps") == config["timing"]["warmup_steps"],
                    "wrong training step counts")
            require(finite(row.get("step_ms")) and row["step_ms"] > 0, "invalid device step time")
            for key in ("losses", "grad_norms"):
                values = row.get(key)
                require(isinstance(values, list) and len(values) == steps and all(finite(v) for v in values),
                        f"invalid {key}")
            for key in ("initialization_sha256", "input_sha256", "final_parameters_sha256"):
                require(valid_hash(row.get(key)), f"missing {key}")
            counts = parameter_counts(config["model"], world)
            require(row.get("parameters_per_rank") == counts["parameters_per_rank"], "parameter count changed")
            require(row.get("tokens_per_step") == config["model"]["sequence"] * config["model"]["micro_batch"]
                    * config["model"]["accumulation_steps"], "wrong tokens per step")
        elif stage == "operator":
            records = row.get("operator_results")
            require(isinstance(records, list) and {r.get("role") for r in records} == {"attn", "mlp"},
                    "missing operator roles")
            for rec in records:
                require(rec.get("correctness_passed") is True, "operator correctness failed")
                require(rec.get("timed_iterations") == config["timing"]["operator_iterations"],
                        "wrong operator iteration count")
                require(finite(rec.get("us_per_call")) and rec["us_per_call"] > 0, "invalid operator time")
                limit = 0.05 if row["arm"] != "flux" else 0.01
                require(finite(rec.get("bf16_relative_l2"), True) and rec["bf16_relative_l2"] <= limit,
                        "operator error above the gate")
                require(row["arm"] == "flux" or rec.get("order_bitwise_equal") is True,
                        "TACO arms are not bitwise equal")
        elif stage == "calibrate":
            require(isinstance(row.get("calibration_plan"), dict), "missing calibration plan")
        elif stage == "preflight":
            require(isinstance(row.get("checks"), dict) and all(v is True for v in row["checks"].values()),
                    "preflight check failed")
    return rows


def training_identity(rows: list) -> list:
    return [(r["rank"], r["losses"], r["grad_norms"], r["final_parameters_sha256"])
            for r in sorted(rows, key=lambda r: r["rank"])]


def compare_taco_trajectories(left: list, right: list) -> None:
    require(training_identity(left) == training_identity(right),
            "TACO arms trained to different trajectories (order must not change arithmetic)")
