"""Read-only replay of a run directory and paired statistics.

`replay(root)` re-reads every job's per-rank rows, re-validates them with the
protocol, checks the TACO-arm trajectory equality and the calibration plan
digest, then summarises each stage.  Arm comparisons are paired by block: the
estimate is the geometric-mean speed-up 100 * (1 - exp(mean(log(cand / ref)))),
with a percentile bootstrap 95 % interval (fixed seed, 10 000 resamples) only
for balanced designs (a multiple of 8 blocks).  Times are device-measured,
max over ranks.  Capabilities follow TempName-5090 tools/5090/report.py.
"""
from __future__ import annotations

import math
import random
import statistics
import hashlib
from pathlib import Path

from . import protocol as P

BOOTSTRAP_SEED = 20261108
COMPARISONS = (("flux_taco", "flux"), ("flux_taco_interleaved", "flux_taco"),
               (P.ARRIVAL, "flux_taco_interleaved"), ("flux_taco_interleaved", "flux"), (P.ARRIVAL, "flux"))


def pair_statistics(candidate, reference, balanced: bool, bootstrap: int = 10000) -> dict:
    P.require(len(candidate) == len(reference) and len(candidate) > 0, "unpaired samples")
    P.require(all(x > 0 for x in candidate + reference), "times must be positive")
    logs = [math.log(c / r) for c, r in zip(candidate, reference)]
    estimate = 100.0 * (1.0 - math.exp(statistics.fmean(logs)))
    interval = None
    if balanced and len(logs) >= 8:
        rng = random.Random(BOOTSTRAP_SEED)
        draws = sorted(100.0 * (1.0 - math.exp(statistics.fmean(rng.choices(logs, k=len(logs)))))
                       for _ in range(bootstrap))
        interval = [draws[int((bootstrap - 1) * 0.025)], draws[int((bootstrap - 1) * 0.975)]]
    return dict(percent_faster=estimate, ci95=interval, paired_blocks=len(logs),
                faster_blocks=sum(c < r for c, r in zip(candidate, reference)))


def _summary(values) -> dict:
    return dict(mean=statistics.fmean(values), median=statistics.median(values), min=min(values),
                max=max(values), windows=len(values))


def samples_from_rows(job: dict, rows: list) -> list:
    """One sample per (role) per job: max over ranks of the device time."""
    if job["stage"] == "train":
        return [dict(stage="train", role="full_step", arm=job["arm"], trial=job["trial"], block=job["block"],
                     value=max(r["step_ms"] for r in rows), tokens_per_step=rows[0]["tokens_per_step"],
                     mean_loss=statistics.fmean(rows[0]["losses"]), final_loss=rows[0]["losses"][-1])]
    out = []
    for role in ("attn", "mlp"):
        recs = [next(x for x in r["operator_results"] if x["role"] == role) for r in rows]
        out.append(dict(stage="operator", role=role, arm=job["arm"], trial=job["trial"], block=job["block"],
                        value=max(x["us_per_call"] for x in recs),
                        bf16_relative_l2=max(x["bf16_relative_l2"] for x in recs),
                        roofline_fraction=min(x.get("roofline_fraction", 0.0) for x in recs)))
    return out


def summarize_stage(samples: list, stage: str, trials: int, blocks: int) -> dict:
    roles = ("attn", "mlp") if stage == "operator" else ("full_step",)
    result = {}
    for trial in range(1, trials + 1):
        per_role = {}
        for role in roles:
            values = {}
            for arm in P.ARMS:
                values[arm] = [next(s["value"] for s in samples if s["trial"] == trial and s["block"] == b
                                    and s["arm"] == arm and s["role"] == role) for b in range(blocks)]
            arms = {arm: _summary(v) for arm, v in values.items()}
            if stage == "train":
                for arm in P.ARMS:
                    sel = [s for s in samples if s["trial"] == trial and s["arm"] == arm and s["role"] == role]
                    arms[arm]["tokens_per_second"] = sel[0]["tokens_per_step"] * 1000.0 / arms[arm]["mean"]
                    arms[arm]["mean_loss"] = statistics.fmean(s["mean_loss"] for s in sel)
            pairs = {f"{c}/{r}": pair_statistics(values[c], values[r], P.balanced(blocks)) for c, r in COMPARISONS}
            per_role[role] = dict(unit="us/call" if stage == "operator" else "ms/step", arms=arms, pairs=pairs)
        result[f"trial{trial}"] = per_role
    return result


def validate_calibration_evidence(execution_plan: dict, config: dict) -> None:
    """Every frozen role plan's decision must follow from its recorded samples."""
    from ..parallel.planning import replay_role_evidence
    for role, rp in sorted(execution_plan["roles"].items()):
        m, n, k = rp["shape"]
        try:
            replay_role_evidence(rp, m, n, k, config["world_size"], rp["chunk_rows"])
        except ValueError as exc:
            raise ValueError(f"calibration evidence of role {role}: {exc}") from exc


def validate_sources(root: Path, plan: dict) -> None:
    """The run's source snapshot still hashes to its manifest (and to the plan's copy)."""
    manifest = P.read(root / "sources-manifest.json")
    P.require(plan.get("sources", manifest) == manifest, "plan and source manifest differ")
    base = root / "sources"
    present = sorted(str(p.relative_to(base)) for p in base.rglob("*") if p.is_file()
                     and "__pycache__" not in p.parts and p.suffix in (".py", ".cu", ".cuh", ".h", ".cpp"))
    P.require(present == sorted(manifest), "source snapshot files differ from the manifest")
    for rel, sha in manifest.items():
        P.require(hashlib.sha256((base / rel).read_bytes()).hexdigest() == sha, f"source {rel} was modified")


def replay(root) -> dict:
    """Re-validate a finished run directory from disk and produce the report dict."""
    root = Path(root)
    plan = P.read(root / "plan.json")
    if (root / "sources-manifest.json").exists():
        validate_sources(root, plan)
    config = plan["config"]
    jobs = plan["jobs"]
    execution_plan = None
    samples = {"operator": [], "train": []}
    train_rows = {}
    for job in jobs:
        directory = root / job["directory"]
        rows = [P.read(directory / f"rank{r}.json") for r in range(config["world_size"])]
        cfg = P.config_for_job(config, job, execution_plan) if job["stage"] in ("operator", "train") else config
        P.validate_rows(rows, job, cfg)
        for row in rows:
            trace = row.get("trace")
            if trace:  # optional profiler trace: the file must still hash to the recorded digest
                data = (directory / trace["path"]).read_bytes()
                P.require(hashlib.sha256(data).hexdigest() == trace["sha256"], "trace file differs from its digest")
        if job["stage"] == "calibrate":
            execution_plan = P.calibration_from_rows(rows, config)
            P.require(P.digest(execution_plan) == plan.get("execution_plan_sha256", P.digest(execution_plan)),
                      "calibration plan digest differs from the frozen plan")
            validate_calibration_evidence(execution_plan, config)
        elif job["stage"] in samples:
            samples[job["stage"]].extend(samples_from_rows(job, rows))
            if job["stage"] == "train":
                train_rows[(job["trial"], job["block"], job["arm"])] = rows
    for (trial, block, arm), rows in train_rows.items():
        if arm in P.TACO_ARMS and arm != "flux_taco":
            other = train_rows.get((trial, block, "flux_taco"))
            if other is not None:
                P.compare_taco_trajectories(other, rows)
    trials, blocks = plan["trials"], plan["blocks"]
    report = dict(protocol=P.PROTOCOL, run_id=config["run_id"], world_size=config["world_size"],
                  model=config["model"], trials=trials, blocks=blocks, balanced=P.balanced(blocks),
                  timing="CUDA events on the launching stream, max over ranks",
                  execution_plan_sha256=P.digest(execution_plan) if execution_plan else None, stages={})
    for stage, s in samples.items():
        if s:
            report["stages"][stage] = summarize_stage(s, stage, trials, blocks)
    return report


def markdown(report: dict) -> str:
    lines = [f"# GemmRS four-arm report ({report['protocol']})", "",
             f"run `{report['run_id']}`, TP{report['world_size']}, trials {report['trials']}, "
             f"blocks {report['blocks']} ({'balanced' if report['balanced'] else 'unbalanced: no CI'}); "
             f"{report['timing']}.", ""]
    for stage, trials in report["stages"].items():
        for trial, roles in trials.items():
            for role, data in roles.items():
                lines += [f"## {stage} / {trial} / {role} ({data['unit']})", "",
                          "| arm | mean | median | min | max |", "| --- | --- | --- | --- | --- |"]
                for arm, s in data["arms"].items():
                    lines.append(f"| {arm} | {s['mean']:.3f} | {s['median']:.3f} | {s['min']:.3f} | {s['max']:.3f} |")
                lines += ["", "| comparison | % faster | 95% CI | faster blocks |", "| --- | --- | --- | --- |"]
                for name, p in data["pairs"].items():
                    ci = "n/a" if p["ci95"] is None else f"[{p['ci95'][0]:.2f}, {p['ci95'][1]:.2f}]"
                    lines.append(f"| {name} | {p['percent_faster']:.2f} | {ci} | {p['faster_blocks']}/{p['paired_blocks']} |")
                lines.append("")
    return "\n".join(lines)
