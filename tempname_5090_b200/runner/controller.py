"""Experiment controller: plan, execute (torchrun windows), validate, report.

    python -m tempname_5090_b200.runner.controller                      # preview plan (JSON), no torch
    python -m tempname_5090_b200.runner.controller --execute --out DIR  # run every job
    python -m tempname_5090_b200.runner.controller --execute --background --out DIR
    python -m tempname_5090_b200.runner.controller --report DIR         # read-only replay

Each job runs as `torch.distributed.run --standalone --local-addr 127.0.0.1 --nnodes=1 --nproc-per-node W
-m tempname_5090_b200.runner.worker ...` in its own process group with a
timeout (SIGTERM, then SIGKILL of that group only).  After every job the
per-rank rows are validated; the calibration plan is frozen into
`arrival-plan.json`; TACO-arm training trajectories must be identical.
Progress is tracked in `batch-state.json` (preparing, running, failed,
interrupted, completed).  The output directory must not exist.  Sources are
snapshotted into the run directory with a SHA-256 manifest.
Capabilities follow TempName-5090 tools/5090/init.py.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import signal
import subprocess
import sys
import time
import uuid
from pathlib import Path

from . import protocol as P

PACKAGE_ROOT = Path(__file__).resolve().parents[1]
REPO_ROOT = PACKAGE_ROOT.parent


def arguments(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--execute", action="store_true")
    ap.add_argument("--background", action="store_true")
    ap.add_argument("--report", type=Path)
    ap.add_argument("--out", type=Path)
    ap.add_argument("--world", type=int, default=8)
    ap.add_argument("--trials", type=int, default=1)
    ap.add_argument("--blocks", type=int, default=8)
    ap.add_argument("--scope", choices=P.SCOPES, default="train")
    ap.add_argument("--small-model", action="store_true")
    ap.add_argument("--reference-model", action="store_true", help="the reference default config (mb1 x acc4, V=33792)")
    ap.add_argument("--profile", action="store_true")
    ap.add_argument("--transport", choices=("nvlink", "nccl"), default="nvlink")
    ap.add_argument("--timeout", type=int, default=3600, help="seconds per job window")
    ap.add_argument("--seed", type=int, default=1234)
    args = ap.parse_args(argv)
    if args.execute and args.out is None:
        ap.error("--execute needs --out")
    if args.background and not args.execute:
        ap.error("--background needs --execute")
    if args.trials < 1 or args.blocks < 1:
        ap.error("trials and blocks must be positive")
    return args


def model_for(args) -> dict:
    if args.small_model:
        return dict(P.SMALL_MODEL)
    if args.reference_model:
        return dict(P.REFERENCE_MODEL)
    return dict(P.MODEL)


def plan_for(args, run_id=None) -> dict:
    model = model_for(args)
    run_id = run_id or uuid.uuid4().hex
    config = P.base_config(model, args.world, run_id=run_id, seed=args.seed, profile=args.profile,
                           transport=args.transport)
    return dict(protocol=P.PROTOCOL, trials=args.trials, blocks=args.blocks, scope=args.scope,
                config=config, jobs=P.jobs(args.trials, args.blocks, args.scope), timeout=args.timeout)


def source_manifest(root: Path) -> dict:
    files = sorted(p for p in root.rglob("*") if p.is_file() and "__pycache__" not in p.parts
                   and p.suffix in (".py", ".cu", ".cuh", ".h", ".cpp"))
    return {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest() for p in files}


def snapshot_sources(out: Path) -> dict:
    dst = out / "sources"
    for sub in ("tempname_5090_b200", "csrc"):
        src = REPO_ROOT / sub
        if src.exists():
            shutil.copytree(src, dst / sub, ignore=shutil.ignore_patterns("__pycache__"))
    manifest = source_manifest(dst)
    P.write(out / "sources-manifest.json", manifest)
    return manifest


def command_for(python: str, directory: Path, job: dict, world: int) -> list:
    # Loopback rendezvous: the host name of a container need not resolve.
    return [python, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1", "--nnodes=1",
            f"--nproc-per-node={world}",
            "-m", "tempname_5090_b200.runner.worker", "--config", str(directory / "config.json"),
            "--out", str(directory), "--stage", job["stage"], "--arm", job["arm"]]


def stop_process_group(proc: subprocess.Popen, grace: float = 20.0) -> None:
    """SIGTERM then SIGKILL the job's own process group (never anything else)."""
    if proc.poll() is not None:
        return
    try:
        os.killpg(proc.pid, signal.SIGTERM)
    except ProcessLookupError:
        return
    deadline = time.time() + grace
    while time.time() < deadline and proc.poll() is None:
        time.sleep(0.2)
    if proc.poll() is None:
        try:
            os.killpg(proc.pid, signal.SIGKILL)
        except ProcessLookupError:
            pass
        proc.wait()


def launch(command: list, directory: Path, timeout: int, env: dict | None = None) -> int:
    directory.mkdir(parents=True, exist_ok=True)
    with open(directory / "stdout.log", "w") as out, open(directory / "stderr.log", "w") as err:
        proc = subprocess.Popen(command, cwd=str(REPO_ROOT), stdout=out, stderr=err, start_new_session=True,
                                env=env)
        try:
            return proc.wait(timeout=timeout)
        except subprocess.TimeoutExpired:
            stop_process_group(proc)
            raise TimeoutError(f"job exceeded {timeout} s and its process group was stopped")
        except BaseException:
            stop_process_group(proc)
            raise


def execute(args, launcher=launch) -> Path:
    out = Path(args.out)
    if out.exists():
        raise FileExistsError(f"{out} already exists; refusing to reuse an output directory")
    out.mkdir(parents=True)
    state = dict(status="preparing", started=time.time(), completed_jobs=0)
    P.write(out / "batch-state.json", state)
    plan = plan_for(args)
    plan["sources"] = snapshot_sources(out)
    P.write(out / "plan.json", plan)
    config = plan["config"]
    execution_plan = None
    train_rows = {}
    env = dict(os.environ, PYTHONPATH=str(REPO_ROOT))
    try:
        state["status"] = "running"
        P.write(out / "batch-state.json", state)
        for job in plan["jobs"]:
            directory = out / job["directory"]
            cfg = P.config_for_job(config, job, execution_plan) if job["stage"] in ("operator", "train") else config
            P.write(directory / "config.json", cfg)
            code = launcher(command_for(sys.executable, directory, job, config["world_size"]), directory,
                            plan["timeout"], env)
            if code != 0:
                raise RuntimeError(f"job {job['directory']} exited with {code}")
            rows = [P.read(directory / f"rank{r}.json") for r in range(config["world_size"])]
            P.validate_rows(rows, job, cfg)
            if job["stage"] == "calibrate":
                execution_plan = P.calibration_from_rows(rows, config)
                P.write(out / "arrival-plan.json", execution_plan)
                plan["execution_plan_sha256"] = P.digest(execution_plan)
                P.write(out / "plan.json", plan)
            if job["stage"] == "train":
                key = (job["trial"], job["block"])
                train_rows.setdefault(key, {})[job["arm"]] = rows
                arms = train_rows[key]
                if "flux_taco" in arms:
                    for other in ("flux_taco_interleaved", P.ARRIVAL):
                        if other in arms:
                            P.compare_taco_trajectories(arms["flux_taco"], arms[other])
            state["completed_jobs"] += 1
            P.write(out / "batch-state.json", state)
        from .report import markdown, replay
        report = replay(out)
        P.write(out / "report.json", report)
        (out / "report.md").write_text(markdown(report))
        state["status"] = "completed"
    except KeyboardInterrupt:
        state["status"] = "interrupted"
        raise
    except BaseException as exc:
        state["status"] = "failed"
        state["error"] = str(exc)
        raise
    finally:
        state["finished"] = time.time()
        P.write(out / "batch-state.json", state)
    return out


def start_background(args, argv) -> dict:
    """Re-execute this controller detached (new session); return the receipt."""
    out = Path(args.out)
    token = uuid.uuid4().hex
    out.parent.mkdir(parents=True, exist_ok=True)
    log = open(str(out) + ".controller.log", "w")
    forwarded = [a for a in argv if a != "--background"]
    proc = subprocess.Popen([sys.executable, "-m", "tempname_5090_b200.runner.controller", *forwarded],
                            cwd=str(REPO_ROOT), stdout=log, stderr=log, start_new_session=True,
                            env=dict(os.environ, PYTHONPATH=str(REPO_ROOT), TN5B_CONTROLLER_TOKEN=token))
    receipt = dict(pid=proc.pid, token=token, out=str(out), argv=forwarded, started=time.time())
    P.write(Path(str(out) + ".launcher.json"), receipt)
    return receipt


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    args = arguments(argv)
    if args.report is not None:
        from .report import markdown, replay
        report = replay(args.report)
        print(markdown(report))
        return 0
    if not args.execute:
        print(json.dumps(plan_for(args, run_id="preview"), indent=2))
        return 0
    if args.background:
        print(json.dumps(start_background(args, argv)))
        return 0
    execute(args)
    return 0


if __name__ == "__main__":
    sys.exit(main())
