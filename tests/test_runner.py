"""Runner layer on CPU: counter-balanced plan, statistics, synthetic execute +
replay with a fake launcher, tamper rejection, and process-group isolation."""
import hashlib
import json
import os
import subprocess
import sys
import time
from collections import Counter
from pathlib import Path

import pytest

from tempname_5090_b200.runner import controller as C
from tempname_5090_b200.runner import protocol as P
from tempname_5090_b200.runner import report as R


def test_preview_imports_no_torch_and_writes_nothing(tmp_path):
    code = ("import sys, io, contextlib; from tempname_5090_b200.runner import controller; "
            "buf = io.StringIO();\nwith contextlib.redirect_stdout(buf): controller.main(['--small-model', '--world', '2'])\n"
            "assert 'torch' not in sys.modules, 'torch imported'; import json; plan = json.loads(buf.getvalue()); "
            "assert plan['jobs'][0]['stage'] == 'preflight'")
    before = set(os.listdir(tmp_path))
    subprocess.run([sys.executable, "-c", code], check=True, cwd=str(tmp_path),
                   env=dict(os.environ, PYTHONPATH=str(Path(__file__).resolve().parents[1])))
    assert set(os.listdir(tmp_path)) == before


def test_orders_are_counter_balanced():
    o = P.orders(1, 8)
    for pos in range(4):
        assert Counter(b["arms"][pos] for b in o) == Counter({a: 2 for a in P.ARMS})
    pairs = Counter((b["arms"][i], b["arms"][i + 1]) for b in o for i in range(3))
    assert len(pairs) == 12 and set(pairs.values()) == {2}
    assert P.orders(2, 8)[8]["arms"] == P.orders(1, 8)[7]["arms"]  # trial 2 runs the cycle reversed


def test_jobs_layout():
    jobs = P.jobs(1, 8, "train")
    assert [j["stage"] for j in jobs[:2]] == ["preflight", "calibrate"]
    assert sum(j["stage"] == "operator" for j in jobs) == 32
    assert sum(j["stage"] == "train" for j in jobs) == 32
    assert len({j["directory"] for j in jobs}) == len(jobs)
    assert len(P.jobs(1, 8, "preflight")) == 1


def test_pair_statistics():
    s = R.pair_statistics([0.9] * 8, [1.0] * 8, balanced=True)
    assert abs(s["percent_faster"] - 10.0) < 1e-9 and s["ci95"] is not None and s["faster_blocks"] == 8
    assert R.pair_statistics([0.9] * 4, [1.0] * 4, balanced=False)["ci95"] is None
    with pytest.raises(ValueError):
        R.pair_statistics([1.0], [1.0, 2.0], balanced=False)


def _hash(text):
    return hashlib.sha256(text.encode()).hexdigest()


def fake_rows(job, cfg, world, timing, *, taco_losses=None):
    rows = []
    for rank in range(world):
        row = dict(rank=rank, world_size=world, stage=job["stage"], arm=job["arm"], run_id=cfg["run_id"],
                   completed=True, passed=True, execution_plan_sha256=cfg.get("execution_plan_sha256"))
        if job["stage"] == "preflight":
            row["checks"] = dict(tcgen05_gemm=True, nccl_all_gather=True)
        elif job["stage"] == "calibrate":
            from tempname_5090_b200.parallel.planning import fit_role, SCHEMA
            m = cfg["model"]
            M = m["sequence"] * m["micro_batch"]

            def evaluate(plan, seed, arm, label):  # deterministic stand-in timings
                return 0.95 if (label.endswith(":challenger") and ":reverse_all:" in label) else 1.0
            settings = dict(cfg["calibration"])
            row["calibration_plan"] = dict(schema=SCHEMA, world_size=world, transport_lanes=2, roles={
                "attn": fit_role(M, m["hidden"], m["hidden"] // world, world, m["chunk_rows"], evaluate,
                                 config=settings),
                "mlp": fit_role(M, m["hidden"], m["ffn"] // world, world, m["chunk_rows"], evaluate,
                                config=settings)})
        elif job["stage"] == "operator":
            base = {"flux": 100.0, "flux_taco": 90.0, "flux_taco_interleaved": 89.0, P.ARRIVAL: 88.0}[job["arm"]]
            row["operator_results"] = [dict(role=role, us_per_call=base + job["block"] * 0.1, correctness_passed=True,
                                            timed_iterations=timing["operator_iterations"], bf16_relative_l2=0.004,
                                            order_bitwise_equal=None if job["arm"] == "flux" else True,
                                            roofline_fraction=0.7) for role in ("attn", "mlp")]
        else:
            steps = timing["timed_steps"]
            losses = taco_losses if (taco_losses is not None and job["arm"] != "flux") else [10.0 - 0.1 * i for i in range(steps)]
            from tempname_5090_b200.config import parameter_counts
            row.update(timed_steps=steps, warmup_steps=timing["warmup_steps"],
                       step_ms={"flux": 50.0, "flux_taco": 48.0}.get(job["arm"], 47.0), losses=list(losses),
                       grad_norms=[1.0] * steps, tokens_per_step=cfg["model"]["sequence"] * cfg["model"]["micro_batch"],
                       initialization_sha256=_hash("init"), input_sha256=_hash("in"),
                       final_parameters_sha256=_hash("final" + ("taco" if job["arm"] != "flux" else "")),
                       parameters_per_rank=parameter_counts(cfg["model"], world)["parameters_per_rank"])
        rows.append(row)
    return rows


def _fake_launcher(world, **kw):
    def launcher(command, directory, timeout, env=None):
        cfg = json.loads((Path(directory) / "config.json").read_text())
        job = cfg.get("job") or dict(stage=command[command.index("--stage") + 1], arm=command[command.index("--arm") + 1])
        for row in fake_rows(job, cfg, world, cfg["timing"], **kw):
            P.write(Path(directory) / f"rank{row['rank']}.json", row)
        return 0
    return launcher


def _args(tmp_path, extra=()):
    return C.arguments(["--execute", "--out", str(tmp_path / "run"), "--world", "2", "--small-model",
                        "--blocks", "8", *extra])


def test_execute_and_replay_synthetic_run(tmp_path):
    out = C.execute(_args(tmp_path), launcher=_fake_launcher(2))
    state = json.loads((out / "batch-state.json").read_text())
    assert state["status"] == "completed" and state["completed_jobs"] == 66
    report = json.loads((out / "report.json").read_text())
    pairs = report["stages"]["operator"]["trial1"]["attn"]["pairs"]
    assert pairs["flux_taco/flux"]["percent_faster"] > 9 and pairs["flux_taco/flux"]["ci95"] is not None
    assert "flux_taco_interleaved/flux" in (out / "report.md").read_text()
    assert (out / "arrival-plan.json").exists() and (out / "sources-manifest.json").exists()
    with pytest.raises(FileExistsError):
        C.execute(_args(tmp_path), launcher=_fake_launcher(2))


def test_replay_rejects_tampering(tmp_path):
    out = C.execute(_args(tmp_path), launcher=_fake_launcher(2))
    victim = out / "operator/trial1/block003-flux" / "rank1.json"
    victim.unlink()
    with pytest.raises((ValueError, FileNotFoundError)):
        R.replay(out)


def _edit(path, fn):
    row = json.loads(Path(path).read_text())
    fn(row)
    Path(path).write_text(json.dumps(row))


def _add_trace(run, directory, tamper):
    d = run / directory
    (d / "trace_rank0.json").write_text('{"traceEvents": []}')
    sha = hashlib.sha256((d / "trace_rank0.json").read_bytes()).hexdigest()
    _edit(d / "rank0.json", lambda r: r.update(trace=dict(path="trace_rank0.json", sha256=sha, untimed=True)))
    if tamper:
        (d / "trace_rank0.json").write_text('{"traceEvents": [{"name": "x"}]}')


TAMPERS = {
    "missing_rank": lambda run: (run / "operator/trial1/block003-flux/rank1.json").unlink(),
    "run_id": lambda run: _edit(run / "train/trial1/block000-flux/rank0.json", lambda r: r.update(run_id="other")),
    "arm_swap": lambda run: _edit(run / "train/trial1/block001-flux_taco/rank1.json", lambda r: r.update(arm="flux")),
    "failed_rank": lambda run: _edit(run / "operator/trial1/block002-flux/rank0.json", lambda r: r.update(passed=False)),
    "negative_step_time": lambda run: _edit(run / "train/trial1/block002-flux/rank1.json",
                                            lambda r: r.update(step_ms=-1.0)),
    "short_losses": lambda run: _edit(run / "train/trial1/block004-flux/rank0.json",
                                      lambda r: r.update(losses=r["losses"][:-1])),
    "plan_digest": lambda run: _edit(run / "train/trial1/block005-flux/rank0.json",
                                     lambda r: r.update(execution_plan_sha256="0" * 64)),
    "frozen_plan_digest": lambda run: _edit(run / "plan.json", lambda p: p.update(execution_plan_sha256="0" * 64)),
    "taco_trajectory": lambda run: _edit(run / "train/trial1/block006-flux_taco_interleaved/rank0.json",
                                         lambda r: r.update(final_parameters_sha256=_hash("different"))),
    "trace_bytes": lambda run: _add_trace(run, "train/trial1/block007-flux", tamper=True),
    "source_bytes": lambda run: (run / "sources/tempname_5090_b200/config.py").write_text("# edited\n"),
    "source_added": lambda run: (run / "sources/csrc/extra.cu").write_text("// new\n"),
    "calibration_samples": lambda run: [_edit(run / "calibrate" / f"rank{r}.json", _doctor_calibration)
                                        for r in range(2)],
}


def _doctor_calibration(row):
    rec = row["calibration_plan"]["roles"]["attn"]["diagnostics"]["trials"][0]
    rec["pairs"][0]["challenger_s"] *= 0.5


@pytest.mark.parametrize("name", sorted(TAMPERS))
def test_replay_rejects_each_tamper(tmp_path, name):
    out = C.execute(_args(tmp_path), launcher=_fake_launcher(2))
    R.replay(out)  # intact run replays
    TAMPERS[name](out)
    with pytest.raises((ValueError, FileNotFoundError, KeyError)):
        R.replay(out)


def test_replay_accepts_an_intact_trace(tmp_path):
    out = C.execute(_args(tmp_path), launcher=_fake_launcher(2))
    _add_trace(out, "train/trial1/block007-flux", tamper=False)
    R.replay(out)


def test_taco_trajectory_mismatch_fails_the_run(tmp_path):
    calls = {"n": 0}
    base = _fake_launcher(2)

    def launcher(command, directory, timeout, env=None):
        base(command, directory, timeout, env)
        if "--arm" in command and command[command.index("--arm") + 1] == P.ARRIVAL and "train" in str(directory):
            for r in range(2):
                p = Path(directory) / f"rank{r}.json"
                row = json.loads(p.read_text())
                row["losses"][0] += 1e-3
                P.write(p, row)
        return 0
    with pytest.raises(ValueError, match="trajectories"):
        C.execute(_args(tmp_path), launcher=launcher)
    assert json.loads((tmp_path / "run" / "batch-state.json").read_text())["status"] == "failed"


def test_failing_launch_marks_batch_failed(tmp_path):
    def launcher(command, directory, timeout, env=None):
        raise RuntimeError("launch failed")
    with pytest.raises(RuntimeError):
        C.execute(_args(tmp_path), launcher=launcher)
    state = json.loads((tmp_path / "run" / "batch-state.json").read_text())
    assert state["status"] == "failed" and "launch failed" in state["error"]


def test_timeout_stops_only_the_owned_process_group(tmp_path):
    bystander = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(60)"], start_new_session=True)
    try:
        with pytest.raises(TimeoutError):
            C.launch([sys.executable, "-c", "import time; time.sleep(60)"], tmp_path / "job", timeout=1)
        assert bystander.poll() is None
    finally:
        bystander.kill()
        bystander.wait()


def test_background_relaunch_preserves_arguments_without_a_shell(tmp_path, monkeypatch):
    """--background re-executes the controller detached with the same arguments
    (minus --background) as an argument list: no shell ever parses them."""
    seen = {}

    class _Proc:
        pid = 4242

    def fake_popen(cmd, **kw):
        seen["cmd"], seen["kw"] = cmd, kw
        return _Proc()
    monkeypatch.setattr(C.subprocess, "Popen", fake_popen)
    odd = str(tmp_path / "run; echo injected $(id)")
    argv = ["--execute", "--background", "--out", odd, "--world", "2", "--small-model"]
    C.main(argv)
    cmd, kw = seen["cmd"], seen["kw"]
    assert isinstance(cmd, list) and not kw.get("shell", False) and kw.get("start_new_session") is True
    assert cmd[1:3] == ["-m", "tempname_5090_b200.runner.controller"]
    assert cmd[3:] == ["--execute", "--out", odd, "--world", "2", "--small-model"]
    receipt = json.loads(Path(odd + ".launcher.json").read_text())
    assert receipt["pid"] == 4242 and receipt["argv"] == cmd[3:] and len(receipt["token"]) == 32
    assert kw["env"]["TN5B_CONTROLLER_TOKEN"] == receipt["token"]
