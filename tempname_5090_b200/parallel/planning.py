"""Arrival-priority plans for the `flux_taco_interleaved_arrival` arm.

A role plan is a JSON-safe dict {shape, chunk_rows, arrival_order, diagnostics};
`arrival_order` is a bijection of physical blocks in which slot s keeps the
interleaved destination s % W.  Plans are fitted from complete-operator
timings measured in AB/BA pairs, then confirmed on disjoint inputs; a
candidate is kept only if every confirmation pair beats `min_gain`.

Behaviour follows TempName-5090 python/flux_5090/planning.py:1-190 (same
candidate family: identity / reverse_all / reverse_odd / reverse_even /
rotate, same geometric-mean paired gain and confirmation rule), so a plan
fitted here is accepted by either implementation.
"""
from __future__ import annotations

import hashlib
import json
import math
import statistics

SCHEMA = "rtx5090-arrival-plan-v1"
ARRIVAL_ARM = "flux_taco_interleaved_arrival"
DEFAULTS = dict(warmup=2, iterations=5, training_pairs=3, confirmation_pairs=3, min_gain=0.002)


def role_digest(plan) -> str:
    text = json.dumps(plan, sort_keys=True, separators=(",", ":"), allow_nan=False)
    return hashlib.sha256(text.encode()).hexdigest()


def _per_destination(m, n, k, world, chunk_rows):
    if any(type(x) is not int or x <= 0 for x in (m, n, k, world, chunk_rows)):
        raise ValueError("positive integer shape/world/chunk_rows required")
    if world < 2 or m % (world * chunk_rows) or n % 128 or chunk_rows % 128 or k % 8:
        raise ValueError("require M divisible by world*chunk_rows and N by 128")
    return m // world // chunk_rows


def base_order(m, n, k, world, chunk_rows):
    per = _per_destination(m, n, k, world, chunk_rows)
    return [(slot % world) * per + slot // world for slot in range(per * world)]


def validate_role_plan(plan, m=None, n=None, k=None, world=None, chunk_rows=None, *,
                       shape=None, world_size=None):
    if shape is not None:
        if not isinstance(shape, (list, tuple)) or len(shape) != 3:
            raise ValueError("shape must be [M,N,K]")
        if any(x is not None for x in (m, n, k)):
            raise ValueError("use shape or M/N/K, not both")
        m, n, k = shape
    if world_size is not None:
        if world is not None and world != world_size:
            raise ValueError("conflicting world/world_size")
        world = world_size
    per = _per_destination(m, n, k, world, chunk_rows)
    if not isinstance(plan, dict) or set(plan) != {"shape", "chunk_rows", "arrival_order",
                                                   "diagnostics"}:
        raise ValueError("unexpected or missing role-plan fields")
    if plan["shape"] != [m, n, k] or plan["chunk_rows"] != chunk_rows:
        raise ValueError("plan shape/chunk_rows differs from the operator")
    order = plan["arrival_order"]
    blocks = per * world
    if (not isinstance(order, list) or len(order) != blocks
            or any(type(v) is not int for v in order) or sorted(order) != list(range(blocks))):
        raise ValueError("arrival order must be a bijection of physical blocks")
    if any(physical // per != slot % world for slot, physical in enumerate(order)):
        raise ValueError("arrival order must keep every interleaved destination slot")
    if not isinstance(plan["diagnostics"], dict):
        raise ValueError("plan diagnostics must be a dictionary")
    role_digest(plan)  # rejects NaN / non-JSON content
    return plan


def make_role(m, n, k, world, chunk_rows, order=None):
    plan = dict(shape=[m, n, k], chunk_rows=chunk_rows,
                arrival_order=list(base_order(m, n, k, world, chunk_rows) if order is None else order),
                diagnostics={})
    return validate_role_plan(plan, m, n, k, world, chunk_rows)


def _transforms(per):
    ident = list(range(per))
    return [
        ("identity", lambda d: ident),
        ("reverse_all", lambda d: ident[::-1]),
        ("reverse_odd", lambda d: ident[::-1] if d % 2 else ident),
        ("reverse_even", lambda d: ident if d % 2 else ident[::-1]),
        ("rotate", lambda d: ident[1:] + ident[:1]),
    ]


def candidates(m, n, k, world, chunk_rows):
    per = _per_destination(m, n, k, world, chunk_rows)
    out, seen = [], set()
    for name, transform in _transforms(per):
        per_dest = [transform(d) for d in range(world)]
        order = [d * per + per_dest[d][w] for w in range(per) for d in range(world)]
        if tuple(order) not in seen:
            seen.add(tuple(order))
            out.append(dict(name=name, arrival_order=order))
    return out


def settings(values=None):
    result = dict(DEFAULTS)
    if values is not None:
        if not isinstance(values, dict) or set(values) - set(DEFAULTS):
            raise ValueError("unknown calibration settings")
        result.update(values)
    for key in ("warmup", "iterations", "training_pairs", "confirmation_pairs"):
        lower = 0 if key == "warmup" else 1
        if type(result[key]) is not int or result[key] < lower:
            raise ValueError(f"invalid calibration {key}")
    gain = result["min_gain"]
    if type(gain) not in (int, float) or not math.isfinite(gain) or not 0 <= gain < 1:
        raise ValueError("invalid calibration min_gain")
    result["min_gain"] = float(gain)
    return result


def _elapsed(value) -> float:
    if isinstance(value, dict) and value.get("correctness_passed", True) is not True:
        raise ValueError("numerical failure in a calibration candidate")
    elapsed = value.get("elapsed_seconds") if isinstance(value, dict) else value
    if type(elapsed) not in (int, float) or not math.isfinite(elapsed) or elapsed <= 0:
        raise ValueError("evaluator must return a positive complete-operator time")
    return float(elapsed)


def paired_measure(reference, candidate, evaluate, *, arm, pairs, seed, phase, name):
    """AB/BA pairs on identical inputs; evaluate(plan, seed, arm, label) -> seconds."""
    records = []
    for pair in range(pairs):
        inputs = seed + pair
        sides = [("reference", reference), ("candidate", candidate)]
        if pair % 2:
            sides.reverse()
        measured = {}
        for side, plan in sides:
            measured[side] = _elapsed(evaluate(plan, inputs, arm, f"{phase}/{name}/pair{pair}/{side}"))
        records.append(dict(pair=pair, seed=inputs, execution_order=[s for s, _ in sides],
                            reference_seconds=measured["reference"],
                            candidate_seconds=measured["candidate"],
                            fractional_gain=1 - measured["candidate"] / measured["reference"]))
    gain = 1 - math.exp(statistics.mean(
        math.log(r["candidate_seconds"] / r["reference_seconds"]) for r in records))
    return dict(name=name, phase=phase, paired_samples=records, fractional_gain=gain,
                worst_pair_gain=min(r["fractional_gain"] for r in records),
                candidate_digest=role_digest(candidate), reference_digest=role_digest(reference))


def confirmed(record, minimum_gain):
    return (record["fractional_gain"] > minimum_gain
            and all(r["fractional_gain"] > minimum_gain for r in record["paired_samples"]))


def replay_role_evidence(plan, m, n, k, world, chunk_rows) -> dict:
    """Re-derive a frozen role plan's decision from its recorded raw samples.

    Checks, from the plan's diagnostics alone: every pair gain and every
    record's geometric-mean gain recomputed from the recorded seconds; AB/BA
    alternation; each training record compares the identity order with the
    candidate of that name (digests); the proposed candidate is the best
    training gain above the bar; confirmation uses disjoint seeds and the
    acceptance rule; the frozen order is the accepted candidate's order or the
    identity.  Returns the recomputed summary; raises ValueError on any
    mismatch.  Mirrors TempName-5090 tools/5090/report.py:214-269."""
    plan = validate_role_plan(plan, m, n, k, world, chunk_rows)
    diag = plan.get("diagnostics") or {}
    cfg = settings(diag.get("settings"))
    arr = diag.get("arrival")
    if not isinstance(arr, dict):
        raise ValueError("plan has no arrival calibration evidence")
    identity = make_role(m, n, k, world, chunk_rows)
    cands = {c["name"]: make_role(m, n, k, world, chunk_rows, c["arrival_order"])
             for c in candidates(m, n, k, world, chunk_rows)[1:]}

    def check_record(rec, name, phase, pairs):
        if rec.get("name") != name or rec.get("phase") != phase:
            raise ValueError("calibration record identity mismatch")
        samples = rec.get("paired_samples")
        if not isinstance(samples, list) or len(samples) != pairs:
            raise ValueError("wrong number of calibration pairs")
        logs = []
        for i, smp in enumerate(samples):
            want_order = ["reference", "candidate"] if i % 2 == 0 else ["candidate", "reference"]
            if smp.get("pair") != i or smp.get("execution_order") != want_order:
                raise ValueError("calibration pairs are not AB/BA alternated")
            ref_s, cand_s = _elapsed(smp.get("reference_seconds")), _elapsed(smp.get("candidate_seconds"))
            if abs((1 - cand_s / ref_s) - smp.get("fractional_gain", float("nan"))) > 1e-12:
                raise ValueError("recorded pair gain differs from its seconds")
            logs.append(math.log(cand_s / ref_s))
        gain = 1 - math.exp(statistics.mean(logs))
        if abs(gain - rec.get("fractional_gain", float("nan"))) > 1e-12:
            raise ValueError("recorded gain differs from its samples")
        if rec.get("reference_digest") != role_digest(identity) or \
                rec.get("candidate_digest") != role_digest(cands[name]):
            raise ValueError("calibration record measured a different order")
        return gain, [s["seed"] for s in samples]

    records = arr.get("training_candidates") or []
    if sorted(r.get("name") for r in records) != sorted(cands):
        raise ValueError("training did not cover exactly the candidate family")
    best_name, best_gain, training_seeds = "identity", 0.0, set()
    for rec in records:
        gain, seeds = check_record(rec, rec.get("name"), "arrival_training", cfg["training_pairs"])
        training_seeds.update(seeds)
        if gain > max(cfg["min_gain"], best_gain):
            best_name, best_gain = rec["name"], gain
    if arr.get("proposed_candidate") != best_name:
        raise ValueError("proposed candidate is not the best training gain")
    accepted = False
    conf = arr.get("confirmation")
    if best_name != "identity":
        if conf is None:
            raise ValueError("a proposed candidate must be confirmed")
        _, seeds = check_record(conf, best_name, "arrival_confirmation", cfg["confirmation_pairs"])
        if training_seeds & set(seeds):
            raise ValueError("confirmation seeds overlap the training seeds")
        accepted = confirmed(conf, cfg["min_gain"])
    elif conf is not None:
        raise ValueError("confirmation recorded without a proposed candidate")
    if arr.get("accepted") != accepted or arr.get("identity_fallback") != (not accepted):
        raise ValueError("recorded acceptance differs from the confirmation rule")
    selected = best_name if accepted else "identity"
    if arr.get("selected_candidate") != selected:
        raise ValueError("recorded selection differs from the evidence")
    want = (cands[best_name] if accepted else identity)["arrival_order"]
    if list(plan["arrival_order"]) != list(want):
        raise ValueError("frozen order differs from the selected candidate")
    return dict(selected=selected, proposed=best_name, accepted=accepted, best_training_gain=best_gain)


def fit_role(m, n, k, world, chunk_rows, evaluate, *, config=None, seed=8000000):
    """Fit, confirm and freeze one role plan (timing injected by `evaluate`)."""
    cfg = settings(config)
    initial = make_role(m, n, k, world, chunk_rows)
    trials = []
    best, best_name, best_gain = initial, "identity", 0.0
    for cand in candidates(m, n, k, world, chunk_rows)[1:]:
        plan = make_role(m, n, k, world, chunk_rows, cand["arrival_order"])
        record = paired_measure(initial, plan, evaluate, arm=ARRIVAL_ARM,
                                pairs=cfg["training_pairs"], seed=seed,
                                phase="arrival_training", name=cand["name"])
        trials.append(record)
        if record["fractional_gain"] > max(cfg["min_gain"], best_gain):
            best, best_name, best_gain = plan, cand["name"], record["fractional_gain"]
    confirmation, accepted = None, False
    if best_name != "identity":
        confirmation = paired_measure(initial, best, evaluate, arm=ARRIVAL_ARM,
                                      pairs=cfg["confirmation_pairs"], seed=seed + 1000000,
                                      phase="arrival_confirmation", name=best_name)
        accepted = confirmed(confirmation, cfg["min_gain"])
    if not accepted:
        best = initial
    order = best["arrival_order"]
    final = make_role(m, n, k, world, chunk_rows, order)
    final["diagnostics"] = dict(
        method="same-codec-paired-full-flux-projection-v1", settings=cfg,
        arrival=dict(selected_candidate=best_name if accepted else "identity",
                     proposed_candidate=best_name, accepted=accepted,
                     identity_fallback=not accepted, training_candidates=trials,
                     confirmation=confirmation,
                     changed_slots=sum(a != b for a, b in zip(initial["arrival_order"], order))),
        limitation="Role-shape calibration of the complete fused GemmRS operator; "
                   "not a layer-specific or full-step guarantee.")
    return validate_role_plan(final, m, n, k, world, chunk_rows)
