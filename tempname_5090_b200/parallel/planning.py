"""Arrival plans of the arrival-first arm (`flux_taco_interleaved_arrival`).

A plan says, for one projection role (a GemmRS shape), in which order the
producer emits the physical row blocks.  The order must keep the interleaved
arm's destination rotation (slot s serves destination s % W), so a plan only
permutes, per destination, the sequence of that destination's own blocks.

Fitting a plan is an experiment, not a guess:

* a small family of per-destination permutations is tried against the
  interleaved identity order;
* every comparison runs complete fused operators in AB/BA-alternated pairs on
  identical inputs (the pair's seed), and scores the challenger by the
  geometric mean of its time ratios;
* the best challenger above the bar is re-measured on inputs that training
  never used, and is frozen only if that confirmation clears the bar overall
  and in every single pair; otherwise the identity order is frozen.

The evidence (every raw time, seed and execution order) is stored in the
plan's diagnostics, and `replay_role_evidence` re-derives the decision from it.

Interface kept identical to TempName-5090 python/flux_5090/planning.py so a
plan from either implementation is accepted by the other: the plan fields
(`shape`, `chunk_rows`, `arrival_order`, `diagnostics`), the schema name, the
five-candidate family, the AB/BA geometric-mean gain and the confirmation rule.
Everything else (structure, seeds, diagnostics) is this module's own.
"""
from __future__ import annotations

import hashlib
import json
import math
from dataclasses import asdict, dataclass

SCHEMA = "rtx5090-arrival-plan-v1"
ARRIVAL_ARM = "flux_taco_interleaved_arrival"
PLAN_FIELDS = frozenset({"shape", "chunk_rows", "arrival_order", "diagnostics"})
EVIDENCE = "b200-paired-arrival-fit-v1"

# The candidate family: per destination d (of W) with `per` blocks each, the
# permutation of its blocks' sequence.  The identity comes first.
FAMILY = (
    ("identity", lambda d, per: list(range(per))),
    ("reverse_all", lambda d, per: list(range(per - 1, -1, -1))),
    ("reverse_odd", lambda d, per: list(range(per - 1, -1, -1)) if d & 1 else list(range(per))),
    ("reverse_even", lambda d, per: list(range(per)) if d & 1 else list(range(per - 1, -1, -1))),
    ("rotate", lambda d, per: [(i + 1) % per for i in range(per)]),
)


def role_digest(obj) -> str:
    """SHA-256 of the canonical JSON text (rejects NaN and non-JSON values)."""
    text = json.dumps(obj, sort_keys=True, separators=(",", ":"), allow_nan=False)
    return hashlib.sha256(text.encode()).hexdigest()


@dataclass(frozen=True)
class RoleGeometry:
    """Block structure of one GemmRS role: M rows cut into chunk_rows blocks, W owners."""
    m: int
    n: int
    k: int
    world: int
    chunk_rows: int

    def __post_init__(self):
        if any(type(v) is not int or v <= 0 for v in asdict(self).values()):
            raise ValueError(f"role geometry needs positive integers, got {asdict(self)}")
        if self.world < 2:
            raise ValueError("an arrival plan needs at least two ranks")
        if self.chunk_rows % 128 or self.n % 128 or self.k % 8 or self.m % (self.world * self.chunk_rows):
            raise ValueError(f"role geometry {asdict(self)}: chunk_rows and N must be multiples of 128, K of 8, "
                             "and M of world * chunk_rows")

    @property
    def per(self) -> int:
        """Blocks per destination."""
        return self.m // (self.world * self.chunk_rows)

    def compose(self, permutation) -> list:
        """Slot order from a per-destination permutation rule: slot w*W + d emits
        destination d's block permutation(d)[w]."""
        seqs = [permutation(d, self.per) for d in range(self.world)]
        return [d * self.per + seqs[d][w] for w in range(self.per) for d in range(self.world)]

    def identity(self) -> list:
        return self.compose(FAMILY[0][1])

    def check_order(self, order) -> None:
        count = self.per * self.world
        if not isinstance(order, list) or len(order) != count or any(type(b) is not int for b in order):
            raise ValueError(f"arrival order must list {count} integer block ids")
        if sorted(order) != list(range(count)):
            raise ValueError("arrival order is not a permutation of the physical blocks")
        moved = [slot for slot, block in enumerate(order) if block // self.per != slot % self.world]
        if moved:
            raise ValueError(f"arrival order moves slot {moved[0]} to another destination")


def base_order(m, n, k, world, chunk_rows) -> list:
    """The interleaved identity order (slot s -> (s % W) * per + s // W)."""
    return RoleGeometry(m, n, k, world, chunk_rows).identity()


def candidates(m, n, k, world, chunk_rows) -> list:
    """Distinct orders of the family, identity first: [{name, arrival_order}]."""
    geo = RoleGeometry(m, n, k, world, chunk_rows)
    seen, out = set(), []
    for name, rule in FAMILY:
        order = geo.compose(rule)
        if tuple(order) in seen:
            continue  # e.g. with one block per destination every rule is the identity
        seen.add(tuple(order))
        out.append(dict(name=name, arrival_order=order))
    return out


def validate_role_plan(plan, m=None, n=None, k=None, world=None, chunk_rows=None, *,
                       shape=None, world_size=None):
    """Check a plan (from either implementation) against the operator it drives."""
    if shape is not None:
        if m is not None or n is not None or k is not None:
            raise ValueError("give the shape either as shape=[M, N, K] or as M, N, K")
        if not isinstance(shape, (list, tuple)) or len(shape) != 3:
            raise ValueError("shape must be [M, N, K]")
        m, n, k = shape
    if world_size is not None:
        if world is not None and world != world_size:
            raise ValueError("world and world_size disagree")
        world = world_size
    geo = RoleGeometry(m, n, k, world, chunk_rows)
    if not isinstance(plan, dict) or set(plan) != PLAN_FIELDS:
        got = sorted(plan) if isinstance(plan, dict) else type(plan).__name__
        raise ValueError(f"a role plan has exactly the fields {sorted(PLAN_FIELDS)}, got {got}")
    if plan["shape"] != [m, n, k] or plan["chunk_rows"] != chunk_rows:
        raise ValueError(f"plan is for shape {plan['shape']} / chunk_rows {plan['chunk_rows']}, "
                         f"operator is {[m, n, k]} / {chunk_rows}")
    geo.check_order(plan["arrival_order"])
    if not isinstance(plan["diagnostics"], dict):
        raise ValueError("plan diagnostics must be a JSON object")
    role_digest(plan)
    return plan


def make_role(m, n, k, world, chunk_rows, order=None):
    geo = RoleGeometry(m, n, k, world, chunk_rows)
    plan = dict(shape=[m, n, k], chunk_rows=chunk_rows,
                arrival_order=list(geo.identity() if order is None else order), diagnostics={})
    return validate_role_plan(plan, m, n, k, world, chunk_rows)


# ------------------------------------------------------------------ settings
@dataclass(frozen=True)
class Settings:
    """Calibration budget.  Key names are the reference configs' keys."""
    warmup: int = 2
    iterations: int = 5
    training_pairs: int = 3
    confirmation_pairs: int = 3
    min_gain: float = 0.002

    @classmethod
    def parse(cls, values=None) -> "Settings":
        values = {} if values is None else values
        if not isinstance(values, dict):
            raise ValueError("calibration settings must be a dictionary")
        unknown = set(values) - set(cls.__dataclass_fields__)
        if unknown:
            raise ValueError(f"unknown calibration settings {sorted(unknown)}")
        s = cls(**values)
        for name, lowest in (("warmup", 0), ("iterations", 1), ("training_pairs", 1), ("confirmation_pairs", 1)):
            v = getattr(s, name)
            if type(v) is not int or v < lowest:
                raise ValueError(f"calibration {name} must be an integer >= {lowest}, got {v!r}")
        if type(s.min_gain) not in (int, float) or not (0 <= s.min_gain < 1) or not math.isfinite(s.min_gain):
            raise ValueError(f"calibration min_gain must be in [0, 1), got {s.min_gain!r}")
        return cls(**{**asdict(s), "min_gain": float(s.min_gain)})


def settings(values=None) -> dict:
    return asdict(Settings.parse(values))


# -------------------------------------------------------------- measurement
def _seconds(measured) -> float:
    """An evaluator returns seconds, or a dict with `elapsed_seconds` and an
    optional `correctness_passed` that must be true."""
    if isinstance(measured, dict):
        if measured.get("correctness_passed", True) is not True:
            raise ValueError("a calibration candidate failed its numerical gate")
        measured = measured.get("elapsed_seconds")
    if type(measured) not in (int, float) or not math.isfinite(measured) or measured <= 0:
        raise ValueError(f"calibration timings must be positive finite seconds, got {measured!r}")
    return float(measured)


def pair_seeds(base: int, candidate_index: int, stage: str, count: int) -> list:
    """Input seeds of one comparison: training pairs take even offsets and
    confirmation pairs odd ones, in a block per candidate, so the two stages
    never share inputs."""
    parity = 0 if stage == "training" else 1
    return [base + 4096 * candidate_index + 2 * p + parity for p in range(count)]


def geometric_gain(ratios) -> float:
    """1 - geometric mean of challenger / baseline times."""
    ratios = list(ratios)
    return 1.0 - math.exp(sum(math.log(r) for r in ratios) / len(ratios))


def compare(baseline, challenger, evaluate, *, stage, name, seeds, arm=ARRIVAL_ARM) -> dict:
    """AB/BA-paired timing of two plans: pair p runs both sides on seed p's
    inputs, baseline first on even pairs and challenger first on odd ones.
    `evaluate(plan, seed, arm, label)` times one complete fused operator."""
    pairs = []
    for index, seed in enumerate(seeds):
        first = "baseline" if index % 2 == 0 else "challenger"
        times = {}
        for side in ((first, "challenger") if first == "baseline" else (first, "baseline")):
            plan = baseline if side == "baseline" else challenger
            times[side] = _seconds(evaluate(plan, seed, arm, f"{stage}:{name}:{index}:{side}"))
        pairs.append(dict(index=index, seed=seed, first=first, baseline_s=times["baseline"],
                          challenger_s=times["challenger"],
                          gain=1.0 - times["challenger"] / times["baseline"]))
    return dict(stage=stage, candidate=name, pairs=pairs,
                gain=geometric_gain(p["challenger_s"] / p["baseline_s"] for p in pairs),
                weakest_pair_gain=min(p["gain"] for p in pairs),
                baseline_sha256=role_digest(baseline), challenger_sha256=role_digest(challenger))


def confirmed(record, minimum_gain) -> bool:
    """The confirmation rule: the overall gain and every pair's gain exceed the bar."""
    return record["gain"] > minimum_gain and all(p["gain"] > minimum_gain for p in record["pairs"])


def fit_role(m, n, k, world, chunk_rows, evaluate, *, config=None, seed=8000000):
    """Fit, confirm and freeze one role's arrival plan from measured timings."""
    cfg = Settings.parse(config)
    identity = make_role(m, n, k, world, chunk_rows)
    family = candidates(m, n, k, world, chunk_rows)
    trials, proposal, proposal_gain = [], None, cfg.min_gain
    for index, cand in enumerate(family[1:], start=1):
        challenger = make_role(m, n, k, world, chunk_rows, cand["arrival_order"])
        trial = compare(identity, challenger, evaluate, stage="training", name=cand["name"],
                        seeds=pair_seeds(seed, index, "training", cfg.training_pairs))
        trials.append(trial)
        if trial["gain"] > proposal_gain:
            proposal, proposal_gain = (index, cand, challenger), trial["gain"]
    confirmation, accepted, selected = None, False, "identity"
    if proposal is not None:
        index, cand, challenger = proposal
        confirmation = compare(identity, challenger, evaluate, stage="confirmation", name=cand["name"],
                               seeds=pair_seeds(seed, index, "confirmation", cfg.confirmation_pairs))
        accepted = confirmed(confirmation, cfg.min_gain)
        if accepted:
            selected = cand["name"]
    order = next(c["arrival_order"] for c in family if c["name"] == selected)
    plan = make_role(m, n, k, world, chunk_rows, order)
    plan["diagnostics"] = dict(
        evidence=EVIDENCE, settings=asdict(cfg), seed_base=seed, trials=trials,
        proposal=None if proposal is None else proposal[1]["name"], confirmation=confirmation,
        accepted=accepted, selected=selected,
        moved_slots=sum(a != b for a, b in zip(identity["arrival_order"], order)),
        scope="timed on the complete fused GemmRS of this role's shape; says nothing about other shapes "
              "or about a full training step")
    return validate_role_plan(plan, m, n, k, world, chunk_rows)


# ------------------------------------------------------------------- replay
def replay_role_evidence(plan, m, n, k, world, chunk_rows) -> dict:
    """Re-derive a frozen plan's decision from its own diagnostics: every pair
    gain and every comparison's geometric-mean gain from the recorded seconds,
    the AB/BA alternation, the seeds (training and confirmation disjoint), the
    orders compared (digests), the proposal (best training gain above the bar),
    the confirmation rule and the frozen order.  Raises ValueError on any
    mismatch; returns the recomputed decision (the counterpart of the
    reference report's calibration replay, tools/5090/report.py:214-269)."""
    plan = validate_role_plan(plan, m, n, k, world, chunk_rows)
    d = plan["diagnostics"]
    if d.get("evidence") != EVIDENCE:
        raise ValueError("the plan carries no calibration evidence of this framework")
    cfg = Settings.parse(d.get("settings"))
    base = d.get("seed_base")
    if type(base) is not int:
        raise ValueError("calibration evidence lacks its seed base")
    identity = make_role(m, n, k, world, chunk_rows)
    family = candidates(m, n, k, world, chunk_rows)
    plans = {c["name"]: make_role(m, n, k, world, chunk_rows, c["arrival_order"]) for c in family}
    index_of = {c["name"]: i for i, c in enumerate(family)}

    def recheck(trial, stage, count):
        name = trial.get("candidate")
        if trial.get("stage") != stage or name not in plans or name == "identity":
            raise ValueError(f"unexpected {stage} comparison {name!r}")
        want_seeds = pair_seeds(base, index_of[name], stage, count)
        pairs = trial.get("pairs")
        if not isinstance(pairs, list) or [p.get("seed") for p in pairs] != want_seeds:
            raise ValueError(f"{stage} comparison of {name} used other inputs than its seeds")
        ratios = []
        for i, p in enumerate(pairs):
            if p.get("index") != i or p.get("first") != ("baseline" if i % 2 == 0 else "challenger"):
                raise ValueError(f"{stage} comparison of {name} is not AB/BA alternated")
            b, c = _seconds(p.get("baseline_s")), _seconds(p.get("challenger_s"))
            if abs((1.0 - c / b) - p.get("gain", math.nan)) > 1e-12:
                raise ValueError(f"{stage} pair {i} of {name}: recorded gain differs from its seconds")
            ratios.append(c / b)
        gain = geometric_gain(ratios)
        if abs(gain - trial.get("gain", math.nan)) > 1e-12:
            raise ValueError(f"{stage} comparison of {name}: recorded gain differs from its pairs")
        if trial.get("baseline_sha256") != role_digest(identity) or \
                trial.get("challenger_sha256") != role_digest(plans[name]):
            raise ValueError(f"{stage} comparison of {name} timed other orders than the family's")
        return name, gain

    trials = d.get("trials")
    if not isinstance(trials, list) or sorted(t.get("candidate") for t in trials) != \
            sorted(c["name"] for c in family[1:]):
        raise ValueError("training does not cover exactly the candidate family")
    proposal, best = None, cfg.min_gain
    for trial in trials:
        name, gain = recheck(trial, "training", cfg.training_pairs)
        if gain > best:
            proposal, best = name, gain
    if d.get("proposal") != proposal:
        raise ValueError(f"recorded proposal {d.get('proposal')!r} is not the best training gain ({proposal!r})")
    accepted = False
    conf = d.get("confirmation")
    if proposal is None:
        if conf is not None:
            raise ValueError("a confirmation was recorded without a proposal")
    else:
        if not isinstance(conf, dict):
            raise ValueError("the proposal was never confirmed")
        name, _ = recheck(conf, "confirmation", cfg.confirmation_pairs)
        if name != proposal:
            raise ValueError("the confirmation measured another candidate than the proposal")
        accepted = confirmed(conf, cfg.min_gain)
    selected = proposal if accepted else "identity"
    if d.get("accepted") is not accepted or d.get("selected") != selected:
        raise ValueError("recorded acceptance differs from the confirmation rule")
    if plan["arrival_order"] != plans[selected]["arrival_order"]:
        raise ValueError("the frozen order is not the selected candidate's")
    return dict(selected=selected, proposed=proposal or "identity", accepted=accepted,
                best_training_gain=best if proposal else 0.0)
