"""Arrival planning: legality, digests and injected-timing calibration."""
import math

import pytest

from tempname_5090_b200.parallel import planning as pl

SHAPE = (2048, 4096, 512, 8, 128)


def test_candidates_are_legal_and_unique():
    cands = pl.candidates(*SHAPE)
    names = [c["name"] for c in cands]
    assert names[0] == "identity"
    assert len({tuple(c["arrival_order"]) for c in cands}) == len(cands)
    for c in cands:
        pl.make_role(*SHAPE, order=c["arrival_order"])


def test_validation_rejects_destination_change():
    plan = pl.make_role(*SHAPE)
    order = plan["arrival_order"][:]
    order[0], order[1] = order[1], order[0]
    bad = dict(plan, arrival_order=order)
    with pytest.raises(ValueError):
        pl.validate_role_plan(bad, *SHAPE)
    with pytest.raises(ValueError):
        pl.validate_role_plan(dict(plan, diagnostics={"x": math.nan}), *SHAPE)


def test_digest_stable():
    a, b = pl.make_role(*SHAPE), pl.make_role(*SHAPE)
    assert pl.role_digest(a) == pl.role_digest(b)


def _evaluator(gains, calls):
    def evaluate(plan, seed, arm, label):
        calls.append((label, seed))
        name = label.split("/")[1]
        side = label.split("/")[-1]
        base = 1.0
        return base * (1 - gains.get(name, 0.0)) if side == "candidate" else base
    return evaluate


def test_fit_selects_and_confirms_best():
    calls = []
    plan = pl.fit_role(*SHAPE, _evaluator({"reverse_all": 0.05, "rotate": 0.01}, calls),
                       config=dict(training_pairs=2, confirmation_pairs=2))
    arrival = plan["diagnostics"]["arrival"]
    assert arrival["selected_candidate"] == "reverse_all" and arrival["accepted"]
    assert plan["arrival_order"] != pl.base_order(*SHAPE)
    train = {s for l, s in calls if "training" in l}
    confirm = {s for l, s in calls if "confirmation" in l}
    assert train.isdisjoint(confirm)
    orders = [l.split("/")[-1] for l, _ in calls if "pair1" in l and "reverse_all" in l
              and "training" in l]
    assert orders == ["candidate", "reference"]   # BA order on odd pairs


def test_unstable_confirmation_falls_back_to_identity():
    state = {"n": 0}

    def evaluate(plan, seed, arm, label):
        if "confirmation" in label and label.endswith("candidate"):
            return 1.2
        return 0.9 if label.endswith("candidate") and "reverse_all" in label else 1.0
    plan = pl.fit_role(*SHAPE, evaluate)
    assert plan["arrival_order"] == pl.base_order(*SHAPE)
    assert plan["diagnostics"]["arrival"]["identity_fallback"]


def test_numerical_failure_is_fatal():
    def evaluate(plan, seed, arm, label):
        return dict(elapsed_seconds=1.0, correctness_passed=False)
    with pytest.raises(ValueError):
        pl.fit_role(*SHAPE, evaluate)


def _fitted(gains, **cfg):
    return pl.fit_role(*SHAPE, _evaluator(gains, []), config=dict(training_pairs=2, confirmation_pairs=2, **cfg))


def test_replay_of_calibration_evidence_matches_the_frozen_plan():
    accepted = _fitted({"reverse_all": 0.05, "rotate": 0.01})
    assert pl.replay_role_evidence(accepted, *SHAPE)["selected"] == "reverse_all"
    identity = _fitted({})
    assert pl.replay_role_evidence(identity, *SHAPE)["selected"] == "identity"


def _tamper(plan, fn):
    import copy
    p = copy.deepcopy(plan)
    fn(p["diagnostics"]["arrival"], p)
    return p


@pytest.mark.parametrize("what", ["seconds", "gain", "order_swap", "accept_flip", "frozen_order", "seed_reuse",
                                  "drop_candidate", "proposal"])
def test_replay_rejects_doctored_evidence(what):
    plan = _fitted({"reverse_all": 0.05, "rotate": 0.01})

    def edit(arr, p):
        rec = arr["training_candidates"][0]
        if what == "seconds":
            rec["paired_samples"][0]["candidate_seconds"] *= 0.5
        elif what == "gain":
            rec["fractional_gain"] += 0.01
        elif what == "order_swap":
            rec["paired_samples"][1]["execution_order"].reverse()
        elif what == "accept_flip":
            arr["accepted"], arr["identity_fallback"] = False, True
        elif what == "frozen_order":
            p["arrival_order"] = pl.base_order(*SHAPE)
        elif what == "seed_reuse":
            arr["confirmation"]["paired_samples"][0]["seed"] = rec["paired_samples"][0]["seed"]
        elif what == "drop_candidate":
            arr["training_candidates"].pop()
        elif what == "proposal":
            arr["proposed_candidate"] = "rotate"
    with pytest.raises(ValueError):
        pl.replay_role_evidence(_tamper(plan, edit), *SHAPE)
