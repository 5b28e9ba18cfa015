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
    """Stand-in timings: the challenger of candidate `name` is `gains[name]` faster."""
    def evaluate(plan, seed, arm, label):
        calls.append((label, seed))
        stage, name, index, side = label.split(":")
        return 1.0 - gains.get(name, 0.0) if side == "challenger" else 1.0
    return evaluate


def test_fit_selects_and_confirms_best():
    calls = []
    plan = pl.fit_role(*SHAPE, _evaluator({"reverse_all": 0.05, "rotate": 0.01}, calls),
                       config=dict(training_pairs=2, confirmation_pairs=2))
    d = plan["diagnostics"]
    assert d["selected"] == "reverse_all" and d["accepted"] and d["proposal"] == "reverse_all"
    assert plan["arrival_order"] != pl.base_order(*SHAPE)
    train = {s for l, s in calls if l.startswith("training")}
    confirm = {s for l, s in calls if l.startswith("confirmation")}
    assert train.isdisjoint(confirm)
    sides = [l.split(":")[-1] for l, _ in calls if l.startswith("training:reverse_all:1:")]
    assert sides == ["challenger", "baseline"]   # BA order on odd pairs
    sides = [l.split(":")[-1] for l, _ in calls if l.startswith("training:reverse_all:0:")]
    assert sides == ["baseline", "challenger"]
    # both sides of one pair see the same inputs
    seeds = {s for l, s in calls if l.startswith("training:reverse_all:1:")}
    assert len(seeds) == 1


def test_geometric_gain_and_confirmation_rule():
    rec = dict(gain=pl.geometric_gain([0.9, 0.8]), pairs=[dict(gain=0.1), dict(gain=0.2)])
    assert abs(rec["gain"] - (1 - math.sqrt(0.72))) < 1e-15
    assert pl.confirmed(rec, 0.05)
    rec["pairs"][1]["gain"] = 0.001  # one weak pair vetoes the candidate
    assert not pl.confirmed(rec, 0.05)


def test_family_orders_keep_every_slot_destination():
    m, n, k, world, chunk = SHAPE
    per = m // world // chunk
    for cand in pl.candidates(*SHAPE):
        order = cand["arrival_order"]
        assert all(block // per == slot % world for slot, block in enumerate(order))
    names = [c["name"] for c in pl.candidates(3 * 8 * 128, 4096, 512, 8, 128)]
    assert names == ["identity", "reverse_all", "reverse_odd", "reverse_even", "rotate"]
    # two blocks per destination: rotating is reversing, listed once
    assert [c["name"] for c in pl.candidates(*SHAPE)] == ["identity", "reverse_all", "reverse_odd", "reverse_even"]
    # one block per destination: every rule collapses to the identity
    assert [c["name"] for c in pl.candidates(1024, 4096, 512, 8, 128)] == ["identity"]


def test_a_plan_in_the_other_implementations_layout_is_accepted():
    """Plans exchanged with the reference carry the same four fields; their
    diagnostics are opaque to validation."""
    order = pl.candidates(*SHAPE)[2]["arrival_order"]
    foreign = dict(shape=list(SHAPE[:3]), chunk_rows=SHAPE[4], arrival_order=order,
                   diagnostics=dict(method="other-implementation", arrival=dict(selected_candidate="reverse_odd")))
    assert pl.validate_role_plan(foreign, *SHAPE) is foreign
    with pytest.raises(ValueError):
        pl.validate_role_plan(dict(foreign, extra=1), *SHAPE)


def test_unstable_confirmation_falls_back_to_identity():
    def evaluate(plan, seed, arm, label):
        stage, name, index, side = label.split(":")
        if stage == "confirmation" and side == "challenger":
            return 1.2
        return 0.9 if side == "challenger" and name == "reverse_all" else 1.0
    plan = pl.fit_role(*SHAPE, evaluate)
    assert plan["arrival_order"] == pl.base_order(*SHAPE)
    d = plan["diagnostics"]
    assert d["proposal"] == "reverse_all" and not d["accepted"] and d["selected"] == "identity"


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
    fn(p["diagnostics"], p)
    return p


@pytest.mark.parametrize("what", ["seconds", "gain", "order_swap", "accept_flip", "frozen_order", "seed_reuse",
                                  "drop_candidate", "proposal", "digest", "settings"])
def test_replay_rejects_doctored_evidence(what):
    plan = _fitted({"reverse_all": 0.05, "rotate": 0.01})

    def edit(d, p):
        rec = d["trials"][0]
        if what == "seconds":
            rec["pairs"][0]["challenger_s"] *= 0.5
        elif what == "gain":
            rec["gain"] += 0.01
        elif what == "order_swap":
            rec["pairs"][1]["first"] = "baseline"
        elif what == "accept_flip":
            d["accepted"], d["selected"] = False, "identity"
        elif what == "frozen_order":
            p["arrival_order"] = pl.base_order(*SHAPE)
        elif what == "seed_reuse":
            d["confirmation"]["pairs"][0]["seed"] = rec["pairs"][0]["seed"]
        elif what == "drop_candidate":
            d["trials"].pop()
        elif what == "proposal":
            d["proposal"] = "rotate"
        elif what == "digest":
            rec["challenger_sha256"] = "0" * 64
        elif what == "settings":
            d["settings"]["min_gain"] = 0.2
    with pytest.raises(ValueError):
        pl.replay_role_evidence(_tamper(plan, edit), *SHAPE)
