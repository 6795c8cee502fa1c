"""Decision rules (hs_guard_b200.rules) against golden vectors from the reference demo's own first_fire and
RuleTracker (tests/golden/make_rules_golden.py)."""
import json
import math
import os

import pytest

from hs_guard_b200.rules import RuleTracker, first_fire, parse_rule, softmax_t

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "rules_golden.json")))


def test_first_fire_and_tracker_match_reference():
    assert len(GOLDEN["cases"]) > 1000
    for case in GOLDEN["cases"]:
        rule, rows = parse_rule(case["rule"]), GOLDEN["sequences"][case["seq"]]
        assert first_fire(rows, rule) == case["first_fire"], case["rule"]
        tracker = RuleTracker(rule)
        for row, (fired_k, best_k, best) in zip(rows, case["trace"]):
            tracker.feed(row)
            assert (tracker.fired_k, tracker.best_k) == (fired_k, best_k)
            assert tracker.best == pytest.approx(best, abs=1e-11)


def test_rejected_rules():
    for value in GOLDEN["rejected"]:
        with pytest.raises(ValueError):
            parse_rule(value)


def test_probability_rows_are_equivalent_to_logits():
    """feed_probs(softmax(z)) scores like feed(z): the engine's probability output can drive a tracker."""
    for case in GOLDEN["cases"][::37]:
        rule = parse_rule(case["rule"])
        a, b = RuleTracker(rule), RuleTracker(rule)
        for row in GOLDEN["sequences"][case["seq"]]:
            a.feed(row)
            b.feed_probs(softmax_t(row, 1.0))
            assert a.fired_k == b.fired_k and a.best_k == b.best_k
            assert math.isclose(a.best, b.best, rel_tol=1e-9, abs_tol=1e-12)
