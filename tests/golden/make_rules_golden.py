"""Golden vectors for the decision rules, produced by the reference demo's own functions.

Run in a container that has the reference checkout (read-only), its root directory in $HSG_REFERENCE:
    HSG_REFERENCE=<reference checkout> python tests/golden/make_rules_golden.py
It imports examples/demo/server.py and records, for seeded logits sequences and a grid of rules, the reference's
first_fire index and its RuleTracker state (fired_k, best_k, best) after every token, into rules_golden.json.
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def rule_grid():
    rules = []
    for score in ("unsafe", "cut"):
        for T in (1.0, 0.5, 2.0):
            rules += [{"rule": "threshold", "score": score, "T": T, "tau": tau, "k": k}
                      for tau in (0.2, 0.5, 0.8) for k in (1, 2, 3)]
            rules += [{"rule": "ema", "score": score, "T": T, "tau": tau, "alpha": a}
                      for tau in (0.3, 0.6) for a in (0.1, 0.5, 1.0)]
            rules += [{"rule": kind, "score": score, "T": T, "tau": 0.5} for kind in ("argmax2", "endpoint", "off")]
    return rules


def sequences():
    rng = np.random.default_rng(11)
    seqs = []
    for n in (0, 1, 2, 5, 17, 40):
        for scale in (0.5, 2.0, 6.0):
            x = rng.normal(size=(n, 3)) * scale
            x[:, 1] += np.linspace(-2, 2, n) if n else 0  # drifting risk so rules fire part-way
            seqs.append(x.round(6).tolist())
    return seqs


def main():
    ref = os.environ.get("HSG_REFERENCE")
    if not ref:
        raise SystemExit("set HSG_REFERENCE to the root of the reference checkout")
    sys.path.insert(0, os.path.join(ref, "examples", "demo"))
    sys.path.insert(0, os.path.join(ref, "src"))
    import server
    seqs, cases = sequences(), []
    for rule_in in rule_grid():
        rule = server.parse_rule(rule_in)
        for si, rows in enumerate(seqs):
            tracker = server.RuleTracker(rule)
            trace = []
            for row in rows:
                tracker.feed(row)
                trace.append([tracker.fired_k, tracker.best_k, round(tracker.best, 12)])
            cases.append({"rule": rule_in, "seq": si, "first_fire": server.first_fire(rows, rule), "trace": trace})
    bad = []
    for value in ({"rule": "nope"}, {"rule": "ema", "alpha": 0.0}, {"rule": "threshold", "k": 300},
                  {"rule": "threshold", "score": "safe"}, [1], {"rule": "ema", "tau": 1.0}):
        try:
            server.parse_rule(value)
        except ValueError:
            bad.append(value)
    with open(os.path.join(HERE, "rules_golden.json"), "w") as f:
        json.dump({"sequences": seqs, "cases": cases, "rejected": bad}, f, separators=(",", ":"))
    print(len(cases), "cases")


if __name__ == "__main__":
    main()
