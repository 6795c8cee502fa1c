"""Decision rules over streamed scores: when a conversation's per-token scores should stop (fire on) a response.

Host-side layer with the decision semantics of the reference demo (examples/demo/server.py:59-117 ``parse_rule``,
``token_score``, ``first_fire``; :248-284 ``RuleTracker``), which golden vectors produced by those functions pin
(tests/golden/make_rules_golden.py). A rule is a dict:

- ``rule``: ``threshold`` (``k`` consecutive tokens whose score exceeds ``tau``), ``ema`` (an exponential moving
  average, weight ``alpha``, of the score's logit exceeds logit(``tau``)), ``argmax2`` (two consecutive tokens share
  the same risky arg-max label), ``endpoint`` (the message's last token exceeds ``tau``) or ``off``;
- ``score``: ``unsafe`` (p(unsafe)) or ``cut`` (1 - p(safe)) of a softmax at temperature ``T``.

Here a tracker is a running maximum plus one small detector object per rule kind, each fed (score, row) per token,
so a server keeps O(1) state per conversation beside StreamingGuard.step. The engine returns probabilities, not
logits; a probability row is accepted through ``feed_probs`` (its log is a logit vector of the same distribution, so
the tempered softmax is unchanged).
"""
from __future__ import annotations

import math

RULE_KINDS = ("threshold", "ema", "argmax2", "endpoint", "off")
SCORE_KINDS = ("unsafe", "cut")
# numeric parameters: (key, default, conversion, lower bound, lower bound allowed, upper bound, upper bound allowed)
_NUMERIC = (("T", 1.0, float, 0.0, False, 20.0, True),
            ("tau", 0.5, float, 0.0, False, 1.0, False),
            ("k", 1, int, 1, True, 256, True),
            ("alpha", 0.1, float, 0.0, False, 1.0, True))
_CLAMP = 1e-9  # scores are kept inside (0, 1) before taking their logit


def _within(x, lo, lo_ok, hi, hi_ok):
    return (x >= lo if lo_ok else x > lo) and (x <= hi if hi_ok else x < hi)


def parse_rule(value):
    """A validated rule dict with every parameter present (defaults filled in); ValueError for anything else."""
    if not isinstance(value, dict):
        raise ValueError("a rule must be a JSON object")
    numbers = {key: conv(value.get(key, default)) for key, default, conv, *_ in _NUMERIC}
    kind, score = value.get("rule"), value.get("score", "unsafe")
    if kind not in RULE_KINDS:
        raise ValueError(f"unknown rule kind {kind!r}")
    if score not in SCORE_KINDS:
        raise ValueError(f"score must be one of {SCORE_KINDS}")
    outside = [key for key, _, _, *bounds in _NUMERIC if not _within(numbers[key], *bounds)]
    if outside:
        raise ValueError("rule parameters out of range: " + ", ".join(outside))
    return {"rule": kind, "score": score, **numbers}


def softmax_t(logits, temperature):
    """Softmax of ``logits / temperature``, shifted by the maximum, as a list of floats."""
    scaled = [x / temperature for x in logits]
    shift = max(scaled)
    weights = [math.exp(x - shift) for x in scaled]
    total = sum(weights)
    return [w / total for w in weights]


def logits_of(probs):
    """A logit vector for a probability row (log p; a zero probability maps to a very negative logit)."""
    return [math.log(p) if p > 0 else -1e30 for p in probs]


def token_score(logits, rule):
    """The rule's score of one token: p(unsafe), or 1 - p(safe), after the tempered softmax."""
    p = softmax_t(logits, rule["T"])
    return p[1] if rule["score"] == "unsafe" else 1.0 - p[0]


def _logit(p):
    return math.log(p / (1 - p))


def _top_label(row):
    """Index of the first maximal entry of a 3-class row."""
    top = 0
    for j in range(1, 3):
        if row[j] > row[top]:
            top = j
    return top


class _ConsecutiveAbove:
    """Fires once ``k`` scores in a row exceed ``tau``."""

    def __init__(self, rule):
        self.tau, self.k, self.streak = rule["tau"], rule["k"], 0

    def update(self, score, row):
        self.streak = self.streak + 1 if score > self.tau else 0
        return self.streak >= self.k


class _LogitAverage:
    """Fires once the exponential moving average of the clamped score's logit exceeds logit(tau); the average
    starts at the first token's logit."""

    def __init__(self, rule):
        self.alpha, self.bound, self.value = rule["alpha"], _logit(rule["tau"]), None

    def update(self, score, row):
        x = _logit(min(max(score, _CLAMP), 1 - _CLAMP))
        self.value = x if self.value is None else self.alpha * x + (1 - self.alpha) * self.value
        return self.value > self.bound


class _RepeatedRiskyLabel:
    """Fires when a token's arg-max label is risky (unsafe; with the cut score also controversial) and equals the
    previous token's label."""

    def __init__(self, rule):
        self.risky = (1,) if rule["score"] == "unsafe" else (1, 2)
        self.last = None

    def update(self, score, row):
        label = _top_label(row)
        fired = label in self.risky and label == self.last
        self.last = label
        return fired


_DETECTORS = {"threshold": _ConsecutiveAbove, "ema": _LogitAverage, "argmax2": _RepeatedRiskyLabel}


class RuleTracker:
    """Feeds one committed token at a time: ``fired_k`` is the index of the token at which the rule fired (-1 until
    then; ``endpoint`` and ``off`` never fire here, a caller applies ``endpoint`` at the end of the message), ``best``
    and ``best_k`` the largest score so far and the first index where it was reached (``best`` starts at -1)."""

    def __init__(self, rule):
        self.rule = rule
        self.reset()

    def reset(self):
        make = _DETECTORS.get(self.rule["rule"])
        self._detector = make(self.rule) if make else None
        self.count, self.fired_k, self.best_k, self.best = 0, -1, -1, -1.0

    def feed_probs(self, probs):
        self.feed(logits_of(probs))

    def feed(self, logits):
        index = self.count
        self.count += 1
        score = token_score(logits, self.rule)
        if score > self.best:
            self.best, self.best_k = score, index
        if self.fired_k < 0 and self._detector is not None and self._detector.update(score, logits):
            self.fired_k = index


def first_fire(rows, rule):
    """Index of the first token (of one message's content tokens, in order) at which ``rule`` fires, else -1."""
    if rule["rule"] == "off" or not rows:
        return -1
    if rule["rule"] == "endpoint":
        return len(rows) - 1 if token_score(rows[-1], rule) > rule["tau"] else -1
    tracker = RuleTracker(rule)
    for row in rows:
        tracker.feed(row)
        if tracker.fired_k >= 0:
            break
    return tracker.fired_k
