"""Decision rules over streamed scores: when a conversation's per-token scores should stop (fire on) a response.

Host-side counterpart of the reference demo's rule layer (examples/demo/server.py:59-117 ``parse_rule``,
``probabilities``, ``token_score``, ``first_fire`` and :248-284 ``RuleTracker``). A rule is a dict with

- ``rule``: ``threshold`` (``k`` consecutive tokens above ``tau``), ``ema`` (exponential moving average of the score's
  logit, weight ``alpha``, above logit(``tau``)), ``argmax2`` (the same risky label as arg-max on two consecutive
  tokens), ``endpoint`` (the last token above ``tau``) or ``off``;
- ``score``: ``unsafe`` (p(unsafe)) or ``cut`` (1 - p(safe)), computed after a softmax at temperature ``T``.

The engine returns probabilities, not logits; a probability row p is accepted directly (its log is a logit vector
for the same distribution, so the temperature softmax is unchanged). Trackers are fed one committed token at a time
and keep O(1) state per conversation, so a server can run one per slot beside StreamingGuard.step.
"""
from __future__ import annotations

import math

RULE_KINDS = ("threshold", "ema", "argmax2", "endpoint", "off")


def parse_rule(value):
    """Validated rule dict with defaults (reference server.py:59-71); ValueError on anything else."""
    if not isinstance(value, dict):
        raise ValueError("rule must be an object")
    rule = {"rule": value.get("rule"), "score": value.get("score", "unsafe"), "T": float(value.get("T", 1.0)),
            "tau": float(value.get("tau", 0.5)), "k": int(value.get("k", 1)), "alpha": float(value.get("alpha", 0.1))}
    if rule["rule"] not in RULE_KINDS:
        raise ValueError("unknown rule")
    if rule["score"] not in ("unsafe", "cut"):
        raise ValueError("score must be unsafe or cut")
    in_range = (0 < rule["T"] <= 20, 0 < rule["tau"] < 1, 1 <= rule["k"] <= 256, 0 < rule["alpha"] <= 1)
    if not all(in_range):
        raise ValueError("rule parameters out of range")
    return rule


def softmax_t(logits, temperature):
    """Softmax of ``logits / temperature`` (max-shifted), as floats."""
    z = [x / temperature for x in logits]
    m = max(z)
    e = [math.exp(x - m) for x in z]
    s = sum(e)
    return [x / s for x in e]


def logits_of(probs):
    """A logit vector for a probability row (log p; zero probabilities map to a very negative logit)."""
    return [math.log(p) if p > 0 else -1e30 for p in probs]


def token_score(logits, rule):
    p = softmax_t(logits, rule["T"])
    return p[1] if rule["score"] == "unsafe" else 1.0 - p[0]


def _risky_labels(rule):
    return (1,) if rule["score"] == "unsafe" else (1, 2)


def _argmax3(row):
    best = 0
    for j in (1, 2):
        if row[j] > row[best]:
            best = j
    return best


def first_fire(rows, rule):
    """Index of the first token (of one message's content tokens, in order) at which ``rule`` fires, else -1."""
    kind = rule["rule"]
    if kind == "off" or not rows:
        return -1
    if kind == "endpoint":
        return len(rows) - 1 if token_score(rows[-1], rule) > rule["tau"] else -1
    tracker = RuleTracker(rule)
    for row in rows:
        tracker.feed(row)
        if tracker.fired_k >= 0:
            return tracker.fired_k
    return -1


class RuleTracker:
    """Streaming form of ``first_fire`` plus the running maximum score (reference server.py:248-284).

    ``feed(row)`` takes one token's logits; ``feed_probs(p)`` one token's probabilities. ``fired_k`` is the index of
    the token that fired the rule (-1 while it has not; ``endpoint`` and ``off`` never fire here, a caller applies
    ``endpoint`` at the end of the message), ``best`` / ``best_k`` the maximum score so far and its index.
    """

    def __init__(self, rule):
        self.rule = rule
        self.bound = math.log(rule["tau"] / (1 - rule["tau"]))
        self.reset()

    def reset(self):
        self.count, self.run, self.ema, self.previous = 0, 0, None, None
        self.fired_k, self.best_k, self.best = -1, -1, -1.0

    def feed_probs(self, probs):
        self.feed(logits_of(probs))

    def feed(self, logits):
        rule, index = self.rule, self.count
        s = token_score(logits, rule)
        if s > self.best:
            self.best, self.best_k = s, index
        self.count += 1
        kind = rule["rule"]
        if self.fired_k >= 0 or kind in ("off", "endpoint"):
            return
        if kind == "argmax2":
            label = _argmax3(logits)
            if label in _risky_labels(rule) and label == self.previous:
                self.fired_k = index
            self.previous = label
        elif kind == "threshold":
            self.run = self.run + 1 if s > rule["tau"] else 0
            if self.run >= rule["k"]:
                self.fired_k = index
        else:  # ema of the score's logit
            c = min(max(s, 1e-9), 1 - 1e-9)
            margin = math.log(c / (1 - c))
            self.ema = margin if self.ema is None else rule["alpha"] * margin + (1 - rule["alpha"]) * self.ema
            if self.ema > self.bound:
                self.fired_k = index
