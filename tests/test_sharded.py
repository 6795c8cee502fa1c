"""ShardedGuard host logic on the CPU: slot routing over devices, request order, validation and per-slot resets, with a
fake device tick whose scores depend on the global slot, the position and the token (so any routing or ordering
mistake changes the result)."""
import numpy as np
import pytest

from hs_guard_b200 import DEFAULT
from hs_guard_b200.engine import bucket, default_session_buckets
from hs_guard_b200.runtime import DEFAULT_METADATA, StreamingGuard, validate_requests
from hs_guard_b200.shard import SlotRouter, route, slot_range
from hs_guard_b200.sharded import ShardedGuard


def _safe(slot, pos, tok):
    return np.float32(((int(slot) * 7919 + int(pos) * 31 + int(tok)) % 997) / 997.0)


class _FakeEngine:
    """The part of SlotEngine that StreamingGuard uses, for slots [lo, lo + n) of a global range."""

    def __init__(self, n, lo=0):
        self.max_slots, self.lo, self.roles, self.cfg = n, lo, ("user", "assistant"), DEFAULT
        self.session_buckets = default_session_buckets(n)
        self.length = np.zeros(n, dtype=np.int64)
        self.calls = 0

    def run_requests(self, requests):
        return None  # the Python tick path

    def fits_one_tick(self, requests):
        return len(requests) <= self.session_buckets[-1] and all(len(ids) <= 64 for _, ids in requests)

    def run_arrays(self, chunks, slots):
        self.calls += 1
        lb = bucket(max(len(c) for c in chunks), (1, 2, 4, 8, 16, 32, 64))
        probs = np.zeros((2, len(chunks), lb, 3), np.float32)
        lens = np.array([len(c) for c in chunks], np.int64)
        for row, (c, s) in enumerate(zip(chunks, slots)):
            for t, tok in enumerate(c):
                p = _safe(self.lo + int(s), self.length[int(s)] + t, tok)
                probs[:, row, t] = [[p, 1 - p, 0], [p / 2, 1 - p / 2, 0]]
        self.length[np.asarray(slots, dtype=np.int64)] += lens
        return probs, lens

    def run_tokens(self, slots, ids):
        return self.run_arrays([[i] for i in ids], slots)

    def tick(self, requests):
        return self.run_arrays([ids for _, ids in requests], [s for s, _ in requests])

    def step(self, requests):
        out = {r: [] for r in self.roles}
        for s, ids in requests:  # long requests one at a time, 64 tokens a tick
            parts = [self.run_arrays([ids[i:i + 64]], [s])[0] for i in range(0, len(ids), 64)]
            for r, role in enumerate(self.roles):
                out[role].append(np.concatenate([p[r, 0, :min(64, len(ids) - 64 * k)] for k, p in enumerate(parts)]))
        return out

    def reset(self):
        self.length[:] = 0

    def reset_slot(self, slot):
        self.length[slot] = 0


def _sharded(sizes):
    guards, lo = [], 0
    for n in sizes:
        guards.append(StreamingGuard.from_engine(_FakeEngine(n, lo), DEFAULT_METADATA))
        lo += n
    return ShardedGuard.from_guards(guards, DEFAULT_METADATA)


def _expected(requests, length, role):
    r = 0 if role == "user" else 1
    out = []
    for s, ids in requests:
        cut = [float(1 - (p if r == 0 else p / 2)) for p in (_safe(s, length[s] + t, tok) for t, tok in enumerate(ids))]
        out.append({"slot": s, "cut_scores": cut, "threshold": DEFAULT_METADATA["thresholds"][role]})
        length[s] += len(ids)
    return out


def test_router_matches_route():
    for world, total in ((1, 5), (2, 704), (3, 100), (8, 2816)):
        router = SlotRouter(world, total)
        for s in range(0, total, 7):
            assert router(s) == route(s, world, total)
        with pytest.raises(ValueError):
            router(total)


def test_sharded_step_routes_and_keeps_request_order():
    g = _sharded([3, 3, 2])
    rng = np.random.default_rng(0)
    length = np.zeros(8, dtype=np.int64)
    ticks = [[(s, [int(rng.integers(0, 1000))]) for s in (7, 0, 4, 3, 1)],        # spread over the three devices
             [(5, [int(x) for x in rng.integers(0, 1000, 9)]), (2, [3, 4])],        # multi-token
             [(6, [int(x) for x in rng.integers(0, 1000, 70)])],                    # one device, > 64 tokens
             [(True, [5]), (4, [6])]]                                              # bool slot, as the reference allows
    for k, tick in enumerate(ticks):
        role = "user" if k % 2 else "assistant"
        got = g.step(tick, role)
        want = _expected([(int(s), ids) for s, ids in tick], length, role)
        assert [r["slot"] for r in got] == [s for s, _ in tick]
        for a, b in zip(got, want):
            np.testing.assert_allclose(a["cut_scores"], b["cut_scores"], rtol=0, atol=1e-6)
            assert a["threshold"] == b["threshold"]
    lengths = np.concatenate([gd.engine.length for gd in g.guards])
    np.testing.assert_array_equal(lengths, length)
    g.reset_slot(6)
    assert g.guards[2].engine.length[0] == 0 and g.guards[2].engine.length[1] == length[7]
    g.reset()
    assert not any(gd.engine.length.any() for gd in g.guards)
    g.close()


def test_sharded_errors_match_reference_without_device_calls():
    g = _sharded([2, 2])
    V = DEFAULT.vocab
    for tick, role in (([], "user"), ([(0, [1]), (0, [2])], "user"), ([(4, [1])], "user"), ([(1, [V])], "user"),
                       ([(3, [])], "user"), ([(2, [1.0])], "user"), ([(0, [1])], "system"),
                       ([(3, [1, -1]), (9, [1])], "user")):
        with pytest.raises(ValueError) as got:
            g.step(tick, role)
        with pytest.raises(ValueError) as want:
            validate_requests(tick, role, 4, V)
        assert str(got.value) == str(want.value)
    assert all(gd.engine.calls == 0 for gd in g.guards)
    g.close()


def test_block_ranges_cover_the_slots():
    g = _sharded([2, 3, 1])
    assert g.ranges == [(0, 2), (2, 5), (5, 6)] and g.max_slots == 6
    assert [g.route(s) for s in range(6)] == [(0, 0), (0, 1), (1, 0), (1, 1), (1, 2), (2, 0)]
    assert slot_range(1, 2, 5) == (3, 5)
    g.close()
