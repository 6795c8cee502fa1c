"""Host-side logic on the CPU: packing, validation, buckets, weight layout, slot sharding, and the C ABI surface."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from golden_inputs import stream_script
from hs_guard_b200 import DEFAULT, HsgConfig
from hs_guard_b200 import weights as W
from hs_guard_b200.engine import bucket, default_session_buckets
from hs_guard_b200.pack import pack_inputs
from hs_guard_b200.runtime import validate_requests
from hs_guard_b200.shard import route, slot_range, split_requests
from oracle.pack import pack_inputs as oracle_pack

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_pack_matches_oracle_and_reference_cases(golden):
    cases = [([[4, 5, 6]], [0], 2, 4, [7], 1),
             ([[1], [2], [3]], [2, 0, 1], 4, 1, [5, 0, 9], 3),
             ([[10, 11], [12, 13, 14, 15, 16], [17]], [1, 3, 0], 4, 8, [100, 3, 0, 511], 4)]
    for i, (chunks, slots, nb, lb, length, max_slots) in enumerate(cases):
        buf = np.full(nb * lb + 3 * nb, -7, dtype=np.int64)
        lens = pack_inputs(chunks, slots, nb, lb, np.asarray(length), max_slots, buf)
        np.testing.assert_array_equal(buf, golden[f"pack{i}_out"])
        np.testing.assert_array_equal(lens, golden[f"pack{i}_lens"])
    rng = np.random.default_rng(0)
    for _ in range(50):
        nb, lb = int(rng.choice([1, 2, 4, 8])), int(rng.choice([1, 2, 4, 16, 64]))
        n = int(rng.integers(1, nb + 1))
        slots = rng.permutation(10)[:n]
        chunks = [list(rng.integers(0, 1000, int(rng.integers(1, lb + 1)))) for _ in range(n)]
        length = rng.integers(0, 9000, 10)
        a, b = np.zeros(nb * lb + 3 * nb, np.int64), np.zeros(nb * lb + 3 * nb, np.int64)
        np.testing.assert_array_equal(pack_inputs(chunks, slots, nb, lb, length, 10, a),
                                      oracle_pack(chunks, slots, nb, lb, length, 10, b))
        np.testing.assert_array_equal(a, b)


def test_buckets():
    assert default_session_buckets(352)[-1] == 352 and 320 in default_session_buckets(352)
    assert default_session_buckets(3) == (1, 2, 3)
    assert default_session_buckets(1) == (1,)
    assert bucket(33, (1, 2, 4, 8, 16, 32, 64)) == 64
    with pytest.raises(ValueError):
        bucket(65, (1, 64))


def test_validation_matches_reference():
    ok = [(0, [1, 2]), (1, [3])]
    validate_requests(ok, "user", 2, 100)
    bad = [([], "user"), (ok, "system"), ([(0, [1]), (0, [2])], "user"), ([(2, [1])], "user"),
           ([(0, [])], "user"), ([(0, [100])], "user"), ([(0, [-1])], "user"), ([(0, [1.0])], "user"),
           ([(True and 0.5, [1])], "user")]
    for req, role in bad:
        with pytest.raises(ValueError):
            validate_requests(req, role, 2, 100)


def test_validate_collect_matches_validate_requests():
    """The one-pass validation raises exactly what validate_requests raises and returns the tick's columns."""
    from hs_guard_b200.runtime import validate_collect
    assert validate_collect([(0, [5]), (2, [7])], "user", 3, 100) == ([0, 2], [5, 7], 1)
    assert validate_collect([(0, [5]), (2, [7, 8])], "user", 3, 100) == ([0, 2], None, 2)
    cases = [([], "user"), ([(0, [1])], "system"), ([(0, [1]), (0, [2])], "user"), ([(3, [1])], "user"),
             ([(0, [])], "user"), ([(0, [100])], "user"), ([(0, [-1])], "user"), ([(0, [1.0])], "user"),
             ([(0.5, [1])], "user"), ([(0, [1]), (5, [1]), (1, [])], "user"), ([(0, [200]), (7, [1])], "user"),
             ([(0, [np.int64(1)])], "user")]
    for req, role in cases:
        want = got = None
        try:
            validate_requests(req, role, 3, 100)
        except ValueError as e:
            want = str(e)
        try:
            validate_collect(req, role, 3, 100)
        except ValueError as e:
            got = str(e)
        assert want is not None and got == want, (req, got, want)


def test_run_tokens_packs_like_pack_inputs():
    """SlotEngine.run_tokens (one token per row, no per-row lists) fills the same tick buffer as pack_inputs."""
    from hs_guard_b200 import engine as E
    seen = {}

    class FakeLib:
        def hsg_step(self, handle, hin, nb, lb, hout):
            seen["buf"] = np.ctypeslib.as_array(ctypes.cast(hin, ctypes.POINTER(ctypes.c_int64)),
                                                shape=(nb * lb + 3 * nb,)).copy()
            return 0

    eng = E.SlotEngine.__new__(E.SlotEngine)
    eng.max_slots, eng.roles = 40, ("user", "assistant")
    eng.session_buckets = E.default_session_buckets(40)
    eng.length = np.arange(40, dtype=np.int64) * 3
    eng.host, eng.stats, eng._lib, eng._h = {}, {"graph_replays": 0, "ticks": 0}, FakeLib(), 1
    slots, ids = [7, 0, 31, 12, 5], [11, 22, 33, 44, 55]
    nb = bucket(len(slots), eng.session_buckets)
    hin = torch.full((4 * nb,), -7, dtype=torch.int64)  # pageable stand-ins for the engine's pinned buffers
    hout = torch.zeros(2, nb, 1, 3)
    eng.host[(nb, 1)] = (hin, hin.numpy(), hout, hout.numpy())
    length_before = eng.length.copy()
    eng.run_tokens(slots, ids)
    want = np.full(nb + 3 * nb, -1, dtype=np.int64)
    pack_inputs([[i] for i in ids], np.array(slots), nb, 1, length_before, 40, want)
    np.testing.assert_array_equal(seen["buf"], want)
    np.testing.assert_array_equal(eng.length - length_before, np.isin(np.arange(40), slots).astype(np.int64))


def test_config_and_parameter_count():
    assert DEFAULT.check() is DEFAULT
    assert sum(int(np.prod(s)) for _, s, _ in W.parameter_specs()) == 754_519_918
    assert DEFAULT.n_gdn == 18 and DEFAULT.n_attn == 6 and DEFAULT.gdn_in_rows == 8320
    with pytest.raises(ValueError):
        HsgConfig(hidden=2048).check()


def test_engine_layout_interleave_and_concat():
    cfg = DEFAULT
    names = {n for n, _, _ in W.parameter_specs(cfg)}
    sd = W.random_state_dict(3, cfg, names={n for n in names if "layers.0." in n or "layers.3." in n or
                                           not n.startswith("backbone.layers")})
    # fill the other layers with zeros of the right shape so engine_layout can run
    for n, shape, _ in W.parameter_specs(cfg):
        if n not in sd:
            sd[n] = torch.zeros(shape, dtype=torch.bfloat16 if n.startswith("backbone") else torch.float32)
    dev = W.engine_layout(sd, cfg, "cpu")
    L0, L3 = dev["layers"][0], dev["layers"][3]
    assert L0["w_in"].shape == (8320, 1024) and L3["w_in"].shape == (5120, 1024)
    p = "backbone.layers.0.linear_attn."
    assert torch.equal(L0["w_in"][:6144], sd[p + "in_proj_qkv.weight"])
    assert torch.equal(L0["w_in"][8192:8208], sd[p + "in_proj_b.weight"])
    assert torch.equal(L0["w_in"][8208:8224], sd[p + "in_proj_a.weight"])
    assert not L0["w_in"][8224:].any()
    g, u = sd["backbone.layers.0.mlp.gate_proj.weight"], sd["backbone.layers.0.mlp.up_proj.weight"]
    assert torch.equal(L0["w_gu"][0::2], g) and torch.equal(L0["w_gu"][1::2], u)
    assert torch.allclose(dev["inv_freq"], 1.0 / (10000 ** (torch.arange(0, 64, 2).float() / 64)))


def test_random_weights_deterministic():
    a = W.random_state_dict(0, names={"backbone.layers.5.linear_attn.A_log", "heads.user.risk.weight"})
    b = W.random_state_dict(0, names={"backbone.layers.5.linear_attn.A_log", "heads.user.risk.weight"})
    assert W.state_dict_digest(a) == W.state_dict_digest(b)
    assert a["heads.user.risk.weight"].dtype == torch.float32
    assert torch.equal(a["heads.user.risk.weight"], a["heads.user.risk.weight"].bfloat16().float())


def test_slot_sharding_partition():
    for world in (1, 2, 3, 4, 8):
        total = 2816
        owned = []
        for r in range(world):
            lo, hi = slot_range(r, world, total)
            owned += list(range(lo, hi))
        assert owned == list(range(total))
        for s in (0, 351, 352, 2815):
            r, local = route(s, world, total)
            lo, _ = slot_range(r, world, total)
            assert lo + local == s
    reqs = [(5, [1]), (400, [2]), (2000, [3])]
    assert split_requests(reqs, 1, 8, 2816) == [(400 - 352, [2])]


def test_stream_script_shape():
    ticks = stream_script()
    assert len(ticks) == 32 and sum(len(ids) for t in ticks for _, ids in t) == 779


def _header_symbols():
    text = open(os.path.join(ROOT, "include", "hsg.h")).read()
    return sorted(set(re.findall(r"\b(hsg_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    from hs_guard_b200 import _lib
    from hs_guard_b200.build import build
    build()
    L = ctypes.CDLL(_lib.LIB_PATH)
    syms = _header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), s
    assert _lib.lib().hsg_version().startswith(b"hsg-b200")


def _fake_safe(slot, pos, tok):
    return np.float32(((int(slot) * 7919 + int(pos) * 31 + int(tok)) % 1000) / 1000.0)


class _FakeStepLib:
    """hsg_step stand-in: reads the packed tick (ids | lens | slots | starts) and writes p = f(slot, position, token)
    per role into the output buffer, as the device would; counts its calls."""

    def __init__(self):
        self.calls = 0

    def hsg_step(self, handle, hin, nb, lb, hout):
        self.calls += 1
        buf = np.ctypeslib.as_array(ctypes.cast(hin, ctypes.POINTER(ctypes.c_int64)), shape=(nb * lb + 3 * nb,))
        out = np.ctypeslib.as_array(ctypes.cast(hout, ctypes.POINTER(ctypes.c_float)), shape=(2, nb, lb, 3))
        ids, lens = buf[:nb * lb].reshape(nb, lb), buf[nb * lb:nb * lb + nb]
        slots, starts = buf[nb * lb + nb:nb * lb + 2 * nb], buf[nb * lb + 2 * nb:]
        out[:] = 0
        for row in range(nb):
            for t in range(int(lens[row])):
                safe = _fake_safe(slots[row], starts[row] + t, ids[row, t])
                out[:, row, t] = [[safe, 1 - safe, 0], [safe / 2, 1 - safe / 2, 0]]
        return 0


def _fake_engine(max_slots):
    """A SlotEngine whose device tick is replaced by a deterministic host function of (slot, position, token):
    run_arrays / run_tokens in Python, hsg_step (the C fast path's call) by _FakeStepLib."""
    from hs_guard_b200 import engine as E
    eng = E.SlotEngine.__new__(E.SlotEngine)
    eng.max_slots, eng.roles = max_slots, ("user", "assistant")
    eng.session_buckets = E.default_session_buckets(max_slots)
    eng.length = np.zeros(max_slots, dtype=np.int64)
    eng.host, eng.stats, eng._lib, eng._h = {}, {"graph_replays": 0, "ticks": 0}, _FakeStepLib(), 1
    eng.cfg = DEFAULT

    def buffers(nb, lb):  # pageable stand-ins for the engine's pinned buffers (no CUDA here)
        if (nb, lb) not in eng.host:
            hin, hout = torch.zeros(nb * lb + 3 * nb, dtype=torch.int64), torch.zeros(2, nb, lb, 3)
            eng.host[(nb, lb)] = (hin, hin.numpy(), hout, hout.numpy())
        return eng.host[(nb, lb)]
    eng._buffers = buffers

    def run_arrays(chunks, slots):
        # deterministic stand-in for the device: p = f(slot, position, token) per role, rows of the tick
        n = len(chunks)
        lb = bucket(max(len(c) for c in chunks), (1, 2, 4, 8, 16, 32, 64))
        probs = np.zeros((2, n, lb, 3), np.float32)
        lens = np.array([len(c) for c in chunks], np.int64)
        for row, (c, s) in enumerate(zip(chunks, slots)):
            for t, tok in enumerate(c):
                safe = _fake_safe(s, eng.length[int(s)] + t, tok)
                probs[:, row, t] = [[safe, 1 - safe, 0], [safe / 2, 1 - safe / 2, 0]]
        eng.length[np.asarray(slots, dtype=np.int64)] += lens
        return probs, lens
    eng.run_arrays = run_arrays
    eng.run_tokens = lambda slots, ids: run_arrays([[i] for i in ids], slots)
    return eng


def test_streaming_guard_single_tick_path_matches_generic_path():
    """StreamingGuard.step's one-tick fast paths (C, then Python) return exactly what the generic per-request path
    returns, and advance the same lengths."""
    from hs_guard_b200.runtime import DEFAULT_METADATA, StreamingGuard
    rng = np.random.default_rng(3)
    ticks = [[(s, [int(rng.integers(0, 1000))]) for s in range(40)],                       # one token each
             [(s, [int(x) for x in rng.integers(0, 1000, rng.integers(1, 9))]) for s in range(0, 40, 3)],
             [[s, [int(x) for x in rng.integers(0, 1000, 64)]] for s in (3, 9, 1)],          # 64 ids, list pairs
             [(5, [int(x) for x in rng.integers(0, 1000, 70)])],                           # > 64 tokens: generic
             [(7, tuple(int(x) for x in rng.integers(0, 1000, 3)))]]                       # tuple ids: Python path
    for role in ("user", "assistant"):
        fast = StreamingGuard.from_engine(_fake_engine(40), DEFAULT_METADATA)
        slow = StreamingGuard.from_engine(_fake_engine(40), DEFAULT_METADATA)
        slow.engine.fits_one_tick = lambda requests: False
        slow.engine.run_requests = lambda requests: None
        for tick in ticks + ticks[:1]:
            assert fast.step(tick, role) == slow.step(tick, role)
        assert fast.engine._lib.calls == 4 and slow.engine._lib.calls == 0  # the C path took ticks 0, 1, 2, 0
        np.testing.assert_array_equal(fast.engine.length, slow.engine.length)


def test_long_request_tick_schedule():
    """Requests longer than 64 tokens run in rounds of 64-token pieces, each round in request order and split into
    groups of at most the largest row bucket (the reference's schedule, slot_engine_v7.py:147-167)."""
    from hs_guard_b200.engine import _tick_schedule
    got = [(list(g), off) for g, off in _tick_schedule([130, 5, 64, 65], 64, 2)]
    assert got == [([0, 1], 0), ([2, 3], 0), ([0, 3], 64), ([0], 128)]
    assert list(_tick_schedule([], 64, 4)) == []
    eng = _fake_engine(8)
    rng = np.random.default_rng(4)
    reqs = [(s, [int(x) for x in rng.integers(0, 1000, n)]) for s, n in zip((6, 2, 0), (150, 1, 64))]
    out = eng.step(reqs)
    for r, role in enumerate(("user", "assistant")):
        for (s, ids), p in zip(reqs, out[role]):
            safe = np.array([_fake_safe(s, t, tok) for t, tok in enumerate(ids)], np.float32)
            np.testing.assert_array_equal(p[:, 0], safe if r == 0 else safe / 2)
    assert eng.length[6] == 150 and eng.length[2] == 1 and eng.length[0] == 64


def test_host_scan_fill_layout_and_fallbacks():
    """_hsg_host.scan accepts exactly (int slot, [int ids]) lists under the reference's rules; fill writes
    pack_inputs' layout; advance adds each row's length."""
    from hs_guard_b200.build import host
    h = host()
    S, V = 40, DEFAULT.vocab
    length = np.arange(S, dtype=np.int64) * 5
    for req in ([(7, [11]), [0, [22]], (31, [V - 1]), (12, [0]), (5, [55])],
                [(7, [11, 12, 13]), [0, [22]], (31, list(range(64))), (12, [0, V - 1])]):
        slots = [s for s, _ in req]
        longest = max(len(ids) for _, ids in req)
        assert h.scan(req, S, V) == longest
        nb, lb = bucket(len(req), default_session_buckets(S)), bucket(longest, (1, 2, 4, 8, 16, 32, 64))
        hin = np.full(nb * lb + 3 * nb, -9, np.int64)
        h.fill(req, hin, nb, lb, length, S)
        want = np.full(nb * lb + 3 * nb, -1, np.int64)
        pack_inputs([ids for _, ids in req], np.array(slots), nb, lb, length, S, want)
        np.testing.assert_array_equal(hin, want)
        before = length.copy()
        h.advance(length, hin, nb, lb, len(req))
        add = np.zeros(S, np.int64)
        add[slots] = [len(ids) for _, ids in req]
        np.testing.assert_array_equal(length - before, add)
    declined = [
        [(1, (2,))],                            # ids not a list
        [(True, [2])],                          # int subclass (valid for the reference; the general path takes it)
        [(1, [np.int64(2)])],                   # not an int (the general path raises)
        [(1, [2]), (1, [3])],                   # duplicate slot
        [(S, [2])], [(-1, [2])], [(1, [V])], [(1, [2, -2])], [(2 ** 70, [1])], [(1, [2 ** 70])],
        [(1, [])], [(1, [2], 3)], [1], [("1", [2])], [],
    ]
    for bad in declined:
        assert h.scan(bad, S, V) == -1, bad
    assert h.scan(tuple([(1, [2])]), S, V) == -1  # requests not a list


def test_streaming_guard_fast_path_errors_match_reference():
    """Invalid one-token ticks get the reference's ValueError through StreamingGuard.step, with no device call
    and no state change; valid unusual ones (bool slot) run through the general path."""
    from hs_guard_b200.runtime import DEFAULT_METADATA, StreamingGuard
    g = StreamingGuard.from_engine(_fake_engine(40), DEFAULT_METADATA)
    V = DEFAULT.vocab
    bad_ticks = [[], [(1, [2]), (1, [3])], [(40, [2])], [(-1, [2])], [(1, [V])], [(1, [])], [(1, [2.0])],
                 [(1.0, [2])], [(1, [np.int64(2)])], [(2, [3]), (1, [-1])]]
    for role in ("user", "assistant", "system"):
        for tick in bad_ticks + ([[(1, [2])]] if role == "system" else []):
            with pytest.raises(ValueError) as got:
                g.step(tick, role)
            with pytest.raises(ValueError) as want:
                validate_requests(tick, role, 40, V)
            assert str(got.value) == str(want.value), (tick, role)
    assert g.engine._lib.calls == 0 and not g.engine.length.any()
    out = g.step([(True, [3]), (2, [4])], "user")
    assert [r["slot"] for r in out] == [True, 2] and g.engine.length[1] == 1 and g.engine.length[2] == 1
