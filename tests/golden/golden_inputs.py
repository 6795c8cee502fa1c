"""Seeded inputs shared by tests/golden/make_golden.py (reference side) and the parity tests (our side).

numpy's PCG64 streams are bit-reproducible across hosts, so large inputs are regenerated here instead of being
stored in the fixture.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

VOCAB = 248320
STREAM_MAX_SLOTS = 3


def _rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def _bf16(x):
    """float32 array -> torch fp32 tensor holding bf16-rounded values."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float()


def gdn_inputs(n, L, seed, heads=16, dim=128):
    """Config-2-style GDN step inputs: q, k, v [n, L, heads, dim] (bf16 values), raw a, b [n, L, heads] ~ N(0, 1)
    so that g = -softplus(a) (A_log = 0, dt_bias = 0) and beta = sigmoid(b), and state [n, heads, dim, dim] ~ N(0, 0.02).
    Returns (q, k, v, g, beta, state) in transformers' recurrent-rule layout, plus the raw (a, b) via gdn_raw."""
    r = _rng(seed)
    q = _bf16(r.standard_normal((n, L, heads, dim), dtype=np.float32))
    k = _bf16(r.standard_normal((n, L, heads, dim), dtype=np.float32))
    v = _bf16(r.standard_normal((n, L, heads, dim), dtype=np.float32))
    a = torch.from_numpy(r.standard_normal((n, L, heads), dtype=np.float32))
    b = torch.from_numpy(r.standard_normal((n, L, heads), dtype=np.float32))
    state = torch.from_numpy(r.standard_normal((n, heads, dim, dim), dtype=np.float32) * np.float32(0.02))
    g = -F.softplus(a)
    beta = torch.sigmoid(b)
    gdn_inputs.raw = (a, b)
    return q, k, v, g, beta, state


def gdn_raw(n, L, seed, heads=16, dim=128):
    """(packed [n, L, 3*heads*dim], a, b, state) for the same draw as gdn_inputs: the fused-kernel layout."""
    q, k, v, g, beta, state = gdn_inputs(n, L, seed, heads, dim)
    a, b = gdn_inputs.raw
    packed = torch.cat([q.reshape(n, L, -1), k.reshape(n, L, -1), v.reshape(n, L, -1)], -1)
    return packed, a, b, state


def ring_positions(start, filled, window=512):
    """ring_pos row for a slot whose last ``filled`` positions before ``start`` are in the ring (col = pos % W)."""
    row = np.full(window + 1, -1, dtype=np.int64)
    for p in range(max(0, start - filled), start):
        row[p % window] = p
    return row


def ring_inputs(lb, seed, n=8, hkv=2, groups=4, dim=256, window=512):
    """Ring-attention inputs with the reference kernel's contract (engine/ring_attention_kernel.py:7-26):
    q [n, hkv, groups*lb, dim], ring_k/v [n+1, hkv, W+1, dim], new_k/v [n, hkv, lb, dim], ring_pos [n+1, W+1],
    slots (a permutation of 0..n-2 plus the scratch slot n), starts, lens. Write position ~ U[0, W), filled ~ U[1, W]
    with wrapped rings; one row is padding (scratch slot, lens 0) and one has lens < lb when lb > 1."""
    r = _rng(seed)
    S = n
    q = _bf16(r.standard_normal((n, hkv, groups * lb, dim), dtype=np.float32))
    ring_k = _bf16(r.standard_normal((S + 1, hkv, window + 1, dim), dtype=np.float32))
    ring_v = _bf16(r.standard_normal((S + 1, hkv, window + 1, dim), dtype=np.float32))
    new_k = _bf16(r.standard_normal((n, hkv, lb, dim), dtype=np.float32))
    new_v = _bf16(r.standard_normal((n, hkv, lb, dim), dtype=np.float32))
    slots = np.concatenate([r.permutation(n - 1), [S]]).astype(np.int64)
    wp = r.integers(0, window, n)
    filled = r.integers(1, window + 1, n)
    starts = np.zeros(n, dtype=np.int64)
    ring_pos = np.full((S + 1, window + 1), -1, dtype=np.int64)
    for row in range(n - 1):
        start = int(wp[row]) + (window if filled[row] > wp[row] else 0)
        starts[row] = start
        ring_pos[slots[row]] = ring_positions(start, int(filled[row]), window)
    lens = np.full(n, lb, dtype=np.int64)
    lens[-1] = 0
    if lb > 1:
        lens[0] = lb - 1
    return (q, ring_k, ring_v, new_k, new_v, torch.from_numpy(ring_pos), torch.from_numpy(slots),
            torch.from_numpy(starts), torch.from_numpy(lens))


def stream_script(seed=7):
    """Ticks of (slot, token ids) for STREAM_MAX_SLOTS slots: multi-token ticks split at 64, padding rows,
    slot 0 wrapping its 512-entry ring, then single-token ticks in rotating row order."""
    r = _rng(seed)
    ids = lambda n: [int(x) for x in r.integers(0, VOCAB, n)]
    ticks = [[(0, ids(70)), (1, ids(5))], [(2, ids(1)), (0, ids(1)), (1, ids(3))]]
    for i in range(8):
        tick = [(0, ids(64))]
        if i % 2:
            tick.append((1, ids(2)))
        ticks.append(tick)
    ticks.append([(2, ids(100))])
    order = [0, 1, 2]
    for i in range(20):
        ticks.append([(s, ids(1)) for s in order])
        order = order[1:] + order[:1]
    ticks.append([(1, ids(17)), (0, ids(2))])
    return ticks


LONG_CONTEXTS = (8000, 2048, 512, 1000)  # the headline's 512 / 2,048 / 8,000-token contexts, plus a ragged one
LONG_STEPS = 256


def long_script(seed=4):
    """Headline-shaped streams for len(LONG_CONTEXTS) slots: one request per slot carrying its whole initial context
    (the engine splits it into 64-token ticks, as the benchmark's prefill does; the 1,000-token context ends in a
    40-token tick), then LONG_STEPS ticks of one token for every slot. Returns a list of ticks."""
    r = _rng(seed)
    prefill = [(s, [int(x) for x in r.integers(0, VOCAB, n)]) for s, n in enumerate(LONG_CONTEXTS)]
    draws = r.integers(0, VOCAB, (LONG_STEPS, len(LONG_CONTEXTS)))
    return [prefill] + [[(s, [int(t)]) for s, t in enumerate(row)] for row in draws]


def sample_index(numel, seed, count=8192):
    """Sorted random flat indices used to compare large state pools by sample."""
    return np.sort(_rng(1000 + seed).choice(numel, size=min(count, numel), replace=False)).astype(np.int64)
