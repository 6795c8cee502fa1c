"""Host packing of one tick (the layout of reference src/hs_guard/engine/slot_engine_v7.py:7-25).

``pack_inputs`` fills an int64 buffer of ``nb*lb + 3*nb`` words:
``[ids nb x lb, right-padded with 0 | lens nb | slots nb (padded rows -> max_slots, the scratch slot) |
starts nb (length[slot]; padded rows 0)]`` and returns the per-request lengths. The engine's kernels read this
buffer directly on the device.
"""
from __future__ import annotations

import numpy as np


def pack_inputs(chunks, slots, nb, lb, length, max_slots, out):
    n = len(chunks)
    lens = np.fromiter(map(len, chunks), dtype=np.int64, count=n)
    if n > nb or (n and int(lens.max()) > lb):
        raise ValueError("tick does not fit its bucket")
    ids = out[:nb * lb].reshape(nb, lb)
    ids.fill(0)
    if lb == 1:
        ids[:n, 0] = [c[0] for c in chunks]
    elif n:
        mask = np.arange(lb)[None, :] < lens[:, None]
        ids[:n][mask] = np.concatenate([np.asarray(c, dtype=np.int64) for c in chunks])
    base = nb * lb
    tail = out[base:base + 3 * nb].reshape(3, nb)
    tail[0].fill(0)
    tail[0, :n] = lens
    tail[1].fill(max_slots)
    tail[1, :n] = slots
    tail[2].fill(0)
    tail[2, :n] = np.asarray(length, dtype=np.int64)[np.asarray(slots, dtype=np.int64)]
    return lens
