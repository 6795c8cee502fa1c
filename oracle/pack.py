"""``pack_inputs`` restated (reference ``src/hs_guard/engine/slot_engine_v7.py:7-25``). Test infrastructure only.

Buffer layout, int64, length ``nb*lb + 3*nb``:
``[ids nb x lb (right-padded with 0) | lens nb | slots nb (padded rows -> max_slots) | starts nb (length[slot])]``.
"""
from __future__ import annotations

import numpy as np


def pack_inputs(chunks, slots, nb, lb, length, max_slots, out):
    n = len(chunks)
    lens = np.array([len(c) for c in chunks], dtype=np.int64)
    slots = np.asarray(slots, dtype=np.int64)
    out[:] = 0
    ids = out[:nb * lb].reshape(nb, lb)
    for row, chunk in enumerate(chunks):
        ids[row, :len(chunk)] = chunk
    base = nb * lb
    out[base:base + n] = lens
    out[base + nb:base + 2 * nb] = max_slots
    out[base + nb:base + nb + n] = slots
    out[base + 2 * nb:base + 2 * nb + n] = np.asarray(length, dtype=np.int64)[slots]
    return lens
