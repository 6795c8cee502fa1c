"""Slot sharding across the GPUs of one node: slots are independent conversations, so each rank (one process per
GPU) owns a contiguous block of global slots with its own full weight replica and pools, and no collective is on
the data path. Only host-side bookkeeping (routing a global slot to its rank, gathering metrics) crosses ranks.
"""
from __future__ import annotations

from bisect import bisect_right


def slot_range(rank, world, total):
    """[lo, hi) global slots owned by ``rank`` when ``total`` slots are split as evenly as possible."""
    if not 0 <= rank < world:
        raise ValueError("rank outside the world")
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def route(slot, world, total):
    """(rank, local slot) for a global slot."""
    if not 0 <= slot < total:
        raise ValueError("slot outside the allocated range")
    for r in range(world):
        lo, hi = slot_range(r, world, total)
        if lo <= slot < hi:
            return r, slot - lo
    raise AssertionError("unreachable")


def split_requests(requests, rank, world, total):
    """The requests (global slot, ids) that ``rank`` serves, rewritten to its local slots, in request order."""
    lo, hi = slot_range(rank, world, total)
    return [(s - lo, ids) for s, ids in requests if lo <= s < hi]


class SlotRouter:
    """route() for many slots: the owner of a global slot by bisection over the blocks' first slots."""

    def __init__(self, world, total):
        self.world, self.total = world, total
        self.first = [slot_range(r, world, total)[0] for r in range(world)]

    def __call__(self, slot):
        if not 0 <= slot < self.total:
            raise ValueError("slot outside the allocated range")
        r = bisect_right(self.first, slot) - 1
        return r, slot - self.first[r]
