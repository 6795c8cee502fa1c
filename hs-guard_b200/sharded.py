"""StreamingGuard over the GPUs of one host, in one process.

Slots are independent conversations, so the global slot range [0, max_slots) is cut into contiguous blocks
(shard.slot_range), one per device; each device holds a full weight replica and the state pools of its block in its
own SlotEngine and is driven by its own host thread. A step validates the requests once with the reference's rules
(runtime.py:161-171, on global slots), hands every device its share rewritten to local slots, runs the shares at the
same time (the C ABI releases the GIL while a device works) and returns the results in request order with the global
slot numbers. Nothing crosses devices: no peer memory, no collective. The reference serves one process per GPU
(examples/demo/OPERATIONS.md); ``bench.py --gpus N`` measures that arrangement, this class the in-process one.
"""
from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

from .runtime import StreamingGuard, validate_requests
from .shard import SlotRouter, slot_range


class ShardedGuard:
    """The StreamingGuard API (``step(requests, role)``, ``reset()``) over ``devices`` (default: every visible GPU)."""

    def __init__(self, model, metadata, max_slots, devices=None, head="redline"):
        import torch
        if not isinstance(max_slots, int) or max_slots < 1:
            raise ValueError("max_slots must be a positive integer")
        devices = list(range(torch.cuda.device_count())) if devices is None else list(devices)
        if not devices or len(set(devices)) != len(devices):
            raise ValueError("devices must be a nonempty list of distinct CUDA device indices")
        if max_slots < len(devices):
            raise ValueError("max_slots must be at least the number of devices")
        self.devices, self.metadata, self.max_slots = devices, metadata, max_slots
        world = len(devices)
        self.ranges = [slot_range(r, world, max_slots) for r in range(world)]
        self.route = SlotRouter(world, max_slots)
        self.guards = [StreamingGuard(model, metadata, max_slots=hi - lo, head=head, device=d)
                       for (lo, hi), d in zip(self.ranges, devices)]
        self.vocab_size = self.guards[0].vocab_size
        self._pool = ThreadPoolExecutor(max_workers=world, thread_name_prefix="hsg-device")

    @classmethod
    def from_guards(cls, guards, metadata):
        """Compose already-built per-device guards (block r = the slots of guards[r], in order)."""
        self = cls.__new__(cls)
        self.guards, self.metadata = list(guards), metadata
        self.devices = [getattr(g.engine, "device", None) for g in self.guards]
        sizes = [g.max_slots for g in self.guards]
        self.max_slots = sum(sizes)
        self.ranges, lo = [], 0
        for n in sizes:
            self.ranges.append((lo, lo + n))
            lo += n
        self.route = _BlockRouter(self.ranges)
        self.vocab_size = self.guards[0].vocab_size
        self._pool = ThreadPoolExecutor(max_workers=len(self.guards), thread_name_prefix="hsg-device")
        return self

    def step(self, requests, role="assistant"):
        validate_requests(requests, role, self.max_slots, self.vocab_size)
        shares = [[] for _ in self.guards]
        where = [[] for _ in self.guards]
        for i, (slot, ids) in enumerate(requests):
            r, local = self.route(slot)
            shares[r].append((local, ids))
            where[r].append(i)
        busy = [r for r, share in enumerate(shares) if share]
        if len(busy) == 1:
            parts = {busy[0]: self.guards[busy[0]].step(shares[busy[0]], role)}
        else:
            futures = {r: self._pool.submit(self.guards[r].step, shares[r], role) for r in busy}
            parts = {r: f.result() for r, f in futures.items()}
        out = [None] * len(requests)
        for r, results in parts.items():
            for i, res in zip(where[r], results):
                res["slot"] = requests[i][0]
                out[i] = res
        return out

    def reset(self):
        for g in self.guards:
            g.reset()

    def reset_slot(self, slot):
        r, local = self.route(slot)
        self.guards[r].engine.reset_slot(local)

    def close(self):
        self._pool.shutdown(wait=True)
        for g in self.guards:
            close = getattr(g.engine, "close", None)
            if close:
                close()


class _BlockRouter:
    """Owner of a global slot for explicitly sized blocks [(lo, hi), ...]."""

    def __init__(self, ranges):
        self.ranges = ranges
        self.total = ranges[-1][1]

    def __call__(self, slot):
        if not 0 <= slot < self.total:
            raise ValueError("slot outside the allocated range")
        for r, (lo, hi) in enumerate(self.ranges):
            if lo <= slot < hi:
                return r, slot - lo
        raise AssertionError("unreachable")
