"""A model of the mbarrier protocol of ring_decode_kernel (hs-guard_b200/csrc/ring_decode.cuh, the single-token
ring-window attention of the headline), checked on the CPU under random interleavings of its roles.

Roles, in the kernel's order of waits and arrivals:
  * producer warp: per item k (metadata block b = k % 2) waits until the consumers have released block b from item
    k - 2 (`meta_free`), writes the item's tile list and arrives on `meta_full`; then streams the item's K tiles and
    after them its V tiles through the STAGES-deep ring, each stage reloaded once all consumer threads have released
    it (`empty`; `full` completes with the copy's bytes). Items of length 0 publish their metadata and load nothing;
  * consumer threads (256, modelled as two groups that drift apart between their block-wide barriers): wait
    `meta_full`, read the metadata; pass 1 waits each K tile, reads it and releases the stage; a block barrier; the
    softmax; a block barrier; pass 2 likewise over the V tiles; a block barrier; the output; release the metadata
    block (`meta_free`) and a last block barrier before the next item.
A wait is for a phase by parity (`mbarrier.try_wait.parity`), so waiting for a phase after the barrier has completed
it and the next one would hang: the model reports that as aliasing. Every access checks that a stage holds the
tile and the metadata block the item it is meant for.
"""
import random

import pytest

CONS = 256


class Bar:
    def __init__(self, name, count):
        self.name, self.count, self.arrivals, self.tx, self.completed = name, count, 0, 0, 0

    def arrive(self, n=1):
        self.arrivals += n
        assert self.arrivals <= self.count, f"{self.name}: over-arrival"
        self._check()

    def expect_tx(self, nbytes):
        self.tx += nbytes

    def complete_tx(self, nbytes):
        self.tx -= nbytes
        self._check()

    def _check(self):
        if self.arrivals == self.count and self.tx == 0:
            self.arrivals, self.completed = 0, self.completed + 1


class Aliased(Exception):
    pass


def wait(bar, phase):
    while True:
        if bar.completed >= phase + 2:
            raise Aliased(f"{bar.name}: waiting for phase {phase} after {bar.completed} completed")
        if bar.completed == phase + 1:
            return
        yield


class BlockBarrier:
    """A named barrier of the consumer threads: the groups meet, in order, at each of their barriers."""

    def __init__(self, groups):
        self.groups, self.arrived, self.generation = groups, 0, 0

    def sync(self):
        gen = self.generation
        self.arrived += 1
        if self.arrived == self.groups:
            self.arrived, self.generation = 0, gen + 1
        while self.generation == gen:
            yield


def run(seed, stages=None, broken=None):
    """One random schedule. broken: 'meta' (the producer reuses a metadata block without waiting for its release)
    or 'stage' (a stage is released by one consumer group only): variants the model must catch."""
    rng = random.Random(seed)
    S = stages or rng.choice([2, 3, 5, 11])
    n_items = rng.randint(1, 10)
    lens = [rng.choice([0, 1, 1, 1]) for _ in range(n_items)]
    ntile = [rng.randint(1, 17) if lens[k] else 0 for k in range(n_items)]
    groups = 2
    full = [Bar(f"full[{s}]", 1) for s in range(S)]
    empty = [Bar(f"empty[{s}]", CONS) for s in range(S)]
    meta_full = [Bar(f"meta_full[{b}]", 1) for b in range(2)]
    meta_free = [Bar(f"meta_free[{b}]", CONS) for b in range(2)]
    meta = [None, None]     # the item whose tile list a block holds
    stage = [None] * S      # (item, pass, tile) a stage holds
    copies = []
    block = BlockBarrier(groups)

    def producer():
        cnt = 0
        for k in range(n_items):
            b = k & 1
            if k >= 2 and broken != "meta":
                yield from wait(meta_free[b], (k >> 1) - 1)
            meta[b] = k
            meta_full[b].arrive(1)
            yield
            if lens[k] == 0:
                continue
            for p in range(2):
                for t in range(ntile[k]):
                    s = cnt % S
                    if cnt >= S:
                        yield from wait(empty[s], cnt // S - 1)
                    stage[s] = (k, p, t)
                    full[s].expect_tx(1)
                    full[s].arrive(1)
                    copies.append(full[s])
                    cnt += 1
                    yield

    def consumers(threads, releases_stages=True):
        cnt = 0
        for k in range(n_items):
            b = k & 1
            yield from wait(meta_full[b], k >> 1)
            assert meta[b] == k, f"item {k}: metadata block holds item {meta[b]}"
            if lens[k] == 0:
                yield
                meta_free[b].arrive(threads)
                continue
            for p in range(2):
                for t in range(ntile[k]):
                    s = cnt % S
                    yield from wait(full[s], cnt // S)
                    assert stage[s] == (k, p, t), f"item {k} pass {p} tile {t}: stage {s} holds {stage[s]}"
                    yield
                    assert stage[s] == (k, p, t), f"item {k} pass {p} tile {t}: stage {s} reloaded while read"
                    if releases_stages:
                        empty[s].arrive(threads)
                    cnt += 1
                yield from block.sync()
                assert meta[b] == k, f"item {k}: metadata block overwritten during the item"
                if p == 0:  # the softmax, then its barrier
                    yield
                    yield from block.sync()
            yield
            assert meta[b] == k, f"item {k}: metadata block overwritten before the output"
            meta_free[b].arrive(threads)
            yield from block.sync()

    if broken == "stage":
        cons = [consumers(CONS // 2), consumers(CONS // 2, releases_stages=False)]
    else:
        cons = [consumers(CONS // 2), consumers(CONS // 2)]
    roles = [producer()] + cons
    for _ in range(300000):
        if not roles and not copies:
            return
        if copies and (not roles or rng.random() < 0.3):  # a copy in flight lands
            copies.pop(rng.randrange(len(copies))).complete_tx(1)
            continue
        role = rng.choice(roles)
        try:
            next(role)
        except StopIteration:
            roles.remove(role)
    raise RuntimeError("no progress: deadlock")


def test_protocol_never_aliases_or_deadlocks():
    for seed in range(400):
        run(seed)


def test_the_kernels_eleven_stages():
    for seed in range(150):
        run(seed, stages=11)


@pytest.mark.parametrize("broken,seeds", [("meta", 150), ("stage", 30)])  # a stuck schedule runs to the step cap
def test_model_catches_a_broken_protocol(broken, seeds):
    failures = 0
    for seed in range(seeds):
        try:
            run(seed, broken=broken)
        except (Aliased, RuntimeError, AssertionError):
            failures += 1
    assert failures > 5
