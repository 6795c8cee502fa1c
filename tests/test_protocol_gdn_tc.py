"""A model of the mbarrier protocol of gdn_tc_kernel (hs-guard_b200/csrc/gdn_tc.cuh, the single-token delta-rule step
of the headline), checked on the CPU under random interleavings of its roles.

Roles, in the kernel's order of waits and arrivals:
  * producer: the first S items' loads are issued up front (state and conv history before the dependency wait, the
    projection slices after it); item i >= S waits for stage i % S to be released (`empty`, by the epilogue once the
    state store of item i - S has read the stage) and reloads it (`full`: one arrival plus the copies' bytes);
  * prologue (two warps, 64 threads): per item waits `full`, and for the per-item scratch buffer (two, by item parity)
    waits until the consumers are done with item i - 2 (`done`), writes the scratch, arrives on `pro`;
  * consumers (256 threads, modelled as two halves that drift apart): wait `full` and `pro`, read the stage and the
    scratch, write the new state into the stage, arrive on `done`;
  * epilogue (one warp): waits `done`, issues the state's TMA stores (which read the stage later, asynchronously),
    makes the output rows, waits until the stores have read the stage, arrives on `empty`.
Copies complete at random later times; a barrier completes a phase when its arrival count is reached with no bytes
pending, and a wait is for a phase by parity, so waiting for a phase after the barrier has completed it and the
next one would hang: the model reports that as aliasing. Every access checks that the stage or scratch buffer still
holds the item it is meant for; a stage refilled while a store still reads it is an error. Items have random
lengths, with runs of padding items (length 0: no copies, no state store).
"""
import random

import pytest

CONS, PRO = 256, 64


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


def run(seed, broken=None, stages=None):
    """One random schedule. broken: 'scratch' (the prologue does not wait for item i - 2's consumers) or 'store'
    (the epilogue releases the stage without waiting for its stores to read it): variants the model must catch.
    stages: force the stage count (default: one of the kernel's)."""
    rng = random.Random(seed)
    # the kernel's stage counts (2 at 16-token ticks, 5 at one token); it never runs with one stage, where the
    # prologue's wait for item i - 2's consumers would alias (gdn_tc.cuh asserts that two stages fit)
    S = rng.choice([2, 3, 4, 5]) if stages is None else stages
    n_items = rng.randint(1, 12)
    lens = [rng.choice([0, 0, 1, 1, 1, 4]) for _ in range(n_items)]
    full = [Bar(f"full[{s}]", 1) for s in range(S)]
    pro = [Bar(f"pro[{s}]", PRO) for s in range(S)]
    done = [Bar(f"done[{s}]", CONS) for s in range(S)]
    empty = [Bar(f"empty[{s}]", 1) for s in range(S)]
    stage = [None] * S        # the item whose data a stage holds
    meta = [None] * S         # (item, length) the producer wrote for a stage
    scratch = [None, None]    # the item whose tables a scratch buffer holds
    reading = [0] * S         # state stores still reading a stage
    copies = []               # in flight: (kind, stage or barrier, bytes)

    def load(s, i, first_part):
        """Part of item i's loads into stage s; the first part carries the expected bytes and the arrival."""
        if first_part:
            assert reading[s] == 0, f"stage {s} refilled while a state store still reads it"
            stage[s], meta[s] = i, (i, lens[i])
            if lens[i] > 0:
                full[s].expect_tx(3)
                copies.append(("tx", full[s], 2))   # state tile + conv history
            full[s].arrive(1)
        elif lens[i] > 0:
            copies.append(("tx", full[s], 1))       # projection slices

    def producer():
        pre = min(n_items, S)
        for i in range(pre):
            load(i % S, i, True)
        yield  # the dependency wait
        for i in range(pre):
            load(i % S, i, False)
        for i in range(pre, n_items):
            s = i % S
            yield from wait(empty[s], i // S - 1)
            load(s, i, True)
            load(s, i, False)
            yield

    def prologue():
        for i in range(n_items):
            s = i % S
            yield from wait(full[s], i // S)
            if i >= 2 and broken != "scratch":
                yield from wait(done[(i - 2) % S], (i - 2) // S)
            assert stage[s] == i and meta[s] == (i, lens[i]), f"prologue, item {i}: stage holds {stage[s]}"
            if lens[i] > 0:
                scratch[i & 1] = i
            yield
            pro[s].arrive(PRO)

    def consumers(threads):
        for i in range(n_items):
            s = i % S
            yield from wait(full[s], i // S)
            yield from wait(pro[s], i // S)
            assert stage[s] == i and meta[s] == (i, lens[i]), f"consumers, item {i}: stage holds {stage[s]}"
            if lens[i] > 0:
                assert scratch[i & 1] == i, f"consumers, item {i}: scratch holds {scratch[i & 1]}"
                yield
                assert scratch[i & 1] == i, f"consumers, item {i}: scratch overwritten while in use"
                assert stage[s] == i, f"consumers, item {i}: stage refilled while in use"
            yield
            done[s].arrive(threads)

    def epilogue():
        for i in range(n_items):
            s = i % S
            yield from wait(done[s], i // S)
            assert stage[s] == i and meta[s] == (i, lens[i]), f"epilogue, item {i}: stage holds {stage[s]}"
            if lens[i] > 0:  # the new state's stores, issued before the output rows
                reading[s] += 1
                copies.append(("read", s, 0))
            yield  # output rows
            assert stage[s] == i, f"epilogue, item {i}: stage refilled before the output rows were made"
            if broken != "store":
                while reading[s]:
                    yield
            empty[s].arrive(1)

    roles = [producer(), prologue(), consumers(CONS // 2), consumers(CONS // 2), epilogue()]
    for _ in range(200000):
        if not roles and not copies:
            return
        if copies and (not roles or rng.random() < 0.3):  # a copy in flight completes
            kind, target, nbytes = copies.pop(rng.randrange(len(copies)))
            if kind == "tx":
                target.complete_tx(nbytes)
            else:
                reading[target] -= 1
            continue
        role = rng.choice(roles)
        try:
            next(role)
        except StopIteration:
            roles.remove(role)
    raise RuntimeError("no progress: deadlock")


def test_protocol_never_aliases_or_deadlocks():
    for seed in range(1500):
        run(seed)


def test_model_shows_why_one_stage_is_excluded():
    with pytest.raises(Aliased):
        for seed in range(400):
            run(seed, stages=1)


def test_model_catches_a_missing_scratch_wait():
    failures = 0
    for seed in range(400):
        try:
            run(seed, broken="scratch")
        except (Aliased, RuntimeError, AssertionError):
            failures += 1
    assert failures > 10


def test_model_catches_a_stage_released_before_its_store_read_it():
    failures = 0
    for seed in range(400):
        try:
            run(seed, broken="store")
        except (Aliased, RuntimeError, AssertionError):
            failures += 1
    assert failures > 10
