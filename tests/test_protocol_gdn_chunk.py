"""A model of the mbarrier protocol of gdn_chunk_kernel (hs-guard_b200/csrc/gdn_chunk.cuh), checked on the CPU
under random interleavings of its roles.

Each role of the kernel is a generator that waits on barrier phases and arrives on barriers in the kernel's order:
the producer warp (inputs and state requests), the epilogue warp (state store), the two prologue warps (per
sub-chunk tables) and the consumer warps (two groups of threads that may drift apart). TMA copies complete at
random later times. A barrier completes a phase when its arrival count is reached and no transaction bytes are
pending; a wait is for a phase by parity, as `mbarrier.try_wait.parity` is, so a waiter that arrives after the
barrier has completed its phase AND the next one would wait forever: the model reports that as aliasing. Items
have random lengths, including runs of padding items (length 0), which release their inputs at once.

The protocol of the kernel passes every schedule; the earlier version (the epilogue warp not counted among the
input readers, padding items not waiting on the state barrier) is caught, which is how the second ordering was found.
"""
import random

import pytest

CONS, PRO, EPI, PROD = 256, 64, 32, 32   # consumer, prologue, epilogue, producer threads
NSUB = 4                                 # 16-token sub-chunks of a 64-token item


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


def run(seed, fixed=True):
    rng = random.Random(seed)
    n_items = rng.randint(1, 9)
    lens = [rng.choice([0, 0, 64, 5]) for _ in range(n_items)]
    full_in, full_st = Bar("inputs full", 1), Bar("state full", 1)
    done, empty_st = Bar("done", CONS), Bar("state free", 1)
    empty_in = Bar("inputs free", CONS + PRO + (EPI if fixed else 0))
    cdone = Bar("conv done", CONS + PRO + EPI + PROD)
    sfull = [Bar("sub-chunk full 0", PRO), Bar("sub-chunk full 1", PRO)]
    sdone = [Bar("sub-chunk done 0", CONS), Bar("sub-chunk done 1", CONS)]
    meta = [None, None]
    copies = []

    def issue(bar, nbytes):
        if nbytes:
            bar.expect_tx(nbytes)
            copies.append((bar, nbytes))
        bar.arrive(1)

    def join_conv(i, threads):
        yield from wait(full_in, i)
        assert meta[i & 1] == lens[i], f"item {i}: stale metadata"
        if lens[i] > 0:
            cdone.arrive(threads)
        return lens[i]

    def producer():
        issue(full_st, 32 if lens[0] else 0)
        meta[0] = lens[0]
        issue(full_in, 96 if lens[0] else 0)
        for i in range(n_items):
            if i > 0:
                yield from wait(empty_st, i - 1)
                issue(full_st, 32 if lens[i] else 0)
            yield from join_conv(i, PROD)
            if i + 1 < n_items:
                yield from wait(empty_in, i)
                meta[(i + 1) & 1] = lens[i + 1]
                issue(full_in, 96 if lens[i + 1] else 0)
            yield

    def epilogue():
        for i in range(n_items):
            yield from join_conv(i, EPI)
            if fixed:
                empty_in.arrive(EPI)
            yield from wait(done, i)
            assert meta[i & 1] == lens[i], f"item {i}: metadata overwritten before the store"
            yield
            empty_st.arrive(1)

    def prologue():
        jsub = item_seq = 0
        for i in range(n_items):
            n = yield from join_conv(i, PRO)
            if n == 0:
                empty_in.arrive(PRO)
                continue
            yield from wait(cdone, item_seq)
            item_seq += 1
            for _ in range(NSUB):
                if jsub >= 2:
                    yield from wait(sdone[jsub & 1], (jsub >> 1) - 1)
                yield
                sfull[jsub & 1].arrive(PRO)
                jsub += 1
            empty_in.arrive(PRO)

    def consumers(threads):
        jsub = 0
        for i in range(n_items):
            yield from wait(full_in, i)
            assert meta[i & 1] == lens[i], f"item {i}: stale metadata"
            if lens[i] == 0:
                empty_in.arrive(threads)
                if fixed:
                    yield from wait(full_st, i)
            else:
                cdone.arrive(threads)
                yield from wait(full_st, i)
                for sc in range(NSUB):
                    yield from wait(sfull[jsub & 1], jsub >> 1)
                    yield
                    if sc == NSUB - 1:
                        empty_in.arrive(threads)
                    yield
                    sdone[jsub & 1].arrive(threads)
                    jsub += 1
            yield
            done.arrive(threads)

    roles = [producer(), epilogue(), prologue(), consumers(CONS // 2), consumers(CONS // 2)]
    for _ in range(200000):
        if not roles and not copies:
            return
        if copies and (not roles or rng.random() < 0.3):  # a copy in flight lands
            bar, nbytes = copies.pop(rng.randrange(len(copies)))
            bar.complete_tx(nbytes)
            continue
        role = rng.choice(roles)
        try:
            next(role)
        except StopIteration:
            roles.remove(role)
    raise RuntimeError("no progress: deadlock")


def test_protocol_never_aliases_or_deadlocks():
    for seed in range(600):
        run(seed)


def test_model_catches_the_earlier_protocol():
    failures = 0
    for seed in range(200):
        try:
            run(seed, fixed=False)
        except (Aliased, RuntimeError, AssertionError):
            failures += 1
    assert failures > 20
