"""A model of the mbarrier protocol of gemm_pc_kernel (hs-guard_b200/csrc/gemm_persist.cuh, the persistent GEMM of
64-token ticks), checked on the CPU under random interleavings of its roles.

Roles, in the kernel's order of waits and arrivals:
  * producer (one thread): one STAGES-deep ring of stages across all of the CTA's tiles; the load of stage use c
    waits until the MMAs of use c - STAGES have completed (`empty`), then arms `full` with the copies' bytes;
  * MMA issuer (one thread): per tile lt, accumulator buffer lt % 2, first waits until the epilogue has drained the
    buffer's previous tile (`acc_empty`, from tile lt - 2 on); per K block waits `full`, issues the MMAs and commits
    the stage back (`empty` arrives once those MMAs have completed); after the tile commits `acc_full`;
  * epilogue (128 threads, modelled as two groups that drift apart between the group's barriers): per tile waits
    `acc_full`, drains the accumulator in chunks and arrives on `acc_empty`.
MMAs complete asynchronously, in issue order, and a commit arrives when every MMA issued before it has completed. A
wait is for a phase by parity, so waiting for a phase after the barrier has completed it and the next one would hang:
the model reports that as aliasing. Every access checks that a stage holds the K block, and an accumulator buffer the
tile, it is meant for.
"""
import random

import pytest

EPI = 128


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


def run(seed, broken=None):
    """One random schedule. broken: 'acc' (the MMA reuses an accumulator buffer without waiting for the epilogue)
    or 'stage' (the producer reloads a stage without waiting for its MMAs): variants the model must catch."""
    rng = random.Random(seed)
    S = rng.choice([2, 3, 4, 6])
    tiles = [rng.randint(1, 6) for _ in range(rng.randint(1, 7))]  # K blocks per tile
    full = [Bar(f"full[{s}]", 1) for s in range(S)]
    empty = [Bar(f"empty[{s}]", 1) for s in range(S)]
    acc_full = [Bar(f"acc_full[{b}]", 1) for b in range(2)]
    acc_empty = [Bar(f"acc_empty[{b}]", EPI) for b in range(2)]
    stage = [None] * S       # (tile, K block) a stage holds
    acc = [None, None]       # the tile whose sums an accumulator buffer holds
    copies = []              # TMA loads in flight: barriers
    pipe = []                # tcgen05 work in flight, in issue order: ("mma", stage, expected) or ("commit", bar)

    def producer():
        c = 0
        for lt, nk in enumerate(tiles):
            for i in range(nk):
                s = c % S
                if c >= S and broken != "stage":
                    yield from wait(empty[s], c // S - 1)
                stage[s] = (lt, i)
                full[s].expect_tx(1)
                full[s].arrive(1)
                copies.append(full[s])
                c += 1
                yield

    def mma():
        c = 0
        for lt, nk in enumerate(tiles):
            b = lt & 1
            if lt >= 2 and broken != "acc":
                yield from wait(acc_empty[b], (lt >> 1) - 1)
            acc[b] = lt
            for i in range(nk):
                s = c % S
                yield from wait(full[s], c // S)
                assert stage[s] == (lt, i), f"tile {lt} K block {i}: stage {s} holds {stage[s]}"
                pipe.append(("mma", s, (lt, i), b, lt))
                pipe.append(("commit", empty[s]))
                c += 1
                yield
            pipe.append(("commit", acc_full[b]))

    def epilogue(threads):
        for lt, _ in enumerate(tiles):
            b = lt & 1
            yield from wait(acc_full[b], lt >> 1)
            for _chunk in range(rng.randint(1, 3)):
                assert acc[b] == lt, f"tile {lt}: accumulator {b} holds tile {acc[b]} while drained"
                yield
            acc_empty[b].arrive(threads)

    def step_pipe():
        kind = pipe[0][0]
        if kind == "mma":
            _, s, expected, b, lt = pipe.pop(0)
            assert stage[s] == expected, f"an MMA of tile {lt} read stage {s} holding {stage[s]}"
            assert acc[b] == lt, f"an MMA of tile {lt} accumulated into buffer {b} holding tile {acc[b]}"
        else:
            pipe.pop(0)[1].arrive(1)

    roles = [producer(), mma(), epilogue(EPI // 2), epilogue(EPI // 2)]
    for _ in range(200000):
        if not roles and not copies and not pipe:
            return
        r = rng.random()
        if copies and (not roles or r < 0.2):
            copies.pop(rng.randrange(len(copies))).complete_tx(1)
            continue
        if pipe and (not roles or r < 0.4):
            step_pipe()
            continue
        if not roles:
            continue
        role = rng.choice(roles)
        try:
            next(role)
        except StopIteration:
            roles.remove(role)
    raise RuntimeError("no progress: deadlock")


def test_protocol_never_aliases_or_deadlocks():
    for seed in range(800):
        run(seed)


@pytest.mark.parametrize("broken", ["acc", "stage"])
def test_model_catches_a_broken_protocol(broken):
    failures = 0
    for seed in range(200):
        try:
            run(seed, broken=broken)
        except (Aliased, RuntimeError, AssertionError):
            failures += 1
    assert failures > 10
