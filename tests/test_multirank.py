"""Multi-rank host logic on CPU with the gloo backend (world size 2): slot sharding, request routing and the
max-over-ranks step time that bench.py reports. No GPU and no collective on the data path are involved: each rank
serves its own block of slots, exactly as on a multi-GPU node."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hs_guard_b200.shard import route, slot_range, split_requests

TOTAL = 37  # global slots, deliberately not divisible by the world size


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cut(global_slot, token):
    return float((global_slot * 131 + token) % 997) / 997.0


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = slot_range(rank, world, TOTAL)
        rng = np.random.default_rng(5)
        requests = [(int(s), [int(t)]) for s, t in zip(rng.permutation(TOTAL)[:29], rng.integers(0, 5000, 29))]
        mine = split_requests(requests, rank, world, TOTAL)
        # each rank scores its requests on its own local slots; the global slot is lo + local slot
        local = [(lo + s, _cut(lo + s, ids[0])) for s, ids in mine]
        assert all(0 <= s < hi - lo for s, _ in mine)
        gathered = [None] * world
        dist.all_gather_object(gathered, local)
        # step time: the slowest rank sets the number, as in bench.py's max over ranks
        t = torch.tensor([1.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            merged = dict(kv for part in gathered for kv in part)
            expected = {s: _cut(s, ids[0]) for s, ids in requests}
            np.save(os.path.join(out_dir, "ok.npy"),
                    np.array([merged == expected, float(t.item()) == float(world), len(merged) == len(requests)]))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_covers_every_request_once(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    assert np.load(tmp_path / "ok.npy").all()


def test_routing_is_a_partition():
    for world in (1, 2, 3, 8):
        owners = [route(s, world, TOTAL) for s in range(TOTAL)]
        for r in range(world):
            lo, hi = slot_range(r, world, TOTAL)
            assert [s for s, (rr, _) in enumerate(owners) if rr == r] == list(range(lo, hi))
        assert sum(hi - lo for lo, hi in (slot_range(r, world, TOTAL) for r in range(world))) == TOTAL
