"""ShardedGuard on two B200s in one process: the reference's multi-slot script (tests/golden/make_golden.py) streamed
over slots spread across both devices gives the same cut scores as one device, and the reference engine's scores
within 2e-3. Skipped when fewer than two GPUs are visible."""
import numpy as np
import pytest
import torch

from golden_inputs import stream_script

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs two GPUs")]

P_TOL = 2e-3


def test_sharded_guard_two_devices_matches_one_and_reference(golden, weights_seed0):
    from hs_guard_b200.runtime import DEFAULT_METADATA, StreamingGuard
    from hs_guard_b200.shard import route
    from hs_guard_b200.sharded import ShardedGuard
    # 4 global slots: 0, 1 on device 0 and 2, 3 on device 1; the script uses slots 0-2
    sharded = ShardedGuard(weights_seed0, DEFAULT_METADATA, max_slots=4, devices=[0, 1])
    # the same two slot blocks as separate guards on device 0, fed one after the other: the same tick shapes
    blocks = [StreamingGuard(weights_seed0, DEFAULT_METADATA, max_slots=2, device=0) for _ in range(2)]
    assert [g.engine.device.index for g in sharded.guards] == [0, 1]
    try:
        got, one = [], []
        for tick in stream_script():
            a = sharded.step(tick, "assistant")
            assert [r["slot"] for r in a] == [s for s, _ in tick]
            shares = [[], []]
            for s, ids in tick:
                r, local = route(s, 2, 4)
                shares[r].append((local, ids))
            b = {}
            for r, share in enumerate(shares):
                if share:
                    for (local, _), res in zip(share, blocks[r].step(share, "assistant")):
                        b[r * 2 + local] = res["cut_scores"]
            for x, (s, ids) in zip(a, tick):
                assert len(x["cut_scores"]) == len(ids) == len(b[s])
                got += x["cut_scores"]
                one += b[s]
        got, one = np.asarray(got), np.asarray(one)
        ref = 1 - golden["stream_probs_assistant"][:, 0]
        print(f"two devices at once vs the same blocks one after the other: max |d cut| {np.abs(got - one).max():.3g}; "
              f"vs reference {np.abs(got - ref).max():.3g}")
        # Runs of the engine are not bit-reproducible: split-K partial sums reach the fp32 residual by atomic
        # reduce-add in no fixed order, and a one-ulp difference can flip an fp16 rounding of the recurrent state,
        # which then carries through the stream (measured ~4e-4 over these 779 tokens, either way of arranging the
        # slots). The bound here is half the parity bound; both arrangements are also checked against the reference.
        assert np.abs(got - one).max() < 1e-3
        assert np.abs(got - ref).max() < P_TOL
        lengths = np.concatenate([g.engine.length for g in sharded.guards])
        np.testing.assert_array_equal(lengths[:3], golden["stream_length"])
        sharded.reset()
        assert not any(g.engine.length.any() for g in sharded.guards)
    finally:
        sharded.close()
        for g in blocks:
            g.engine.close()
