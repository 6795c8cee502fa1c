"""Pin the CPU oracle to the reference: every golden vector in tests/golden/golden.npz was produced by the reference
implementation itself (tests/golden/make_golden.py)."""
import numpy as np
import torch

from golden_inputs import STREAM_MAX_SLOTS, gdn_raw, ring_inputs, sample_index, stream_script
from oracle import kernels as K
from oracle.pack import pack_inputs
from oracle.stream import StreamOracle, score_complete
from hs_guard_b200 import DEFAULT
from hs_guard_b200 import weights as W

PACK_CASES = [([[4, 5, 6]], [0], 2, 4, [7], 1),
              ([[1], [2], [3]], [2, 0, 1], 4, 1, [5, 0, 9], 3),
              ([[10, 11], [12, 13, 14, 15, 16], [17]], [1, 3, 0], 4, 8, [100, 3, 0, 511], 4)]


def test_pack_inputs_matches_reference(golden):
    for i, (chunks, slots, nb, lb, length, max_slots) in enumerate(PACK_CASES):
        buf = np.full(nb * lb + 3 * nb, -7, dtype=np.int64)
        lens = pack_inputs(chunks, slots, nb, lb, np.asarray(length), max_slots, buf)
        np.testing.assert_array_equal(buf, golden[f"pack{i}_out"])
        np.testing.assert_array_equal(lens, golden[f"pack{i}_lens"])


def test_pack_inputs_contract_case():
    # the reference's own unit test (tests/test_contract.py:14-18)
    out = np.empty(2 * 4 + 3 * 2, dtype=np.int64)
    lens = pack_inputs([[4, 5, 6]], [0], 2, 4, np.array([7]), 1, out)
    assert lens.tolist() == [3] and out[:8].tolist() == [4, 5, 6, 0, 0, 0, 0, 0]
    assert out[8:10].tolist() == [3, 0] and out[10:12].tolist() == [0, 1] and out[12:].tolist() == [7, 0]


def test_gdn_step_matches_reference(golden):
    for name, n, L, seed in (("gdn_a", 3, 5, 21), ("gdn_b", 2, 1, 22)):
        packed, a, b, state = gdn_raw(n, L, seed)
        zeros = torch.zeros(16)
        o = K.gdn_slot_step(packed, a, b, zeros, zeros, state, torch.arange(n), torch.full((n,), L))
        np.testing.assert_allclose(o.numpy(), golden[name + "_o"], rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(state.pow(2).sum((-1, -2)).sqrt().numpy(), golden[name + "_state_norm"], rtol=1e-5)
        sample = state.reshape(-1)[torch.from_numpy(sample_index(state.numel(), 4))].numpy()
        np.testing.assert_allclose(sample, golden[name + "_state_sample"], rtol=1e-4, atol=1e-6)


def test_ring_attention_matches_reference(golden):
    for name, lb in (("ring_a", 1), ("ring_b", 3)):
        o = K.ring_attention(*ring_inputs(lb=lb, seed=31 + lb), scale=256 ** -0.5, window=512)
        np.testing.assert_allclose(o.numpy(), golden[name + "_o"], rtol=1e-4, atol=1e-4)


def test_stream_oracle_matches_reference_engine(golden, weights_seed0):
    """The whole streaming engine: per-token probs, lengths, ring positions (bit-exact) and state pools."""
    sd = weights_seed0
    assert W.state_dict_digest(sd) == str(golden["weights_digest"])
    orc = StreamOracle(sd, DEFAULT, STREAM_MAX_SLOTS)
    pu, pa = [], []
    for tick in stream_script():
        res = orc.step(tick)
        pu += res["user"]
        pa += res["assistant"]
    np.testing.assert_allclose(np.concatenate(pu), golden["stream_probs_user"], atol=2e-5)
    np.testing.assert_allclose(np.concatenate(pa), golden["stream_probs_assistant"], atol=2e-5)
    np.testing.assert_array_equal(orc.length, golden["stream_length"])
    np.testing.assert_array_equal(orc.ring_pos.numpy()[:STREAM_MAX_SLOTS], golden["stream_ring_pos"][:STREAM_MAX_SLOTS])
    rec = orc.rec[:, :STREAM_MAX_SLOTS]
    np.testing.assert_allclose(rec.pow(2).sum((-1, -2)).sqrt().numpy(), golden["stream_rec_norm"], rtol=1e-3)
    sample = rec.reshape(-1)[torch.from_numpy(sample_index(rec.numel(), 1))].numpy()
    ref = golden["stream_rec_sample"]
    assert np.abs(sample - ref).max() <= 1e-3 * np.abs(ref).max()
    conv = orc.conv[:, :STREAM_MAX_SLOTS]
    np.testing.assert_allclose(conv.reshape(-1)[torch.from_numpy(sample_index(conv.numel(), 2))].numpy(),
                               golden["stream_conv_sample"], atol=1e-4)
    # complete-message scores of slot 0's stream agree with the streamed ones (the reference's own invariant)
    cm = score_complete(sd, DEFAULT, [t for tick in stream_script() for s, ids in tick if s == 0 for t in ids])
    np.testing.assert_allclose(cm.numpy(), golden["cm_slot0_probs"], atol=5e-5)


def test_long_golden_fixture(weights_seed0):
    """tests/golden/golden_long.npz (the reference on the headline's context lengths, make_golden_long.py): lengths and
    ring positions are the exact windows the script implies, the reference's own stream agrees with its
    complete-message scores, and the oracle's complete-message scorer reproduces the reference's on the ragged
    1,000-token slot."""
    import os
    from golden_inputs import LONG_CONTEXTS, LONG_STEPS, long_script, ring_positions
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden_long.npz"))
    assert W.state_dict_digest(weights_seed0) == str(g["weights_digest"])
    lengths = np.asarray(LONG_CONTEXTS) + LONG_STEPS
    np.testing.assert_array_equal(g["stream_length"], lengths)
    for s, n in enumerate(lengths):
        np.testing.assert_array_equal(g["stream_ring_pos"][s], ring_positions(int(n), 512))
    assert (g["stream_ring_pos"][len(lengths)] == -1).all()
    for r, role in enumerate(("user", "assistant")):
        assert np.abs(g[f"stream_probs_{role}"] - g["cm_probs"][r]).max() < 1e-4
    s = 3
    ids = [t for tick in long_script() for slot, chunk in tick if slot == s for t in chunk]
    off = int(np.sum(lengths[:s]))
    cm = score_complete(weights_seed0, DEFAULT, ids)
    np.testing.assert_allclose(cm.numpy(), g["cm_probs"][:, off:off + len(ids)], atol=5e-5)


def test_chunked_delta_rule_matches_recurrence_and_reference(golden):
    """oracle.kernels.gdn_chunked (the chunked WY form of the reference's complete-message path) against the
    reference's recurrent-rule golden vectors, and against the token-by-token recurrence on long inputs with ragged
    chunks and strong decay (exponents far below the fp32 range must underflow to 0, not 0/0)."""
    from oracle.kernels import gdn_chunked, l2norm
    for name, n, L, seed in (("gdn_a", 3, 5, 21), ("gdn_b", 2, 1, 22)):
        qr, kr, vr, g, beta, state = __import__("golden_inputs").gdn_inputs(n=n, L=L, seed=seed)
        for row in range(n):
            q = l2norm(qr[row]) * 128 ** -0.5
            k = l2norm(kr[row])
            st = state[row].clone()
            o = gdn_chunked(q, k, vr[row], g[row], beta[row], st, chunk=4)
            np.testing.assert_allclose(o.numpy(), golden[name + "_o"][row], rtol=1e-4, atol=1e-5)
            np.testing.assert_allclose(st.pow(2).sum((-1, -2)).sqrt().numpy(), golden[name + "_state_norm"][row],
                                       rtol=1e-5)
    gen = torch.Generator().manual_seed(3)
    T, H, D = 150, 2, 128
    q = l2norm(torch.randn(T, H, D, generator=gen)) * D ** -0.5
    k = l2norm(torch.randn(T, H, D, generator=gen))
    v = torch.randn(T, H, D, generator=gen)
    beta = torch.sigmoid(torch.randn(T, H, generator=gen))
    for scale in (1.0, 40.0):
        g = -torch.nn.functional.softplus(torch.randn(T, H, generator=gen)) * scale
        s0 = torch.randn(H, D, D, generator=gen) * 0.02
        st, ref = s0.clone(), torch.zeros(T, H, D)
        for t in range(T):
            st = st * torch.exp(g[t])[:, None, None]
            st = st + k[t][:, :, None] * (beta[t][:, None] * (v[t] - torch.einsum("hkv,hk->hv", st, k[t])))[:, None]
            ref[t] = torch.einsum("hkv,hk->hv", st, q[t])
        s1 = s0.clone()
        o = gdn_chunked(q, k, v, g, beta, s1, chunk=64)
        assert torch.isfinite(o).all()
        torch.testing.assert_close(o, ref, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(s1, st, rtol=1e-4, atol=1e-6)
