"""Kernel parity on a B200 through the C ABI: tensor-core GEMM, gated-delta-rule step, ring-window attention."""
import ctypes as C

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from golden_inputs import gdn_raw, ring_inputs, ring_positions
from oracle import kernels as K

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    from hs_guard_b200 import _lib
    from hs_guard_b200.build import build
    build()
    return _lib


def _err():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


def _done(L, err):
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"device error flag {int(err.item())}"


def _split(x):
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return hi.contiguous(), lo.contiguous()


# ---- GEMM -------------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("m", [1, 16, 33, 176, 352, 600])
@pytest.mark.parametrize("use_lo", [True, False])
def test_gemm_store(L, m, use_lo):
    torch.manual_seed(m)
    n, k = 384, 1024
    w = (torch.randn(n, k, device="cuda") * 0.05).to(torch.bfloat16)
    x = torch.randn(m + 40, k, device="cuda")
    hi, lo = _split(x)
    y = torch.full((m + 40, n), 7.0, device="cuda")
    err = _err()
    L.check(L.lib().hsg_gemm(w.data_ptr(), n, k, hi.data_ptr(), lo.data_ptr() if use_lo else None, m, m + 40,
                             y.data_ptr(), None, None, 0, 0, err.data_ptr(), None))
    _done(L, err)
    xin = (hi.double() + lo.double()) if use_lo else hi.double()
    ref = (xin[:m] @ w.double().T).float()
    torch.testing.assert_close(y[:m], ref, rtol=1e-4, atol=1e-4)
    assert torch.all(y[m:] == 7.0), "rows beyond m must not be written"


@pytest.mark.parametrize("m,splits", [(1, 4), (352, 0), (352, 8), (100, 3)])
def test_gemm_atomic_split_k(L, m, splits):
    torch.manual_seed(1)
    n, k = 1024, 2048
    w = (torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, device="cuda")
    hi, lo = _split(x)
    base = torch.randn(m, n, device="cuda")
    y = base.clone()
    err = _err()
    L.check(L.lib().hsg_gemm(w.data_ptr(), n, k, hi.data_ptr(), lo.data_ptr(), m, m, y.data_ptr(), None, None,
                             1, splits, err.data_ptr(), None))
    _done(L, err)
    ref = (base.double() + (hi.double() + lo.double()) @ w.double().T).float()
    torch.testing.assert_close(y, ref, rtol=1e-4, atol=2e-4)


@pytest.mark.parametrize("m", [5, 352])
def test_gemm_silu_mul(L, m):
    torch.manual_seed(2)
    f, k = 512, 1024
    g = (torch.randn(f, k, device="cuda") * 0.03).to(torch.bfloat16)
    u = (torch.randn(f, k, device="cuda") * 0.03).to(torch.bfloat16)
    w = torch.stack([g, u], 1).reshape(2 * f, k).contiguous()
    x = torch.randn(m, k, device="cuda")
    hi, lo = _split(x)
    ahi = torch.zeros(m, f, dtype=torch.bfloat16, device="cuda")
    alo = torch.zeros_like(ahi)
    err = _err()
    L.check(L.lib().hsg_gemm(w.data_ptr(), 2 * f, k, hi.data_ptr(), lo.data_ptr(), m, m, None, ahi.data_ptr(),
                             alo.data_ptr(), 2, 0, err.data_ptr(), None))
    _done(L, err)
    xin = hi.double() + lo.double()
    ref = F.silu(xin @ g.double().T) * (xin @ u.double().T)
    torch.testing.assert_close(ahi.double() + alo.double(), ref, rtol=1e-4, atol=1e-5)


def test_gemm_rejects_bad_shapes(L):
    with pytest.raises(ValueError):
        L.check(L.lib().hsg_gemm(None, 128, 64, None, None, 1, 1, None, None, None, 0, 0, None, None))
    w = torch.zeros(100, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        L.check(L.lib().hsg_gemm(w.data_ptr(), 100, 64, w.data_ptr(), None, 1, 1, w.data_ptr(), None, None, 0, 0,
                                 None, None))


# ---- gated delta rule -----------------------------------------------------------------------------------------
def _gdn_gpu(L, packed, a, b, state, slots, lens, A_log=None, dt_bias=None):
    n, lb = packed.shape[:2]
    H = 16
    A_log = torch.zeros(H) if A_log is None else A_log
    dt_bias = torch.zeros(H) if dt_bias is None else dt_bias
    dev = dict(packed=packed.to(torch.bfloat16).cuda().contiguous(), a=a.float().cuda().contiguous(),
               b=b.float().cuda().contiguous(), A=A_log.float().cuda(), dt=dt_bias.float().cuda(),
               slots=torch.as_tensor(slots, dtype=torch.int64).cuda(),
               lens=torch.as_tensor(lens, dtype=torch.int64).cuda())
    o = torch.full((n, lb, H, 128), 3.0, device="cuda")
    err = _err()
    dtype = L.HSG_STATE_F16 if state.dtype == torch.float16 else L.HSG_STATE_F32
    L.check(L.lib().hsg_gdn_step(dev["packed"].data_ptr(), dev["a"].data_ptr(), dev["b"].data_ptr(),
                                 dev["A"].data_ptr(), dev["dt"].data_ptr(), state.data_ptr(), dtype,
                                 dev["slots"].data_ptr(), dev["lens"].data_ptr(), n, lb, state.shape[0] - 1,
                                 o.data_ptr(), err.data_ptr(), None))
    _done(L, err)
    return o


@pytest.mark.parametrize("name,n,lb,seed", [("gdn_a", 3, 5, 21), ("gdn_b", 2, 1, 22)])
@pytest.mark.parametrize("state_dtype", [torch.float32, torch.float16])
def test_gdn_step_matches_reference_golden(L, golden, name, n, lb, seed, state_dtype):
    """fp32 state: the reference's fp32 result to 1e-3; fp16 state (the input state rounded to fp16, the result
    stored in fp16 as the reference's StreamingGuard pools do): within fp16 rounding of it."""
    packed, a, b, state = gdn_raw(n, lb, seed)
    pool = torch.zeros(n + 1, 16, 128, 128, device="cuda", dtype=state_dtype)
    pool[:n] = state.cuda().to(state_dtype)
    o = _gdn_gpu(L, packed, a, b, pool, np.arange(n), [lb] * n)
    f16 = state_dtype == torch.float16
    np.testing.assert_allclose(o.cpu().numpy(), golden[name + "_o"], rtol=1e-2 if f16 else 1e-3,
                               atol=1e-3 if f16 else 1e-4)
    norms = pool[:n].float().pow(2).sum((-1, -2)).sqrt().cpu().numpy()
    np.testing.assert_allclose(norms, golden[name + "_state_norm"], rtol=1e-3 if f16 else 1e-4)


def test_gdn_step_padding_and_permuted_slots(L):
    """Rows map to arbitrary slots; rows with lens 0 (scratch slot) and padded tokens give zeros and touch nothing."""
    packed, a, b, state = gdn_raw(4, 4, 5)
    pool = torch.randn(6, 16, 128, 128) * 0.02
    slots, lens = np.array([3, 0, 5, 1]), np.array([4, 2, 0, 1])
    A_log, dt = torch.randn(16) * 0.5, torch.randn(16)
    gpu_pool = pool.cuda()
    o = _gdn_gpu(L, packed, a, b, gpu_pool, slots, lens, A_log, dt)
    ref_pool = pool.clone()
    ref = K.gdn_slot_step(packed, a, b, A_log, dt, ref_pool, torch.from_numpy(slots), torch.from_numpy(lens))
    torch.testing.assert_close(o.cpu(), ref, rtol=1e-3, atol=1e-4)
    torch.testing.assert_close(gpu_pool.cpu(), ref_pool, rtol=1e-4, atol=1e-6)
    assert torch.equal(gpu_pool[5].cpu(), pool[5]) and torch.equal(gpu_pool[2].cpu(), pool[2])


def test_gdn_step_large_batch_fp32(L):
    """More than 32 rows with fp32 state take the persistent kernel (smaller batches the column-slice kernel):
    ragged lengths, a padding row and permuted slots against the oracle."""
    n, lb = 40, 3
    packed, a, b, state = gdn_raw(n, lb, 9)
    S = n + 3
    perm = np.random.default_rng(9).permutation(S)[:n]
    lens = np.array([lb - (i % 3) for i in range(n)])
    lens[7] = 0
    perm[7] = S
    pool = torch.randn(S + 1, 16, 128, 128) * 0.02
    A_log, dt = torch.randn(16) * 0.5, torch.randn(16)
    gpu_pool = pool.cuda()
    o = _gdn_gpu(L, packed, a, b, gpu_pool, perm, lens, A_log, dt)
    ref_pool = pool.clone()
    ref = K.gdn_slot_step(packed, a, b, A_log, dt, ref_pool, torch.from_numpy(perm), torch.from_numpy(lens))
    torch.testing.assert_close(o.cpu(), ref, rtol=1e-3, atol=1e-4)
    torch.testing.assert_close(gpu_pool.cpu(), ref_pool, rtol=1e-4, atol=1e-6)


def test_gdn_config2_size(L):
    """Config 2 in full: 16 slots x 16 heads, fp32 state N(0, 0.02), 1,000 consecutive single-token steps vs the
    oracle (outputs at every step, final state within 1e-3 relative: ten times tighter than the 1e-2 state bound);
    then the same tokens as 64-token ticks plus one 40-token tick must land on the same state (tick-size
    independence)."""
    steps, n = 1000, 16
    packed, a, b, state = gdn_raw(n, steps, 2)
    pool = torch.zeros(n + 1, 16, 128, 128, device="cuda")
    pool[:n] = state.cuda()
    pool2 = pool.clone()
    ref_pool = torch.zeros(n + 1, 16, 128, 128)
    ref_pool[:n] = state
    slots = np.arange(n)
    outs = []
    for t in range(steps):
        outs.append(_gdn_gpu(L, packed[:, t:t + 1], a[:, t:t + 1], b[:, t:t + 1], pool, slots, [1] * n).cpu())
    ref_o = K.gdn_slot_step(packed, a, b, torch.zeros(16), torch.zeros(16), ref_pool, torch.arange(n),
                            torch.full((n,), steps))
    got = torch.cat(outs, 1)
    print(f"config 2, 1000 steps: max |do| {float((got - ref_o).abs().max()):.3g}")
    torch.testing.assert_close(got, ref_o, rtol=2e-3, atol=2e-4)
    rel = float((pool.cpu() - ref_pool).norm() / ref_pool.norm())
    print(f"config 2, 1000 steps: state relative error {rel:.3g}")
    assert rel < 1e-3, rel
    for t0 in range(0, steps, 64):
        t1 = min(t0 + 64, steps)
        _gdn_gpu(L, packed[:, t0:t1], a[:, t0:t1], b[:, t0:t1], pool2, slots, [t1 - t0] * n)
    assert ((pool2 - pool).norm() / pool.norm()) < 1e-4


def test_gdn_config2_size_fp16_state(L):
    """As above with the state stored in fp16 between steps (the reference StreamingGuard's pools): the GPU matches
    an oracle that rounds its state to fp16 after every step, and stays within 1e-2 of the fp32-state oracle."""
    steps, n = 100, 16
    packed, a, b, state = gdn_raw(n, steps, 2)
    pool = torch.zeros(n + 1, 16, 128, 128, device="cuda", dtype=torch.float16)
    pool[:n] = state.cuda().half()
    pool2 = pool.clone()
    ref16 = torch.zeros(n + 1, 16, 128, 128)
    ref16[:n] = state.half().float()
    ref32 = ref16.clone()
    slots = np.arange(n)
    outs, ref_outs = [], []
    for t in range(steps):
        outs.append(_gdn_gpu(L, packed[:, t:t + 1], a[:, t:t + 1], b[:, t:t + 1], pool, slots, [1] * n))
        ref_outs.append(K.gdn_slot_step(packed[:, t:t + 1], a[:, t:t + 1], b[:, t:t + 1], torch.zeros(16),
                                        torch.zeros(16), ref16, torch.arange(n), torch.ones(n, dtype=torch.int64)))
        ref16.copy_(ref16.half().float())
    ref_o32 = K.gdn_slot_step(packed, a, b, torch.zeros(16), torch.zeros(16), ref32, torch.arange(n),
                              torch.full((n,), steps))
    got = torch.cat(outs, 1).cpu()
    torch.testing.assert_close(got, torch.cat(ref_outs, 1), rtol=5e-3, atol=5e-4)
    assert float((got - ref_o32).norm() / ref_o32.norm()) < 1e-2
    rel16 = (pool.cpu().float() - ref16).norm() / ref16.norm()
    rel32 = (pool.cpu().float() - ref32).norm() / ref32.norm()
    assert rel16 < 2e-3 and rel32 < 1e-2, (rel16, rel32)
    _gdn_gpu(L, packed[:, :64], a[:, :64], b[:, :64], pool2, slots, [64] * n)
    _gdn_gpu(L, packed[:, 64:], a[:, 64:], b[:, 64:], pool2, slots, [36] * n)
    assert ((pool2.float() - pool.float()).norm() / pool.float().norm()) < 1e-2


@pytest.mark.parametrize("lb,lens", [(64, [64, 50, 0, 1, 64]), (32, [32, 17, 0, 31, 2])])
def test_gdn_chunked_vs_oracle(L, lb, lens):
    """fp16-state ticks of 32 and 64 tokens run the chunked (WY) kernel: against the token-by-token oracle from the
    same fp16 initial state, with ragged lengths, a padding row on the scratch slot and permuted slots."""
    n = len(lens)
    packed, a, b, state = gdn_raw(n, lb, 70 + lb)
    S = n + 2
    slots = np.array([3, 0, S, 5, 1])[:n]
    g = torch.Generator().manual_seed(lb)
    pool = (torch.randn(S + 1, 16, 128, 128, generator=g) * 0.05).half()
    A_log, dt = torch.randn(16, generator=g) * 0.5, torch.randn(16, generator=g)
    gpu_pool = pool.cuda()
    o = _gdn_gpu(L, packed, a, b, gpu_pool, slots, np.array(lens), A_log, dt)
    ref_pool = pool.float().clone()
    ref = K.gdn_slot_step(packed, a, b, A_log, dt, ref_pool, torch.from_numpy(slots), torch.tensor(lens))
    got = o.cpu()
    assert float((got - ref).norm() / ref.norm()) < 5e-3
    torch.testing.assert_close(got, ref, rtol=2e-2, atol=2e-3)
    rows = [int(s_) for s_, l_ in zip(slots, lens) if l_ > 0]
    new = gpu_pool.float().cpu()
    rel = (new[rows] - ref_pool[rows]).norm() / ref_pool[rows].norm()
    assert rel < 5e-3, rel
    untouched = [r for r in range(S + 1) if r not in rows]
    assert torch.equal(new[untouched], pool.float()[untouched])
    for row, l_ in enumerate(lens):  # padded positions are zero
        assert torch.count_nonzero(got[row, l_:]) == 0


# ---- ring attention ---------------------------------------------------------------------------------------------
def _ring_gpu(L, q, ring_k, ring_v, new_k, new_v, ring_pos, slots, starts, lens, write_ring=0):
    n, _, m, _ = q.shape
    lb = new_k.shape[2]
    d = dict(q=q.float().cuda().contiguous(), rk=ring_k.half().cuda().contiguous(),
             rv=ring_v.half().cuda().contiguous(), nk=new_k.half().cuda().contiguous(),
             nv=new_v.half().cuda().contiguous(), rp=ring_pos.cuda().contiguous(), s=slots.cuda(), st=starts.cuda(),
             ln=lens.cuda())
    out = torch.full(q.shape, 5.0, device="cuda")
    err = _err()
    L.check(L.lib().hsg_ring_attention(d["q"].data_ptr(), d["rk"].data_ptr(), d["rv"].data_ptr(), d["nk"].data_ptr(),
                                       d["nv"].data_ptr(), d["rp"].data_ptr(), d["s"].data_ptr(), d["st"].data_ptr(),
                                       d["ln"].data_ptr(), n, lb, ring_k.shape[0] - 1, 256 ** -0.5, out.data_ptr(),
                                       write_ring, err.data_ptr(), None))
    _done(L, err)
    return out, d


@pytest.mark.parametrize("name,lb", [("ring_a", 1), ("ring_b", 3)])
def test_ring_attention_matches_reference_golden(L, golden, name, lb):
    args = ring_inputs(lb=lb, seed=31 + lb)
    out, _ = _ring_gpu(L, *args)
    np.testing.assert_allclose(out.cpu().numpy(), golden[name + "_o"], rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("lb", [1, 2, 8, 16, 32, 64])
def test_ring_attention_vs_oracle(L, lb):
    q, rk, rv, nk, nv, rp, slots, starts, lens = ring_inputs(lb=lb, seed=40 + lb, n=6)
    # use fp16-rounded K/V on both sides (the engine's ring precision)
    rk, rv, nk, nv = (t.half().float() for t in (rk, rv, nk, nv))
    out, _ = _ring_gpu(L, q, rk, rv, nk, nv, rp, slots, starts, lens)
    ref = K.ring_attention(q, rk, rv, nk, nv, rp, slots, starts, lens, 256 ** -0.5, 512)
    torch.testing.assert_close(out.cpu(), ref, rtol=2e-3, atol=2e-3)


@pytest.mark.parametrize("n", [64, 96])
def test_ring_attention_config3_with_ring_write(L, n):
    """64 slots (config 3), W = 512, 8/2 heads, D = 256, one query each, write position ~ U[0, 512), fill ~ U[1, 512]
    with wrap; the new key/value land in column start % 512 of each slot. 64 slots (128 items, fewer than the SMs) run
    the split-KV kernel on 2-CTA clusters, 96 slots the persistent one-CTA-per-SM kernel of the engine's batches."""
    r = np.random.default_rng(3)
    q = torch.randn(n, 2, 4, 256).bfloat16().float()
    rk = torch.randn(n + 1, 2, 513, 256).half().float()
    rv = torch.randn(n + 1, 2, 513, 256).half().float()
    nk = torch.randn(n, 2, 1, 256).half().float()
    nv = torch.randn(n, 2, 1, 256).half().float()
    rp = np.full((n + 1, 513), -1, dtype=np.int64)
    starts = np.zeros(n, dtype=np.int64)
    for s in range(n):
        wp, filled = int(r.integers(0, 512)), int(r.integers(1, 513))
        start = wp + (512 if filled > wp else 0)
        starts[s] = start
        rp[s] = ring_positions(start, filled)
    slots, lens = torch.arange(n), torch.ones(n, dtype=torch.int64)
    rp, starts = torch.from_numpy(rp), torch.from_numpy(starts)
    out, d = _ring_gpu(L, q, rk, rv, nk, nv, rp, slots, starts, lens, write_ring=1)
    ref = K.ring_attention(q, rk, rv, nk, nv, rp, slots, starts, lens, 256 ** -0.5, 512)
    torch.testing.assert_close(out.cpu(), ref, rtol=2e-3, atol=2e-3)
    ring_k = d["rk"].cpu().float()
    for s in range(n):
        col = int(starts[s]) % 512
        assert torch.equal(ring_k[s, :, col], nk[s, :, 0]), s


@pytest.mark.parametrize("mode,n", [(0, 1024), (1, 1024), (2, 1024), (1, 1152)])
def test_gemm_large_m_persistent(L, mode, n):
    """Long-running grids (>= 4 waves of 256-token tiles) take the persistent kernel: 128 x 256 tiles, or for the
    reduce-add mode 256 x 128 tiles (n = 1152: the last tile's upper weight half lies beyond the matrix)."""
    torch.manual_seed(3)
    m, k = 19000, 1024
    w = (torch.randn(n, k, device="cuda") * 0.03).to(torch.bfloat16)
    x = torch.randn(m, k, device="cuda")
    hi, lo = _split(x)
    xin = hi.double() + lo.double()
    err = _err()
    if mode == 2:
        ahi = torch.zeros(m, n // 2, dtype=torch.bfloat16, device="cuda")
        alo = torch.zeros_like(ahi)
        L.check(L.lib().hsg_gemm(w.data_ptr(), n, k, hi.data_ptr(), lo.data_ptr(), m, m, None, ahi.data_ptr(),
                                 alo.data_ptr(), 2, 0, err.data_ptr(), None))
        _done(L, err)
        g, u = xin @ w[0::2].double().T, xin @ w[1::2].double().T
        torch.testing.assert_close(ahi.double() + alo.double(), F.silu(g) * u, rtol=1e-4, atol=1e-5)
        return
    base = torch.randn(m, n, device="cuda") if mode == 1 else torch.zeros(m, n, device="cuda")
    y = base.clone()
    L.check(L.lib().hsg_gemm(w.data_ptr(), n, k, hi.data_ptr(), lo.data_ptr(), m, m, y.data_ptr(), None, None, mode,
                             0, err.data_ptr(), None))
    _done(L, err)
    ref = ((base.double() if mode == 1 else 0) + xin @ w.double().T).float()
    torch.testing.assert_close(y, ref, rtol=1e-4, atol=2e-4)
