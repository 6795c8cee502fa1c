"""hsg_gemm_f32_noalloc (the GEMM whose bf16 operand pair lives in a scratch area compiled into the library) against
hsg_gemm given the same operand pair split by torch, through the C ABI, on two calls in a row per mode.

The file name sorts last so the test also runs after every other test in the session; it passes alone too."""
import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ELEMS = 1 << 21  # HSG_NOALLOC_MAX_ELEMS in include/hsg.h


@pytest.fixture(scope="module")
def L():
    from hs_guard_b200 import _lib
    from hs_guard_b200.build import build
    build()
    return _lib


def _split(x):
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return hi.contiguous(), lo.contiguous()


def _err():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


def _sync_ok(err):
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"device error flag {int(err.item())}"


@pytest.mark.parametrize("mode,m,n,k,splits", [(0, 200, 384, 1024, 0), (1, 352, 1024, 2048, 4),
                                               (2, 77, 1024, 1024, 0), (0, 2048, 256, 1024, 0)])
def test_noalloc_gemm_matches_hsg_gemm(L, mode, m, n, k, splits):
    lib = L.lib()
    gen = torch.Generator(device="cuda").manual_seed(1000 + mode)
    w = (torch.randn(n, k, device="cuda", generator=gen) * 0.03).to(torch.bfloat16)
    hi, lo = _split(torch.randn(m, k, device="cuda", generator=gen))
    err = _err()

    def outputs():
        if mode == 2:
            return (torch.zeros(m, n // 2, dtype=torch.bfloat16, device="cuda"),
                    torch.zeros(m, n // 2, dtype=torch.bfloat16, device="cuda"))
        return torch.zeros(m, n, device="cuda"), None

    def ptrs(out):
        if mode == 2:
            return None, out[0].data_ptr(), out[1].data_ptr()
        return out[0].data_ptr(), None, None

    def value(out):
        return out[0].double() + out[1].double() if mode == 2 else out[0].double()

    ref_out = outputs()
    y, ah, al = ptrs(ref_out)
    L.check(lib.hsg_gemm(w.data_ptr(), n, k, hi.data_ptr(), lo.data_ptr(), m, m, y, ah, al, mode, splits,
                         err.data_ptr(), None))
    _sync_ok(err)
    ref = value(ref_out)
    scale = float(ref.abs().max())
    x = (hi.float() + lo.float()).clone()
    out = outputs()
    y, ah, al = ptrs(out)
    for call in range(2):
        # the same fp32 values rewritten in place each call, so the second call cannot reuse the first's split
        x.copy_(hi.float() + lo.float())
        for t in out:
            if t is not None:
                t.zero_()
        torch.cuda.synchronize()
        free_before, held_before = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
        L.check(lib.hsg_gemm_f32_noalloc(w.data_ptr(), n, k, x.data_ptr(), m, y, ah, al, mode, splits,
                                         err.data_ptr(), None))
        _sync_ok(err)
        if call == 1:  # the first call on a device may load the module; every later call allocates nothing
            assert torch.cuda.mem_get_info()[0] == free_before, "device memory changed across the call"
            assert torch.cuda.memory_allocated() == held_before
        diff = float((value(out) - ref).abs().max())
        assert diff <= 1e-5 * scale + 1e-6, f"call {call}: max |diff| {diff} (scale {scale})"


def test_noalloc_gemm_rejects_oversize_and_bad_args(L):
    lib = L.lib()
    w = torch.zeros(128, 64, dtype=torch.bfloat16, device="cuda")
    x = torch.zeros(8, 64, device="cuda")
    y = torch.zeros(8, 128, device="cuda")
    m = MAX_ELEMS // 64 + 1
    with pytest.raises(ValueError, match="HSG_NOALLOC_MAX_ELEMS"):
        L.check(lib.hsg_gemm_f32_noalloc(w.data_ptr(), 128, 64, x.data_ptr(), m, y.data_ptr(), None, None, 0, 0,
                                         None, None))
    with pytest.raises(ValueError):
        L.check(lib.hsg_gemm_f32_noalloc(w.data_ptr(), 100, 64, x.data_ptr(), 8, y.data_ptr(), None, None, 0, 0,
                                         None, None))
    with pytest.raises(ValueError):
        L.check(lib.hsg_gemm_f32_noalloc(w.data_ptr(), 128, 64, x.data_ptr() + 4, 8, y.data_ptr(), None, None, 0, 0,
                                         None, None))
