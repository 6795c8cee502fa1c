"""ctypes binding of libhsg.so (the C ABI declared in include/hsg.h).

The library is the only compute path: if it is missing or fails to load, ``lib()`` raises; nothing falls back to
the CPU. Build it with ``python -m hs_guard_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libhsg.so")

HSG_OK, HSG_ERR_INVALID, HSG_ERR_CUDA, HSG_ERR_DEVICE, HSG_ERR_UNSUPPORTED = 0, -1, -2, -3, -4
HSG_FLAG_BF16_ACT = 1
HSG_FLAG_STATE_F32 = 2
HSG_STATE_F32, HSG_STATE_F16 = 0, 1
N_LAYERS = 24
HSG_PROF_N = 13
PROF_NAMES = ("embed", "gemm_in", "gdn", "attn_prep", "ring_attn", "ring_append", "gemm_out", "norm", "gemm_gu",
              "gemm_down", "head_gemm", "head", "commit")


class Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden", "intermediate", "n_layers", "full_attn_interval", "gdn_heads",
                                          "gdn_head_dim", "conv_kernel", "attn_heads", "kv_heads", "attn_head_dim",
                                          "rotary_dim", "vocab", "window", "head_hidden", "n_classes", "n_roles")] + \
              [("rms_eps", C.c_float), ("head_ln_eps", C.c_float)]


class LayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("w_in", "w_out", "w_gu", "w_down", "norm_in", "norm_post", "conv_w",
                                          "A_log", "dt_bias", "gnorm_w", "q_norm", "k_norm")]


class Weights(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("final_norm", C.c_void_p), ("inv_freq", C.c_void_p),
                ("layers", LayerWeights * N_LAYERS)] + \
               [(n, C.c_void_p) for n in ("head_w1", "head_b1", "head_ln_w", "head_ln_b", "head_w2", "head_b2")]


class Pools(C.Structure):
    _fields_ = [("rec", C.c_void_p), ("conv", C.c_void_p), ("ring_k", C.c_void_p), ("ring_v", C.c_void_p),
                ("ring_pos", C.c_void_p), ("max_slots", C.c_int32), ("n_gdn", C.c_int32), ("n_attn", C.c_int32),
                ("rec_dtype", C.c_int32)]


class HsgError(RuntimeError):
    """A libhsg call failed; ``code`` is the HSG_ERR_* value."""

    def __init__(self, code, message):
        super().__init__(message)
        self.code = code


_LIB = None
P, I, F = C.c_void_p, C.c_int, C.c_float


def lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m hs_guard_b200.build`")
        L = C.CDLL(LIB_PATH)
        sig = {
            "hsg_create": [C.POINTER(Config), C.POINTER(Weights), I, I, I, C.POINTER(P)],
            "hsg_destroy": [P],
            "hsg_step": [P, P, I, I, P],
            "hsg_stage": [P, P, I, I],
            "hsg_launch": [P, P, I, I],
            "hsg_fetch": [P, I, I, P],
            "hsg_synchronize": [P],
            "hsg_reset_all": [P],
            "hsg_reset_slot": [P, I],
            "hsg_snapshot_slot": [P, I, P],
            "hsg_restore_slot": [P, I, P],
            "hsg_get_pools": [P, C.POINTER(Pools)],
            "hsg_profile_step": [P, P, I, I, P, P, P],
            "hsg_launches_per_step": [P, I, I],
            "hsg_gdn_step": [P, P, P, P, P, P, I, P, P, I, I, I, P, P, P],
            "hsg_ring_attention": [P, P, P, P, P, P, P, P, P, I, I, I, F, P, I, P, P],
            "hsg_gemm": [P, I, I, P, P, I, I, P, P, P, I, I, P, P],
            "hsg_gemm_f32_noalloc": [P, I, I, P, I, P, P, P, I, I, P, P],
            "hsg_check_bounded_wait": [I, C.POINTER(C.c_double)],
        }
        for name, args in sig.items():
            fn = getattr(L, name)
            fn.argtypes, fn.restype = args, C.c_int
        L.hsg_slot_state_bytes.argtypes, L.hsg_slot_state_bytes.restype = [P], C.c_size_t
        L.hsg_stream.argtypes, L.hsg_stream.restype = [P], P
        L.hsg_last_error.argtypes, L.hsg_last_error.restype = [], C.c_char_p
        L.hsg_version.argtypes, L.hsg_version.restype = [], C.c_char_p
        _LIB = L
    return _LIB


def check(rc):
    """Raise on a negative status: ValueError for invalid arguments (the reference's error type for bad input),
    HsgError otherwise."""
    if rc == HSG_OK:
        return rc
    msg = lib().hsg_last_error().decode(errors="replace")
    if rc == HSG_ERR_INVALID:
        raise ValueError(msg)
    raise HsgError(rc, msg)


def ptr(t):
    """Device (or host) address of a tensor / numpy array, for the C ABI."""
    if t is None:
        return None
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    return t.ctypes.data
