"""Slot engine host: the B200 counterpart of the reference's SlotStreamEngineV7/V8 host loop.

It keeps the reference's host-side contract (engine/slot_engine_v7.py:88-167, engine/bucketed_engine.py:8-16):
per-slot lengths on the host, ticks of at most 64 tokens per row and at most the largest session bucket of rows,
bucket choice (rows from ``session_buckets``, tokens from 1, 2, 4, ..., 64), the ``pack_inputs`` buffer, and the
return formats of ``step`` and ``step_packed``. Everything on the device -- state pools, the CUDA graph per
(rows, tokens) bucket, every kernel -- lives in libhsg.so behind the C ABI of include/hsg.h.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from ._lib import check, ptr
from .build import host
from .config import DEFAULT, ROLES, SESSION_BUCKETS, TOKEN_BUCKETS, HsgConfig
from .pack import pack_inputs
from .weights import engine_layout, extract_state_dict


def bucket(value, choices):
    for c in choices:
        if value <= c:
            return c
    raise ValueError(f"{value} exceeds the largest bucket {choices[-1]}")


def default_session_buckets(max_slots):
    """The row buckets StreamingGuard uses (reference runtime.py:154-156)."""
    b = tuple(x for x in SESSION_BUCKETS if x <= max_slots)
    if not b or b[-1] != max_slots:
        b += (max_slots,)
    return b


def c_config(cfg: HsgConfig):
    return _lib.Config(hidden=cfg.hidden, intermediate=cfg.intermediate, n_layers=cfg.n_layers,
                       full_attn_interval=cfg.full_attn_interval, gdn_heads=cfg.gdn_heads,
                       gdn_head_dim=cfg.gdn_head_dim, conv_kernel=cfg.conv_kernel, attn_heads=cfg.attn_heads,
                       kv_heads=cfg.kv_heads, attn_head_dim=cfg.attn_head_dim, rotary_dim=cfg.rotary_dim,
                       vocab=cfg.vocab, window=cfg.window, head_hidden=cfg.head_hidden, n_classes=cfg.n_classes,
                       n_roles=len(cfg.roles), rms_eps=cfg.rms_eps, head_ln_eps=cfg.head_ln_eps)


def c_weights(dev):
    w = _lib.Weights()
    w.embed, w.final_norm, w.inv_freq = ptr(dev["embed"]), ptr(dev["final_norm"]), ptr(dev["inv_freq"])
    for i, lay in enumerate(dev["layers"]):
        L = w.layers[i]
        for name in ("w_in", "w_out", "w_gu", "w_down", "norm_in", "norm_post", "conv_w", "A_log", "dt_bias",
                     "gnorm_w", "q_norm", "k_norm"):
            setattr(L, name, ptr(lay.get(name)))
    for name in ("head_w1", "head_b1", "head_ln_w", "head_ln_b", "head_w2", "head_b2"):
        setattr(w, name, ptr(dev[name]))
    return w


class SlotEngine:
    """Fixed per-slot state pools on one GPU and one tick per call (see module docstring).

    model: a reference ``Classifier`` (``.backbone`` + ``.heads``), a ``RandomInitModel`` or a reference-named state
    dict. ``state_dtype`` is the recurrent state's storage type, "float16" (what the reference's StreamingGuard
    uses, runtime.py:157) or "float32". ``precise_activations=False`` feeds the tensor cores bf16 activations only
    (the reference's autocast precision) instead of the hi/lo pair.
    """

    def __init__(self, model, max_slots, head="redline", device=None, session_buckets=None,
                 precise_activations=True, roles=ROLES, state_dtype="float16"):
        if not isinstance(max_slots, int) or max_slots < 1:
            raise ValueError("max_slots must be a positive integer")
        if state_dtype not in ("float16", "float32"):
            raise ValueError("state_dtype must be float16 or float32")
        if tuple(roles) != ROLES:
            raise ValueError("the engine computes both roles (user, assistant)")
        cfg, sd = extract_state_dict(model, head)
        self.cfg = cfg.check()
        self.max_slots, self.roles = max_slots, tuple(roles)
        self.session_buckets = tuple(session_buckets) if session_buckets else default_session_buckets(max_slots)
        if self.session_buckets[-1] > max_slots:
            raise ValueError("session buckets larger than max_slots")
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        self._lib = _lib.lib()
        with torch.cuda.device(self.device):
            self.weights = engine_layout(sd, cfg, self.device)
        self._cw = c_weights(self.weights)
        self._cc = c_config(cfg)
        handle = C.c_void_p()
        flags = (0 if precise_activations else _lib.HSG_FLAG_BF16_ACT) | \
            (_lib.HSG_FLAG_STATE_F32 if state_dtype == "float32" else 0)
        self.state_dtype = state_dtype
        check(self._lib.hsg_create(C.byref(self._cc), C.byref(self._cw), max_slots, self.device.index, flags,
                                   C.byref(handle)))
        self._h = handle
        self.length = np.zeros(max_slots, dtype=np.int64)
        self.host = {}
        self.stats = {"graph_replays": 0, "ticks": 0}

    # ---- lifecycle ----
    def close(self):
        if getattr(self, "_h", None):
            self._lib.hsg_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        if not self._h:
            raise RuntimeError("engine is closed")
        return self._h

    def reset(self):
        """Zero every slot (reference bucketed_engine.py:51-55, slot_engine_v7.py:54-56)."""
        check(self._lib.hsg_reset_all(self.handle))
        self.length[:] = 0

    def reset_slot(self, slot):
        check(self._lib.hsg_reset_slot(self.handle, int(slot)))
        self.length[slot] = 0

    def slot_state_bytes(self):
        return int(self._lib.hsg_slot_state_bytes(self.handle))

    def snapshot_slot(self, slot):
        """(device uint8 tensor with every pool row of ``slot``, its length) -- the demo's checkpoint
        (examples/demo/runtime_v10.py:98-111)."""
        buf = torch.empty(self.slot_state_bytes(), dtype=torch.uint8, device=self.device)
        check(self._lib.hsg_snapshot_slot(self.handle, int(slot), ptr(buf)))
        return buf, int(self.length[slot])

    def restore_slot(self, slot, snapshot):
        buf, length = snapshot
        if buf.numel() != self.slot_state_bytes() or buf.device != self.device:
            raise ValueError("snapshot does not belong to this engine")
        check(self._lib.hsg_restore_slot(self.handle, int(slot), ptr(buf)))
        self.length[slot] = length

    def pools(self):
        """torch views of the device pools: rec, conv, ring_k, ring_v, ring_pos (for tests and diagnostics)."""
        p = _lib.Pools()
        check(self._lib.hsg_get_pools(self.handle, C.byref(p)))
        S1 = p.max_slots + 1
        c = self.cfg

        def view(addr, shape, dtype):
            return _from_device(addr, int(np.prod(shape)), dtype, self.device).view(shape)
        rec_dtype = torch.float16 if p.rec_dtype == _lib.HSG_STATE_F16 else torch.float32
        return {"rec": view(p.rec, (p.n_gdn, S1, c.gdn_heads, c.gdn_head_dim, c.gdn_head_dim), rec_dtype),
                "conv": view(p.conv, (p.n_gdn, S1, c.conv_kernel - 1, c.conv_dim), torch.float32),
                "ring_k": view(p.ring_k, (p.n_attn, S1, c.kv_heads, c.window + 1, c.attn_head_dim), torch.float16),
                "ring_v": view(p.ring_v, (p.n_attn, S1, c.kv_heads, c.window + 1, c.attn_head_dim), torch.float16),
                "ring_pos": view(p.ring_pos, (S1, c.window + 1), torch.int64)}

    # ---- one tick ----
    def _buffers(self, nb, lb):
        key = (nb, lb)
        if key not in self.host:
            hin = torch.zeros(nb * lb + 3 * nb, dtype=torch.int64, pin_memory=True)
            hout = torch.zeros(len(self.roles), nb, lb, 3, dtype=torch.float32, pin_memory=True)
            self.host[key] = (hin, hin.numpy(), hout, hout.numpy())
        return self.host[key]

    def run_arrays(self, chunks, slots):
        """One tick of <= largest-bucket rows, <= 64 tokens each (reference slot_engine_v7.py:117-136).
        Returns ([roles, n, lb, 3] numpy copy, lens)."""
        n = len(chunks)
        nb = bucket(n, self.session_buckets)
        lb = bucket(max(len(c) for c in chunks), TOKEN_BUCKETS)
        hin, hin_np, hout, out_np = self._buffers(nb, lb)
        slots = np.asarray(slots, dtype=np.int64)
        lens = pack_inputs(chunks, slots, nb, lb, self.length, self.max_slots, hin_np)
        check(self._lib.hsg_step(self.handle, ptr(hin), nb, lb, ptr(hout)))
        self.stats["graph_replays"] += 1
        self.stats["ticks"] += 1
        self.length[slots] += lens
        return out_np[:, :n].copy(), lens

    def step_packed(self, requests):
        """One tick without per-row objects (reference slot_engine_v7.py:138-145)."""
        slots = np.fromiter((s for s, _ in requests), dtype=np.int64, count=len(requests))
        if len(np.unique(slots)) != len(slots):
            raise ValueError("a session may appear once per tick")
        return self.run_arrays([c for _, c in requests], slots)

    def run_tokens(self, slots, ids):
        """One tick of one token per row (``slots`` and ``ids`` as lists, already validated): the packed layout of
        pack_inputs with lb = 1, filled without per-row lists. Returns ([roles, n, 1, 3] numpy copy, lens)."""
        n = len(slots)
        nb = bucket(n, self.session_buckets)
        hin, hin_np, hout, out_np = self._buffers(nb, 1)
        sl = np.asarray(slots, dtype=np.int64)
        hin_np[:nb] = 0
        hin_np[:n] = ids
        tail = hin_np[nb:4 * nb].reshape(3, nb)
        tail[0].fill(0)
        tail[0, :n] = 1
        tail[1].fill(self.max_slots)
        tail[1, :n] = sl
        tail[2].fill(0)
        tail[2, :n] = self.length[sl]
        check(self._lib.hsg_step(self.handle, ptr(hin), nb, 1, ptr(hout)))
        self.stats["graph_replays"] += 1
        self.stats["ticks"] += 1
        self.length[sl] += 1
        return out_np[:, :n].copy(), np.ones(n, dtype=np.int64)

    def run_requests(self, requests):
        """One tick straight from the request list when it is a list of (int slot, [int ids]) that fits one
        launch (<= largest row bucket, <= 64 ids each): the reference's validation (runtime.py:161-171), the
        packing and the length update run in C (``_hsg_host``). Returns (probs [roles, nb, lb, 3] host view,
        valid until the next tick; n; nb; lb), or None when the requests need the general path -- which is also
        where every invalid input gets its error."""
        if type(requests) is not list:
            return None
        n = len(requests)
        if not 0 < n <= self.session_buckets[-1]:
            return None
        h = host()
        longest = h.scan(requests, self.max_slots, self.cfg.vocab)
        if not 0 < longest <= TOKEN_BUCKETS[-1]:
            return None
        nb, lb = bucket(n, self.session_buckets), bucket(longest, TOKEN_BUCKETS)
        hin, hin_np, hout, out_np = self._buffers(nb, lb)
        h.fill(requests, hin_np, nb, lb, self.length, self.max_slots)
        check(self._lib.hsg_step(self.handle, ptr(hin), nb, lb, ptr(hout)))
        self.stats["graph_replays"] += 1
        self.stats["ticks"] += 1
        h.advance(self.length, hin_np, nb, lb, n)
        return out_np, n, nb, lb

    def fits_one_tick(self, requests):
        """Whether ``requests`` run as a single tick (<= largest row bucket, every request <= 64 tokens)."""
        largest = TOKEN_BUCKETS[-1]
        return len(requests) <= self.session_buckets[-1] and all(len(ids) <= largest for _, ids in requests)

    def tick(self, requests):
        """One tick for requests that fit one (``fits_one_tick``): ([roles, n, lb, 3] probabilities, lens)."""
        slots = np.fromiter((s for s, _ in requests), dtype=np.int64, count=len(requests))
        return self.run_arrays([ids for _, ids in requests], slots)

    def step(self, requests):
        """requests [(slot, token_ids)], each slot at most once -> {role: [np.ndarray [L_i, 3]]}.

        Long requests run as consecutive <=64-token ticks with the reference's schedule (slot_engine_v7.py:147-167):
        round r carries token piece r of every request longer than 64 r, in request order, in groups of at most the
        largest row bucket. Each request's probabilities are written into one preallocated array per role."""
        if len({s for s, _ in requests}) != len(requests):
            raise ValueError("a session may appear once per tick")
        if requests and self.fits_one_tick(requests):
            probs, lens = self.tick(requests)
            return {role: [probs[r, row, :n] for row, n in enumerate(lens.tolist())]
                    for r, role in enumerate(self.roles)}
        piece = TOKEN_BUCKETS[-1]
        sizes = [len(ids) for _, ids in requests]
        out = np.empty((len(self.roles), sum(sizes), 3), dtype=np.float32)
        first = np.concatenate([[0], np.cumsum(sizes)[:-1]]).astype(np.int64)  # each request's offset in ``out``
        for group, off in _tick_schedule(sizes, piece, self.session_buckets[-1]):
            chunks = [requests[i][1][off:off + piece] for i in group]
            probs, lens = self.run_arrays(chunks, np.fromiter((requests[i][0] for i in group), dtype=np.int64,
                                                              count=len(group)))
            for row, (i, n) in enumerate(zip(group, lens.tolist())):
                out[:, first[i] + off:first[i] + off + n] = probs[:, row, :n]
        return {role: [out[r, first[i]:first[i] + n] for i, n in enumerate(sizes)]
                for r, role in enumerate(self.roles)}

    # ---- measurement helpers ----
    def profile_tick(self, chunks, slots):
        """Run one tick eagerly with per-kernel CUDA-event timing. Returns (probs, {kernel: (ms, launches)})."""
        n = len(chunks)
        nb = bucket(n, self.session_buckets)
        lb = bucket(max(len(c) for c in chunks), TOKEN_BUCKETS)
        hin, hin_np, hout, out_np = self._buffers(nb, lb)
        slots = np.asarray(slots, dtype=np.int64)
        lens = pack_inputs(chunks, slots, nb, lb, self.length, self.max_slots, hin_np)
        ms = (C.c_float * _lib.HSG_PROF_N)()
        cnt = (C.c_int * _lib.HSG_PROF_N)()
        check(self._lib.hsg_profile_step(self.handle, ptr(hin), nb, lb, ptr(hout), ms, cnt))
        self.length[slots] += lens
        return out_np[:, :n].copy(), {name: (ms[i], cnt[i]) for i, name in enumerate(_lib.PROF_NAMES)}

    def launches_per_step(self, nb, lb):
        return int(self._lib.hsg_launches_per_step(self.handle, nb, lb))


def _tick_schedule(sizes, piece, rows):
    """The ticks that carry requests of ``sizes`` tokens in pieces of ``piece``: yields (request indices, token
    offset) per tick. Round r (offset r * piece) holds every request still longer than the offset, in request order,
    split into groups of at most ``rows``; a request's pieces therefore run in order, one per round."""
    rounds = max((n + piece - 1) // piece for n in sizes) if sizes else 0
    for r in range(rounds):
        live = [i for i, n in enumerate(sizes) if n > r * piece]
        for g in range(0, len(live), rows):
            yield live[g:g + rows], r * piece


def _from_device(addr, numel, dtype, device):
    """A torch tensor aliasing ``numel`` elements of device memory at ``addr`` (owned by the engine)."""
    class _Arr:
        __cuda_array_interface__ = {
            "shape": (numel,), "typestr": {torch.float32: "<f4", torch.float16: "<f2", torch.int64: "<i8"}[dtype],
            "data": (int(addr), False), "version": 3, "strides": None}
    with torch.cuda.device(device):
        return torch.as_tensor(_Arr(), device=device)
