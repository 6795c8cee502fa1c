"""Whole streaming engine and complete-message scorer on the CPU in fp32. Test infrastructure only.

``StreamOracle`` restates the reference's pure-torch slot engine: state pools and scratch slot
(``engine/bucketed_engine.py:37-42``, ring layout of ``engine/slot_engine.py:14-18``), one tick
(``bucketed_engine.py:58-132``), the role heads (``engine/slot_engine_v7.py:58-61``, ``runtime.py:71-74``) and the
host loop that splits requests into <=64-token, <=largest-bucket ticks (``slot_engine_v7.py:117-167``).
``score_complete`` restates the complete-message path (``runtime.py:136-145``): a full causal forward where
attention sees only the last 512 positions (``window_attention.py:34-53``) and the GDN layers run from a zero state.
All math is fp32 on bf16-valued weights.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from .kernels import causal_conv_step, gdn_chunked, gdn_decay, l2norm
from .pack import pack_inputs

SESSION_BUCKETS = (1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 352, 384, 448, 512)
TOKEN_BUCKETS = (1, 2, 4, 8, 16, 32, 64)


def bucket(value, choices):
    for c in choices:
        if value <= c:
            return c
    raise ValueError(f"{value} exceeds the largest bucket {choices[-1]}")


def session_buckets(max_slots):
    """Buckets StreamingGuard builds for ``max_slots`` (reference runtime.py:154-156)."""
    b = tuple(x for x in SESSION_BUCKETS if x <= max_slots)
    if not b or b[-1] != max_slots:
        b += (max_slots,)
    return b


def rms_norm(x, w1, eps):
    """Qwen3_5RMSNorm with the weight pre-added: x * rsqrt(mean(x^2) + eps) * (1 + w)."""
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w1


def rope(x, cos, sin, rot):
    """apply_rotary_pos_emb on the first ``rot`` dims (rotate_half within them); x [..., D], cos/sin [..., rot]."""
    xr, xp = x[..., :rot], x[..., rot:]
    half = rot // 2
    rotated = torch.cat([-xr[..., half:], xr[..., :half]], -1)
    return torch.cat([xr * cos + rotated * sin, xp], -1)


class Weights:
    """fp32 views of a reference-named state dict (see hs_guard_b200.weights)."""

    def __init__(self, sd, cfg):
        self.cfg = cfg
        f = lambda name: sd[name].float()
        self.embed = sd["backbone.embed_tokens.weight"]            # kept bf16; rows gathered then cast
        self.final_norm = 1.0 + f("backbone.norm.weight")
        ang = torch.arange(0, cfg.rotary_dim, 2, dtype=torch.int64).float() / cfg.rotary_dim
        self.inv_freq = 1.0 / (cfg.rope_theta ** ang)
        self.layers = []
        for i, kind in enumerate(cfg.layer_types):
            p = f"backbone.layers.{i}."
            lay = {"kind": kind, "norm_in": 1.0 + f(p + "input_layernorm.weight"),
                   "norm_post": 1.0 + f(p + "post_attention_layernorm.weight"),
                   "gate": f(p + "mlp.gate_proj.weight"), "up": f(p + "mlp.up_proj.weight"),
                   "down": f(p + "mlp.down_proj.weight")}
            if kind == "linear_attention":
                a = p + "linear_attn."
                for k in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj"):
                    lay[k] = f(a + k + ".weight")
                lay["conv_w"] = f(a + "conv1d.weight").reshape(cfg.conv_dim, cfg.conv_kernel)
                lay["A_log"], lay["dt_bias"], lay["gnorm"] = f(a + "A_log"), f(a + "dt_bias"), f(a + "norm.weight")
            else:
                a = p + "self_attn."
                for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
                    lay[k] = f(a + k + ".weight")
                lay["q_norm"], lay["k_norm"] = 1.0 + f(a + "q_norm.weight"), 1.0 + f(a + "k_norm.weight")
            self.layers.append(lay)
        self.heads = {}
        for role in cfg.roles:
            q = f"heads.{role}."
            self.heads[role] = tuple(f(q + n) for n in ("projection.0.weight", "projection.0.bias",
                                                        "projection.1.weight", "projection.1.bias",
                                                        "risk.weight", "risk.bias"))

    def cos_sin(self, pos):
        freqs = pos.float()[..., None] * self.inv_freq
        emb = torch.cat([freqs, freqs], -1)
        return emb.cos(), emb.sin()

    def readout(self, hidden, role):
        """Risk logits: Linear -> LayerNorm(eps 1e-5) -> SiLU -> Linear (reference runtime.py:71-74)."""
        w1, b1, lw, lb, w2, b2 = self.heads[role]
        x = F.linear(hidden, w1, b1)
        x = F.layer_norm(x, (x.shape[-1],), lw, lb, self.cfg.head_ln_eps)
        return F.linear(F.silu(x), w2, b2)

    def mlp(self, lay, x):
        return F.linear(F.silu(F.linear(x, lay["gate"])) * F.linear(x, lay["up"]), lay["down"])

    def gated_norm(self, lay, o, z):
        """Qwen3_5RMSNormGated over dv: w * (o * rsqrt(mean(o^2) + eps)) * silu(z)."""
        o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + self.cfg.rms_eps)
        return lay["gnorm"] * o * F.silu(z)


class StreamOracle:
    """fp32 CPU restatement of the slot-based streaming engine (see module docstring)."""

    def __init__(self, sd, cfg, max_slots, window=512):
        self.w, self.cfg, self.window, self.max_slots = Weights(sd, cfg), cfg, window, max_slots
        self.buckets = session_buckets(max_slots)
        s, c = max_slots + 1, cfg
        self.rec = torch.zeros(c.n_gdn, s, c.gdn_heads, c.gdn_head_dim, c.gdn_head_dim)
        self.conv = torch.zeros(c.n_gdn, s, c.conv_kernel - 1, c.conv_dim)
        self.ring_k = torch.zeros(c.n_attn, s, c.kv_heads, window + 1, c.attn_head_dim)
        self.ring_v = torch.zeros_like(self.ring_k)
        self.ring_pos = torch.full((s, window + 1), -1, dtype=torch.int64)
        self.length = np.zeros(max_slots, dtype=np.int64)

    def reset(self):
        for t in (self.rec, self.conv, self.ring_k, self.ring_v):
            t.zero_()
        self.ring_pos.fill_(-1)
        self.length[:] = 0

    # ---- one tick --------------------------------------------------------------------------------------------
    @torch.no_grad()
    def tick(self, ids, lens, slots, starts):
        """ids [nb, lb], lens/slots/starts [nb] int64 -> probs [roles, nb, lb, 3] fp32."""
        cfg, w, W = self.cfg, self.w, self.window
        nb, lb = ids.shape
        steps = torch.arange(lb)
        valid = steps[None] < lens[:, None]
        pos = starts[:, None] + steps[None]
        hidden = w.embed[ids].float()
        cos, sin = w.cos_sin(pos)
        ring_col = torch.where(valid, pos % W, torch.full_like(pos, W))
        for lay, (kind, index) in zip(w.layers, cfg.layer_index()):
            x = rms_norm(hidden, lay["norm_in"], cfg.rms_eps)
            if kind == "linear_attention":
                mixed = self._gdn(lay, x, index, slots, lens, valid)
            else:
                mixed = self._attention(lay, x, index, slots, pos, valid, cos, sin, ring_col)
            hidden = hidden + mixed
            hidden = hidden + w.mlp(lay, rms_norm(hidden, lay["norm_post"], cfg.rms_eps))
        hidden = rms_norm(hidden, w.final_norm, cfg.rms_eps)
        probs = torch.stack([torch.softmax(w.readout(hidden, role), -1) for role in cfg.roles])
        self.ring_pos[slots[:, None], ring_col] = torch.where(valid, pos, torch.full_like(pos, -1))
        return probs

    def _gdn(self, lay, x, gi, slots, lens, valid):
        cfg = self.cfg
        nb, lb, _ = x.shape
        H, D = cfg.gdn_heads, cfg.gdn_head_dim
        qkv = F.linear(x, lay["in_proj_qkv"])
        z = F.linear(x, lay["in_proj_z"]).reshape(nb, lb, H, D)
        b, a = F.linear(x, lay["in_proj_b"]), F.linear(x, lay["in_proj_a"])
        conv = causal_conv_step(qkv, self.conv[gi], lay["conv_w"], slots, lens)
        kd = cfg.key_dim
        q = l2norm(conv[..., :kd].reshape(nb, lb, H, D)) * D ** -0.5
        k = l2norm(conv[..., kd:2 * kd].reshape(nb, lb, H, D))
        v = conv[..., 2 * kd:].reshape(nb, lb, H, D)
        mask = valid[:, :, None].float()
        beta = torch.sigmoid(b) * mask
        g = gdn_decay(a, lay["A_log"], lay["dt_bias"]) * mask
        state = self.rec[gi, slots].clone()                      # [nb, H, dk, dv]
        out = torch.zeros(nb, lb, H, D)
        for t in range(lb):
            state = state * torch.exp(g[:, t])[:, :, None, None]
            kv = torch.einsum("nhkv,nhk->nhv", state, k[:, t])
            delta = beta[:, t, :, None] * (v[:, t] - kv)
            state = state + k[:, t, :, :, None] * delta[:, :, None, :]
            out[:, t] = torch.einsum("nhkv,nhk->nhv", state, q[:, t])
        real = lens > 0                                          # padded rows leave the scratch slot alone
        self.rec[gi, slots[real]] = state[real]
        out = self.w.gated_norm(lay, out, z).reshape(nb, lb, H * D)
        return F.linear(out, lay["out_proj"])

    def _attention(self, lay, x, ai, slots, pos, valid, cos, sin, ring_col):
        cfg, W = self.cfg, self.window
        nb, lb, _ = x.shape
        hq, hkv, d = cfg.attn_heads, cfg.kv_heads, cfg.attn_head_dim
        qg = F.linear(x, lay["q_proj"]).view(nb, lb, hq, 2 * d)
        query, gate = qg[..., :d], qg[..., d:].reshape(nb, lb, hq * d)
        query = rms_norm(query, lay["q_norm"], cfg.rms_eps)
        key = rms_norm(F.linear(x, lay["k_proj"]).view(nb, lb, hkv, d), lay["k_norm"], cfg.rms_eps)
        value = F.linear(x, lay["v_proj"]).view(nb, lb, hkv, d)
        rot = cfg.rotary_dim
        query = rope(query, cos[:, :, None], sin[:, :, None], rot)
        key = rope(key, cos[:, :, None], sin[:, :, None], rot)
        keys = torch.cat([self.ring_k[ai, slots, :, :W], key.transpose(1, 2)], 2)      # [nb, hkv, W+lb, d]
        values = torch.cat([self.ring_v[ai, slots, :, :W], value.transpose(1, 2)], 2)
        kpos = torch.cat([self.ring_pos[slots, :W], torch.where(valid, pos, torch.full_like(pos, -1))], 1)
        qq, kk = pos[:, :, None], kpos[:, None, :]
        allowed = (kk >= 0) & (kk <= qq) & (kk > qq - W) & valid[:, :, None]             # [nb, lb, W+lb]
        group = hq // hkv
        qh = query.permute(0, 2, 1, 3)                                                   # [nb, hq, lb, d]
        kh = keys.repeat_interleave(group, 1)
        vh = values.repeat_interleave(group, 1)
        scores = torch.matmul(qh, kh.transpose(-1, -2)) * d ** -0.5
        scores = scores.masked_fill(~allowed[:, None], float("-inf"))
        probs = torch.softmax(scores, -1).nan_to_num(0.0)
        out = torch.matmul(probs, vh).permute(0, 2, 1, 3).reshape(nb, lb, hq * d)
        self.ring_k[ai, slots[:, None], :, ring_col] = key
        self.ring_v[ai, slots[:, None], :, ring_col] = value
        return F.linear(out * torch.sigmoid(gate), lay["o_proj"])

    # ---- host loop -------------------------------------------------------------------------------------------
    def run_arrays(self, chunks, slots):
        """One tick of <= largest-bucket rows, <= 64 tokens each: pack, run, advance lengths."""
        n = len(chunks)
        nb = bucket(n, self.buckets)
        lb = bucket(max(len(c) for c in chunks), TOKEN_BUCKETS)
        buf = np.zeros(nb * lb + 3 * nb, dtype=np.int64)
        lens = pack_inputs(chunks, slots, nb, lb, self.length, self.max_slots, buf)
        o = nb * lb
        t = torch.from_numpy(buf)
        probs = self.tick(t[:o].view(nb, lb), t[o:o + nb], t[o + nb:o + 2 * nb], t[o + 2 * nb:])
        self.length[np.asarray(slots, dtype=np.int64)] += lens
        return probs[:, :n].numpy(), lens

    def step(self, requests):
        """requests [(slot, ids)], unique slots -> {role: [np [L_i, 3]]} (reference slot_engine_v7.py:147-167)."""
        if len({s for s, _ in requests}) != len(requests):
            raise ValueError("a session may appear once per tick")
        largest, rows = TOKEN_BUCKETS[-1], self.buckets[-1]
        res = {role: [[] for _ in requests] for role in self.cfg.roles}
        pending = [(i, s, list(ids)) for i, (s, ids) in enumerate(requests)]
        while pending:
            batch = [(i, s, ids[:largest]) for i, s, ids in pending]
            for start in range(0, len(batch), rows):
                part = batch[start:start + rows]
                probs, lens = self.run_arrays([c for _, _, c in part], [s for _, s, _ in part])
                for r, role in enumerate(self.cfg.roles):
                    for row, (i, _, _) in enumerate(part):
                        res[role][i].append(probs[r, row, :lens[row]])
            pending = [(i, s, ids[largest:]) for i, s, ids in pending if len(ids) > largest]
        return {role: [np.concatenate(c) for c in rows_] for role, rows_ in res.items()}


@torch.no_grad()
def score_complete(sd, cfg, ids, window=512, w=None):
    """Per-token probs [roles, T, 3] of one complete message (reference runtime.py:136-145, all positions)."""
    w = w or Weights(sd, cfg)
    ids = torch.as_tensor(ids, dtype=torch.int64)
    T = ids.shape[0]
    pos = torch.arange(T)
    hidden = w.embed[ids].float()
    cos, sin = w.cos_sin(pos)
    causal = (pos[None] <= pos[:, None]) & (pos[None] > pos[:, None] - window)
    for lay in w.layers:
        x = rms_norm(hidden, lay["norm_in"], cfg.rms_eps)
        if lay["kind"] == "linear_attention":
            H, D, kd = cfg.gdn_heads, cfg.gdn_head_dim, cfg.key_dim
            qkv = F.linear(x, lay["in_proj_qkv"])
            z = F.linear(x, lay["in_proj_z"]).reshape(T, H, D)
            b, a = F.linear(x, lay["in_proj_b"]), F.linear(x, lay["in_proj_a"])
            ext = torch.cat([torch.zeros(cfg.conv_kernel - 1, cfg.conv_dim), qkv], 0)
            conv = sum(lay["conv_w"][:, j] * ext[j:j + T] for j in range(cfg.conv_kernel))
            conv = F.silu(conv)
            q = l2norm(conv[:, :kd].reshape(T, H, D)) * D ** -0.5
            k = l2norm(conv[:, kd:2 * kd].reshape(T, H, D))
            v = conv[:, 2 * kd:].reshape(T, H, D)
            beta, g = torch.sigmoid(b), gdn_decay(a, lay["A_log"], lay["dt_bias"])
            out = gdn_chunked(q, k, v, g, beta, torch.zeros(H, D, D))
            mixed = F.linear(w.gated_norm(lay, out, z).reshape(T, H * D), lay["out_proj"])
        else:
            hq, hkv, d = cfg.attn_heads, cfg.kv_heads, cfg.attn_head_dim
            qg = F.linear(x, lay["q_proj"]).view(T, hq, 2 * d)
            query, gate = qg[..., :d], qg[..., d:].reshape(T, hq * d)
            query = rope(rms_norm(query, lay["q_norm"], cfg.rms_eps), cos[:, None], sin[:, None], cfg.rotary_dim)
            key = rms_norm(F.linear(x, lay["k_proj"]).view(T, hkv, d), lay["k_norm"], cfg.rms_eps)
            key = rope(key, cos[:, None], sin[:, None], cfg.rotary_dim)
            value = F.linear(x, lay["v_proj"]).view(T, hkv, d)
            group = hq // hkv
            kh = key.repeat_interleave(group, 1).transpose(0, 1)                 # [hq, T, d]
            vh = value.repeat_interleave(group, 1).transpose(0, 1)
            scores = torch.matmul(query.transpose(0, 1), kh.transpose(-1, -2)) * d ** -0.5
            scores = scores.masked_fill(~causal[None], float("-inf"))
            out = torch.matmul(torch.softmax(scores, -1), vh).transpose(0, 1).reshape(T, hq * d)
            mixed = F.linear(out * torch.sigmoid(gate), lay["o_proj"])
        hidden = hidden + mixed
        hidden = hidden + w.mlp(lay, rms_norm(hidden, lay["norm_post"], cfg.rms_eps))
    hidden = rms_norm(hidden, w.final_norm, cfg.rms_eps)
    return torch.stack([torch.softmax(w.readout(hidden, role), -1) for role in cfg.roles])
