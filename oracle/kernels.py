"""Kernel-level CPU oracles (fp32 torch). Test infrastructure only; see ``oracle/__init__.py``."""
from __future__ import annotations

import torch
import torch.nn.functional as F


def l2norm(x, eps=1e-6):
    """x / sqrt(sum(x^2) + eps) over the last dim (transformers' ``l2norm``, FLA's in-kernel q/k norm)."""
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def gdn_decay(a, A_log, dt_bias):
    """g = -exp(A_log) * softplus(a + dt_bias) with softplus threshold 20 (reference fused_kernels.py:172-173)."""
    x = a.float() + dt_bias.float()
    sp = torch.where(x > 20.0, x, torch.log1p(torch.exp(torch.clamp(x, max=20.0))))
    return -torch.exp(A_log.float()) * sp


def gdn_slot_step(packed, a, b, A_log, dt_bias, state, slots, lens, heads=16, head_dim=128):
    """Gated delta rule over one tick, per (row, head), as reference engine/fused_kernels.py:140-211.

    packed [N, L, 3*heads*head_dim]: q at 0, k at heads*head_dim, v at 2*heads*head_dim (post conv+silu);
    a, b [N, L, heads] raw projections; state [S, heads, dk, dv] fp32, updated in place at ``slots[n]`` for rows
    with ``lens[n] > 0``. Returns o [N, L, heads, dv] fp32 with zeros at padded positions.
    """
    n, L, _ = packed.shape
    kd = heads * head_dim
    q = packed[..., :kd].float().reshape(n, L, heads, head_dim)
    k = packed[..., kd:2 * kd].float().reshape(n, L, heads, head_dim)
    v = packed[..., 2 * kd:3 * kd].float().reshape(n, L, heads, head_dim)
    q = l2norm(q) * head_dim ** -0.5
    k = l2norm(k)
    g = gdn_decay(a, A_log, dt_bias)            # [N, L, H]
    beta = torch.sigmoid(b.float())
    o = torch.zeros(n, L, heads, head_dim)
    for row in range(n):
        length = int(lens[row])
        if length <= 0:
            continue
        s = int(slots[row])
        h = state[s].clone()                    # [H, dk, dv]
        for t in range(length):
            h = h * torch.exp(g[row, t])[:, None, None]
            kv = torch.einsum("hkv,hk->hv", h, k[row, t])
            delta = beta[row, t][:, None] * (v[row, t] - kv)
            h = h + k[row, t][:, :, None] * delta[:, None, :]
            o[row, t] = torch.einsum("hkv,hk->hv", h, q[row, t])
        state[s] = h
    return o


def gdn_chunked(q, k, v, g, beta, state, chunk=64):
    """The gated delta rule over one sequence in its chunked (WY) form: the published algorithm behind FLA's
    ``chunk_gated_delta_rule`` (chunk.py:29-114) and transformers' ``torch_chunk_gated_delta_rule``, which the
    reference's complete-message path runs (runtime.py:78-89). Same result as the token-by-token recurrence.

    q, k, v [T, H, D] (q, k already L2-normalised, q scaled), g, beta [T, H] (log decay <= 0, write strength),
    state [H, D, D] (updated in place). Per chunk of C tokens with cumulative log decay gam (within the chunk):
      A[t, s] = beta_t e^(gam_t - gam_s) k_t . k_s (s < t),   T = (I + A)^-1 (unit lower triangular solve),
      Delta = T (beta v) - T (beta e^gam k) S,   O = (e^gam q) S + ([s <= t] e^(gam_t - gam_s) q_t . k_s) Delta,
      S <- e^(gam_C) S + (e^(gam_C - gam) k)^T Delta.
    Every exponent is <= 0. Returns o [T, H, D]."""
    T, H, D = q.shape
    out = torch.empty(T, H, D)
    for c0 in range(0, T, chunk):
        c1 = min(c0 + chunk, T)
        n = c1 - c0
        qc, kc, vc = (x[c0:c1].transpose(0, 1).float() for x in (q, k, v))       # [H, n, D]
        gam = torch.cumsum(g[c0:c1].t().float(), -1)                             # [H, n]
        bc = beta[c0:c1].t().float()
        diff = gam[:, :, None] - gam[:, None, :]
        lower = torch.ones(n, n, dtype=torch.bool).tril()
        decay = torch.where(lower, torch.exp(torch.where(lower, diff, torch.zeros_like(diff))), torch.zeros_like(diff))
        a = (bc[:, :, None] * (kc @ kc.transpose(-1, -2)) * decay).tril(-1)
        eye = torch.eye(n).expand(H, n, n)
        u = torch.linalg.solve_triangular(eye + a, bc[..., None] * vc, upper=False, unitriangular=True)
        w = torch.linalg.solve_triangular(eye + a, (bc * torch.exp(gam))[..., None] * kc, upper=False,
                                          unitriangular=True)
        delta = u - w @ state
        o = (qc * torch.exp(gam)[..., None]) @ state + ((qc @ kc.transpose(-1, -2)) * decay) @ delta
        last = gam[:, -1:]
        state.mul_(torch.exp(last)[..., None]).add_((kc * torch.exp(last - gam)[..., None]).transpose(-1, -2) @ delta)
        out[c0:c1] = o.transpose(0, 1)
    return out


def causal_conv_step(qkv, pool, weight, slots, lens):
    """silu(causal depthwise conv, kernel K) over [K-1 saved rows | L new rows], then roll the history of rows
    with ``lens > 0`` (reference fused_kernels.py:94-136 without its bf16 roundings; bucketed_engine.py:94-98).

    qkv [N, L, C]; pool [S, K-1, C] (updated in place); weight [C, K]. Returns [N, L, C] fp32."""
    n, L, c = qkv.shape
    keep = weight.shape[1] - 1
    ext = torch.cat([pool[slots.long()].float(), qkv.float()], 1)          # [N, keep+L, C]
    out = torch.zeros(n, L, c)
    for j in range(keep + 1):
        out += weight[:, j].float() * ext[:, j:j + L]
    for row in range(n):
        length = int(lens[row])
        if length > 0:
            pool[int(slots[row])] = ext[row, length:length + keep].to(pool.dtype)
    return F.silu(out)


def ring_attention(q, ring_k, ring_v, new_k, new_v, ring_pos, slots, starts, lens, scale, window):
    """Windowed GQA over a slot's ring plus this tick's keys (reference engine/ring_attention_kernel.py:7-26).

    q [N, Hkv, G*Lb, D] (row r is query group r // Lb, token r % Lb); ring_k/v [S, Hkv, W+1, D];
    new_k/v [N, Hkv, Lb, D]; ring_pos [S, W+1]. Key j is visible to query position p iff
    0 <= kpos <= p and kpos > p - W. Rows with no visible key (padded tokens) are 0. Returns fp32 [N, Hkv, G*Lb, D].
    """
    n, hkv, m, d = q.shape
    lb = new_k.shape[2]
    slots, starts, lens = slots.long(), starts.long(), lens.long()
    rows = torch.arange(m)
    l_idx = rows % lb
    qpos = starts[:, None] + l_idx[None]
    q_valid = l_idx[None] < lens[:, None]
    steps = torch.arange(lb)
    new_pos = torch.where(steps[None] < lens[:, None], starts[:, None] + steps[None], torch.full((n, lb), -1))
    kpos = torch.cat([ring_pos[slots, :window], new_pos], 1)
    ok = (kpos[:, None] >= 0) & (kpos[:, None] <= qpos[..., None]) & (kpos[:, None] > qpos[..., None] - window)
    ok = ok & q_valid[..., None]
    keys = torch.cat([ring_k[slots, :, :window].float(), new_k.float()], 2)
    values = torch.cat([ring_v[slots, :, :window].float(), new_v.float()], 2)
    scores = torch.matmul(q.float(), keys.transpose(-1, -2)) * scale
    scores = scores.masked_fill(~ok[:, None], float("-inf"))
    probs = torch.softmax(scores, -1).nan_to_num(0.0)
    return torch.matmul(probs, values)
