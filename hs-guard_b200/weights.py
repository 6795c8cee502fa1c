"""Weight bundles: deterministic random-init weights and the engine's device layout.

HS-Guard's released weights live on the Hugging Face Hub only (reference ``src/hs_guard/runtime.py:8``),
so benchmarks and parity tests use a seeded random initialisation of the same architecture. Every
tensor is drawn from its own numpy PCG64 stream, keyed by (seed, parameter index), so any process on
any host regenerates identical bits without shipping 1.5 GB of weights. Backbone tensors are bf16,
as ``load_model`` casts them (reference ``runtime.py:114-116``); head tensors are fp32 holding
bf16-representable values, so the complete-message readout (fp32, ``runtime.py:71-74``) and the
streaming engine's bf16 head copies (``engine/slot_engine_v7.py:44-51``) see the same numbers.

Names follow the reference ``Classifier`` state dict (``runtime.py:54-75`` wrapping transformers'
``Qwen3_5TextModel``), so a bundle loads into the reference model with ``load_state_dict(strict=True)``.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from .config import DEFAULT, HsgConfig

_CATEGORIES = {"user": 9, "assistant": 8}


def parameter_specs(cfg: HsgConfig = DEFAULT):
    """[(name, shape, init)] in a fixed order; init = (kind, a, b): ('normal', mean, std) or ('uniform', lo, hi)
    or ('log_uniform', lo, hi) (A_log = log(U(lo, hi)), as transformers' GDN initialiser)."""
    h, f = cfg.hidden, cfg.intermediate
    specs = [("backbone.embed_tokens.weight", (cfg.vocab, h), ("normal", 0.0, 0.02))]
    for i, kind in enumerate(cfg.layer_types):
        p = f"backbone.layers.{i}."
        if kind == "linear_attention":
            a = p + "linear_attn."
            specs += [(a + "dt_bias", (cfg.gdn_heads,), ("normal", 1.0, 0.2)),
                      (a + "A_log", (cfg.gdn_heads,), ("log_uniform", 1.0, 16.0)),
                      (a + "conv1d.weight", (cfg.conv_dim, 1, cfg.conv_kernel), ("uniform", -0.5, 0.5)),
                      (a + "norm.weight", (cfg.gdn_head_dim,), ("normal", 1.0, 0.1)),
                      (a + "out_proj.weight", (h, cfg.key_dim), ("normal", 0.0, 0.02)),
                      (a + "in_proj_qkv.weight", (cfg.conv_dim, h), ("normal", 0.0, 0.02)),
                      (a + "in_proj_z.weight", (cfg.key_dim, h), ("normal", 0.0, 0.02)),
                      (a + "in_proj_b.weight", (cfg.gdn_heads, h), ("normal", 0.0, 0.02)),
                      (a + "in_proj_a.weight", (cfg.gdn_heads, h), ("normal", 0.0, 0.02))]
        else:
            a = p + "self_attn."
            d = cfg.attn_head_dim
            specs += [(a + "q_proj.weight", (2 * cfg.attn_heads * d, h), ("normal", 0.0, 0.02)),
                      (a + "k_proj.weight", (cfg.kv_heads * d, h), ("normal", 0.0, 0.02)),
                      (a + "v_proj.weight", (cfg.kv_heads * d, h), ("normal", 0.0, 0.02)),
                      (a + "o_proj.weight", (h, cfg.attn_heads * d), ("normal", 0.0, 0.02)),
                      (a + "q_norm.weight", (d,), ("normal", 0.0, 0.1)),
                      (a + "k_norm.weight", (d,), ("normal", 0.0, 0.1))]
        specs += [(p + "mlp.gate_proj.weight", (f, h), ("normal", 0.0, 0.02)),
                  (p + "mlp.up_proj.weight", (f, h), ("normal", 0.0, 0.02)),
                  (p + "mlp.down_proj.weight", (h, f), ("normal", 0.0, 0.02)),
                  (p + "input_layernorm.weight", (h,), ("normal", 0.0, 0.1)),
                  (p + "post_attention_layernorm.weight", (h,), ("normal", 0.0, 0.1))]
    specs.append(("backbone.norm.weight", (h,), ("normal", 0.0, 0.1)))
    e = cfg.head_hidden
    for role in cfg.roles:
        for proj, risk, cat in (("projection", "risk", "category"),
                                ("general_projection", "general", "general_category")):
            q = f"heads.{role}."
            specs += [(q + proj + ".0.weight", (e, h), ("normal", 0.0, 0.02)),
                      (q + proj + ".0.bias", (e,), ("normal", 0.0, 0.02)),
                      (q + proj + ".1.weight", (e,), ("normal", 1.0, 0.1)),
                      (q + proj + ".1.bias", (e,), ("normal", 0.0, 0.1)),
                      (q + risk + ".weight", (cfg.n_classes, e), ("normal", 0.0, 0.1)),
                      (q + risk + ".bias", (cfg.n_classes,), ("normal", 0.0, 0.1)),
                      (q + cat + ".weight", (_CATEGORIES[role], e), ("normal", 0.0, 0.1)),
                      (q + cat + ".bias", (_CATEGORIES[role],), ("normal", 0.0, 0.1))]
    return specs


def _draw(index, shape, init, seed):
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, index])))
    n = int(np.prod(shape))
    kind, a, b = init
    if kind == "normal":
        x = rng.standard_normal(n, dtype=np.float32)
        x *= np.float32(b)
        x += np.float32(a)
    elif kind == "uniform":
        x = rng.random(n, dtype=np.float32) * np.float32(b - a) + np.float32(a)
    elif kind == "log_uniform":
        x = np.log(rng.random(n, dtype=np.float32) * np.float32(b - a) + np.float32(a))
    else:
        raise ValueError(kind)
    # Round to bf16 so every consumer sees identical values whatever dtype it stores.
    return torch.from_numpy(x.reshape(shape)).to(torch.bfloat16)


def random_state_dict(seed: int = 0, cfg: HsgConfig = DEFAULT, names=None):
    """Deterministic random-init weights keyed by reference parameter name. Backbone tensors are bf16;
    head tensors fp32 (bf16-representable). ``names``: optional subset to generate."""
    out = {}
    for index, (name, shape, init) in enumerate(parameter_specs(cfg)):
        if names is not None and name not in names:
            continue
        t = _draw(index, shape, init, seed)
        out[name] = t.float() if name.startswith("heads.") else t
    return out


def state_dict_digest(sd):
    """sha256 over names, shapes and raw bytes: pins that two hosts generated the same weights."""
    h = hashlib.sha256()
    for name in sorted(sd):
        t = sd[name].detach().cpu().contiguous()
        h.update(name.encode())
        h.update(str(tuple(t.shape)).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16
                 else t.view(torch.int16).numpy().tobytes())
    return h.hexdigest()


class RandomInitModel:
    """A stand-in for the reference ``Classifier`` when no checkpoint is present: it carries a config and a
    state dict with the reference's parameter names. ``StreamingGuard`` accepts either."""

    def __init__(self, seed: int = 0, cfg: HsgConfig = DEFAULT):
        self.cfg, self.seed = cfg, seed
        self._sd = None

    def state_dict(self):
        if self._sd is None:
            self._sd = random_state_dict(self.seed, self.cfg)
        return self._sd


def extract_state_dict(model, head="redline"):
    """(HsgConfig, state dict) from a reference ``Classifier`` (``.backbone`` + ``.heads``), a RandomInitModel or
    loaded bundle (``.cfg`` + ``.state_dict()``), or a plain dict. ``head='general'`` maps the general heads onto the redline names
    (the swap ``load_model`` performs, reference runtime.py:120-122)."""
    if head not in ("redline", "general"):
        raise ValueError("head must be redline or general")
    if isinstance(model, dict):
        cfg, sd = DEFAULT, model
    elif isinstance(getattr(model, "cfg", None), HsgConfig) and callable(getattr(model, "state_dict", None)):
        cfg, sd = model.cfg, model.state_dict()  # RandomInitModel, bundle.BundleModel
    elif hasattr(model, "backbone") and hasattr(model, "heads"):
        cfg = HsgConfig.from_hf(model.backbone.config)
        sd = {"backbone." + k: v for k, v in model.backbone.state_dict().items()}
        for role in cfg.roles:
            h = model.heads[role]
            for part in ("projection", "risk", "general_projection", "general"):
                if part in h:
                    for k, v in h[part].state_dict().items():
                        sd[f"heads.{role}.{part}.{k}"] = v
    else:
        raise TypeError("model must expose .backbone and .heads, or be a RandomInitModel or a state dict")
    if head == "general":
        sd = dict(sd)
        for role in cfg.roles:
            for suffix in ("0.weight", "0.bias", "1.weight", "1.bias"):
                sd[f"heads.{role}.projection.{suffix}"] = sd[f"heads.{role}.general_projection.{suffix}"]
            for suffix in ("weight", "bias"):
                sd[f"heads.{role}.risk.{suffix}"] = sd[f"heads.{role}.general.{suffix}"]
    return cfg, sd


def rope_inv_freq(cfg: HsgConfig = DEFAULT):
    """fp32 inverse frequencies exactly as transformers computes them (compute_default_rope_parameters)."""
    dim = cfg.rotary_dim
    return 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim))


def engine_layout(sd, cfg: HsgConfig = DEFAULT, device="cuda"):
    """Rearrange reference-named weights into the device layout the CUDA engine reads.

    - GDN layer ``w_in``: rows [in_proj_qkv | in_proj_z | in_proj_b | in_proj_a | zero pad] (bf16, K-major),
      one GEMM per layer for the four projections of reference engine/slot_engine_v8.py:230-232.
    - attention layer ``w_in``: rows [q_proj (query|gate per head) | k_proj | v_proj].
    - ``w_gu``: gate_proj and up_proj interleaved row by row (row 2f = gate f, row 2f+1 = up f), so one 128-row
      GEMM tile holds both halves of silu(g)*u for 64 features, each pair in adjacent accumulator lanes.
    - RMSNorm weights are stored as ``1 + w`` in fp32 (Qwen3_5RMSNorm), the gated norm as ``w``.
    - heads: ``head_w1`` [roles*512, 1024] bf16, LayerNorm and the 512->3 readout in fp32.
    """
    bf, f32 = torch.bfloat16, torch.float32

    def g(name, dtype=None):
        t = sd[name]
        return t.to(device=device, dtype=dtype or t.dtype).contiguous()

    out = {"embed": g("backbone.embed_tokens.weight", bf),
           "final_norm": (1.0 + g("backbone.norm.weight", f32)).contiguous(),
           "inv_freq": rope_inv_freq(cfg).to(device), "layers": []}
    for i, kind in enumerate(cfg.layer_types):
        p = f"backbone.layers.{i}."
        lay = {"kind": kind}
        if kind == "linear_attention":
            a = p + "linear_attn."
            w = torch.cat([g(a + "in_proj_qkv.weight", bf), g(a + "in_proj_z.weight", bf),
                           g(a + "in_proj_b.weight", bf), g(a + "in_proj_a.weight", bf)], 0)
            pad = cfg.gdn_in_rows - w.shape[0]
            lay["w_in"] = torch.cat([w, torch.zeros(pad, cfg.hidden, dtype=bf, device=device)], 0).contiguous()
            lay["w_out"] = g(a + "out_proj.weight", bf)
            lay["conv_w"] = g(a + "conv1d.weight", f32).reshape(cfg.conv_dim, cfg.conv_kernel).contiguous()
            lay["A_log"] = g(a + "A_log", f32)
            lay["dt_bias"] = g(a + "dt_bias", f32)
            lay["gnorm_w"] = g(a + "norm.weight", f32)
        else:
            a = p + "self_attn."
            lay["w_in"] = torch.cat([g(a + "q_proj.weight", bf), g(a + "k_proj.weight", bf),
                                     g(a + "v_proj.weight", bf)], 0).contiguous()
            lay["w_out"] = g(a + "o_proj.weight", bf)
            lay["q_norm"] = (1.0 + g(a + "q_norm.weight", f32)).contiguous()
            lay["k_norm"] = (1.0 + g(a + "k_norm.weight", f32)).contiguous()
        gate, up = g(p + "mlp.gate_proj.weight", bf), g(p + "mlp.up_proj.weight", bf)
        lay["w_gu"] = torch.stack([gate, up], 1).reshape(2 * cfg.intermediate, cfg.hidden).contiguous()
        lay["w_down"] = g(p + "mlp.down_proj.weight", bf)
        lay["norm_in"] = (1.0 + g(p + "input_layernorm.weight", f32)).contiguous()
        lay["norm_post"] = (1.0 + g(p + "post_attention_layernorm.weight", f32)).contiguous()
        out["layers"].append(lay)
    w1, b1, lw, lb, w2, b2 = [], [], [], [], [], []
    for role in cfg.roles:
        q = f"heads.{role}."
        w1.append(g(q + "projection.0.weight", bf))
        b1.append(g(q + "projection.0.bias", f32))
        lw.append(g(q + "projection.1.weight", f32))
        lb.append(g(q + "projection.1.bias", f32))
        w2.append(g(q + "risk.weight", f32))
        b2.append(g(q + "risk.bias", f32))
    out.update(head_w1=torch.cat(w1).contiguous(), head_b1=torch.cat(b1).contiguous(),
               head_ln_w=torch.cat(lw).contiguous(), head_ln_b=torch.cat(lb).contiguous(),
               head_w2=torch.stack(w2).contiguous(), head_b2=torch.stack(b2).contiguous())
    return out
