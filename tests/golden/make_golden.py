"""Generate the golden vectors in tests/golden/golden.npz by running the REFERENCE implementation on the CPU.

Run once in a container that has the reference checkout (its root directory in $HSG_REFERENCE):

    HSG_REFERENCE=<reference checkout> python tests/golden/make_golden.py

What it runs (all fp32 on bf16-valued random-init weights from hs_guard_b200.weights, seed 0):
- ``pack_inputs`` from the reference (src/hs_guard/engine/slot_engine_v7.py:7-25) on fixed cases;
- transformers' ``torch_recurrent_gated_delta_rule`` (the recurrent rule the reference's pure-torch slot engine calls,
  engine/bucketed_engine.py:109-111) on seeded q/k/v/g/beta;
- ``ring_attention_reference`` (engine/ring_attention_kernel.py:7-26) on seeded rings with wrap-around;
- the reference's own slot engine (``BucketedStreamEngine``, engine/bucketed_engine.py) with its pools on the CPU, driven
  through a fixed multi-slot script (multi-token ticks, padding rows, ring wrap past 512 tokens, single-token ticks);
- the reference's complete-message forward (runtime.py:136-145 with window_attention.py) on slot 0's whole stream.
Inputs that are large are regenerated from seeds by ``golden_inputs.py`` on both sides; the fixture keeps outputs,
summaries of the state pools and a weight digest so a test host can confirm it regenerated the same weights.
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, HERE)
REF = os.environ.get("HSG_REFERENCE")
if not REF:
    raise SystemExit("set HSG_REFERENCE to the root of the reference checkout")
sys.path.insert(0, os.path.join(REF, "src"))

from golden_inputs import (STREAM_MAX_SLOTS, gdn_inputs, ring_inputs, sample_index, stream_script)  # noqa: E402
from hs_guard_b200 import DEFAULT  # noqa: E402
from hs_guard_b200 import weights as W  # noqa: E402


def reference_model(sd):
    """The reference Classifier (runtime._build over transformers' Qwen3_5TextModel) loaded with ``sd``, fp32, CPU."""
    import transformers.models.qwen3_5.modeling_qwen3_5 as tfm
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    from hs_guard import runtime, window_attention

    # transformers 5.5 expects a single mask where the reference (written for 5.17) passes a per-layer-type dict
    # (window_attention.py:255-259); both entries are None or the same 2-D mask for unpadded input.
    if not getattr(tfm, "_hsg_mask_shim", False):
        orig_ccm, orig_upd = tfm.create_causal_mask, tfm.Qwen3_5TextModel._update_linear_attn_mask

        def ccm(*a, **k):
            if isinstance(k.get("attention_mask"), dict):
                k["attention_mask"] = k["attention_mask"]["full_attention"]
            return orig_ccm(*a, **k)

        def upd(self, attention_mask, *a, **k):
            if isinstance(attention_mask, dict):
                attention_mask = attention_mask["linear_attention"]
            return orig_upd(self, attention_mask, *a, **k)
        tfm.create_causal_mask, tfm.Qwen3_5TextModel._update_linear_attn_mask = ccm, upd
        tfm._hsg_mask_shim = True
    cfg = Qwen3_5TextConfig(**DEFAULT.hf_kwargs())
    cfg._attn_implementation = "sdpa"
    backbone = tfm.Qwen3_5TextModel(cfg)
    window_attention.set_window(backbone, 512)
    clf = runtime._build(backbone)
    clf.load_state_dict(sd, strict=True)
    return clf.float().eval()


def reference_stream_engine(clf, max_slots):
    """BucketedStreamEngine with its pools on the CPU and transformers' torch recurrent GDN rule; its tick, GDN and
    attention code (bucketed_engine.py:58-201) run unchanged."""
    import transformers.models.qwen3_5.modeling_qwen3_5 as tfm
    from hs_guard.engine.bucketed_engine import BucketedStreamEngine

    class CpuEngine(BucketedStreamEngine):
        def __init__(self, model):
            self.rope = tfm.apply_rotary_pos_emb
            self.model, self.backbone = model, model.backbone
            cfg = self.backbone.config
            self.layers = list(self.backbone.layers[:cfg.num_hidden_layers])
            types = list(cfg.layer_types[:cfg.num_hidden_layers])
            self.kind = [(t, sum(1 for u in types[:i] if u == t)) for i, t in enumerate(types)]
            self.kernel = tfm.torch_recurrent_gated_delta_rule
            self.window, self.max_slots, self.roles, self.use_graphs = 512, max_slots, ("user", "assistant"), False
            gdn = next(layer.linear_attn for layer in self.layers if hasattr(layer, "linear_attn"))
            att = next(layer.self_attn for layer in self.layers if hasattr(layer, "self_attn"))
            n_gdn, n_att = types.count("linear_attention"), types.count("full_attention")
            slots = max_slots + 1
            self.rec = torch.zeros(n_gdn, slots, gdn.num_v_heads, gdn.head_k_dim, gdn.head_v_dim)
            self.conv = torch.zeros(n_gdn, slots, gdn.conv_kernel_size - 1, gdn.conv_dim)
            self.ring_k = torch.zeros(n_att, slots, 513, cfg.num_key_value_heads, att.head_dim)
            self.ring_v = torch.zeros_like(self.ring_k)
            self.ring_pos = torch.full((slots, 513), -1, dtype=torch.long)
            self.length = [0] * max_slots
            self.graphs, self.pool = {}, None
            self.stats = {"graph_replays": 0, "eager_steps": 0, "captures": 0}
            b = tuple(x for x in (1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 160, 192, 224, 256, 320, 352, 384, 448, 512)
                      if x <= max_slots)
            self.session_buckets = b if b and b[-1] == max_slots else b + (max_slots,)

        def _static(self, nb, lb):
            key = (nb, lb)
            if key not in self.graphs:
                static = {"ids": torch.zeros(nb, lb, dtype=torch.long), "lens": torch.zeros(nb, dtype=torch.long),
                          "slots": torch.full((nb,), self.max_slots, dtype=torch.long),
                          "starts": torch.zeros(nb, dtype=torch.long)}
                self.graphs[key] = (None, static)
            return self.graphs[key]

    return CpuEngine(clf)


def main():
    out = {}
    t0 = time.time()
    # ---- pack_inputs -------------------------------------------------------------------------------------------
    from hs_guard.engine.slot_engine_v7 import pack_inputs
    cases = [([[4, 5, 6]], [0], 2, 4, [7], 1),
             ([[1], [2], [3]], [2, 0, 1], 4, 1, [5, 0, 9], 3),
             ([[10, 11], [12, 13, 14, 15, 16], [17]], [1, 3, 0], 4, 8, [100, 3, 0, 511], 4)]
    for i, (chunks, slots, nb, lb, length, max_slots) in enumerate(cases):
        buf = np.full(nb * lb + 3 * nb, -7, dtype=np.int64)
        lens = pack_inputs(chunks, np.asarray(slots, dtype=np.int64), nb, lb, np.asarray(length, dtype=np.int64),
                           max_slots, buf)
        out[f"pack{i}_out"], out[f"pack{i}_lens"] = buf, lens

    # ---- GDN recurrent rule ------------------------------------------------------------------------------------
    import transformers.models.qwen3_5.modeling_qwen3_5 as tfm
    for name, case in (("gdn_a", dict(n=3, L=5, seed=21)), ("gdn_b", dict(n=2, L=1, seed=22))):
        q, k, v, g, beta, state = gdn_inputs(**case)
        o, final = tfm.torch_recurrent_gated_delta_rule(q, k, v, g, beta, initial_state=state.clone(),
                                                        output_final_state=True, use_qk_l2norm_in_kernel=True)
        out[name + "_o"] = o.numpy()
        out[name + "_state_norm"] = final.pow(2).sum((-1, -2)).sqrt().numpy()
        out[name + "_state_sample"] = final.reshape(-1)[torch.from_numpy(sample_index(final.numel(), 4))].numpy()

    # ---- ring attention contract -------------------------------------------------------------------------------
    from hs_guard.engine.ring_attention_kernel import ring_attention_reference
    for name, lb in (("ring_a", 1), ("ring_b", 3)):
        args = ring_inputs(lb=lb, seed=31 + lb)
        o = ring_attention_reference(*args, scale=256 ** -0.5, window=512)
        out[name + "_o"] = o.numpy()

    # ---- whole model ----------------------------------------------------------------------------------------------
    sd = W.random_state_dict(0)
    out["weights_digest"] = np.array(W.state_dict_digest(sd))
    clf = reference_model(sd)
    eng = reference_stream_engine(clf, STREAM_MAX_SLOTS)
    script = stream_script()
    probs_u, probs_a = [], []
    with torch.inference_mode():
        for tick in script:
            res = eng.step(tick)
            for i in range(len(tick)):
                probs_u.append(res["user"][i].numpy())
                probs_a.append(res["assistant"][i].numpy())
    out["stream_probs_user"] = np.concatenate(probs_u)
    out["stream_probs_assistant"] = np.concatenate(probs_a)
    out["stream_length"] = np.asarray(eng.length, dtype=np.int64)
    out["stream_ring_pos"] = eng.ring_pos.numpy()
    real = slice(0, STREAM_MAX_SLOTS)
    rec = eng.rec[:, real]
    out["stream_rec_norm"] = rec.pow(2).sum((-1, -2)).sqrt().numpy()
    out["stream_rec_sample"] = rec.reshape(-1)[torch.from_numpy(sample_index(rec.numel(), 1))].numpy()
    conv = eng.conv[:, real]
    out["stream_conv_sample"] = conv.reshape(-1)[torch.from_numpy(sample_index(conv.numel(), 2))].numpy()
    ring_k = eng.ring_k[:, real].permute(0, 1, 3, 2, 4)          # -> [layer, slot, head, col, dim]
    out["stream_ringk_sample"] = ring_k.reshape(-1)[torch.from_numpy(sample_index(ring_k.numel(), 3))].numpy()
    # complete-message forward over slot 0's whole stream
    ids0 = [t for tick in script for s, ids in tick if s == 0 for t in ids]
    with torch.inference_mode():
        x = torch.tensor([ids0])
        hidden = clf(x, attention_mask=torch.ones_like(x), use_cache=False).last_hidden_state[0]
        cm = torch.stack([clf.readout(hidden, role)[0].float().softmax(-1) for role in ("user", "assistant")])
    out["cm_slot0_probs"] = cm.numpy()
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    print(f"wrote golden.npz in {time.time() - t0:.1f}s; stream tokens {len(out['stream_probs_user'])}")


if __name__ == "__main__":
    main()
