"""Generate tests/golden/golden_long.npz: the REFERENCE implementation on the headline's context lengths.

Run once in a container that has the reference checkout (its root directory in $HSG_REFERENCE):

    HSG_REFERENCE=<reference checkout> python tests/golden/make_golden_long.py

It drives the reference's own slot engine (``BucketedStreamEngine``, engine/bucketed_engine.py:58-201, pools on the
CPU, transformers' torch recurrent rule; see make_golden.reference_stream_engine) through ``golden_inputs.long_script``:
four slots whose initial contexts are 8,000, 2,048, 512 and 1,000 uniform-random ids, sent as one request each (the
engine splits them into 64-token ticks, bucketed_engine.py:180-194), then 256 single-token ticks of every slot. It
then scores each slot's whole sequence with the reference's complete-message forward (runtime.py:136-145 with
window_attention.py:34-53). Stored: the streamed probabilities of both roles, the complete-message probabilities,
lengths and ring positions (bit-exact quantities), per-(layer, slot, head) recurrent-state norms and samples of the
recurrent, conv and ring pools, and the weight digest. Everything is fp32 on the bf16-valued seed-0 weights.
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from golden_inputs import LONG_CONTEXTS, long_script, sample_index  # noqa: E402
from make_golden import reference_model, reference_stream_engine  # noqa: E402  (checks $HSG_REFERENCE)
from hs_guard_b200 import weights as W  # noqa: E402


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.time()
    sd = W.random_state_dict(0)
    clf = reference_model(sd)
    n = len(LONG_CONTEXTS)
    eng = reference_stream_engine(clf, n)
    script = long_script()
    per_slot = {role: [[] for _ in range(n)] for role in ("user", "assistant")}
    with torch.inference_mode():
        for k, tick in enumerate(script):
            res = eng.step(tick)
            for role in per_slot:
                for (s, _), p in zip(tick, res[role]):
                    per_slot[role][s].append(p.numpy())
            if k == 0:
                print(f"prefill done in {time.time() - t0:.0f}s", flush=True)
    out = {"weights_digest": np.array(W.state_dict_digest(sd))}
    for role in per_slot:
        out[f"stream_probs_{role}"] = np.concatenate([np.concatenate(c) for c in per_slot[role]])
    out["stream_length"] = np.asarray(eng.length, dtype=np.int64)
    out["stream_ring_pos"] = eng.ring_pos.numpy()
    real = slice(0, n)
    rec = eng.rec[:, real]
    out["stream_rec_norm"] = rec.pow(2).sum((-1, -2)).sqrt().numpy()
    out["stream_rec_sample"] = rec.reshape(-1)[torch.from_numpy(sample_index(rec.numel(), 1))].numpy()
    conv = eng.conv[:, real]
    out["stream_conv_sample"] = conv.reshape(-1)[torch.from_numpy(sample_index(conv.numel(), 2))].numpy()
    ring_k = eng.ring_k[:, real].permute(0, 1, 3, 2, 4)  # -> [layer, slot, head, col, dim]
    out["stream_ringk_sample"] = ring_k.reshape(-1)[torch.from_numpy(sample_index(ring_k.numel(), 3))].numpy()
    print(f"stream done in {time.time() - t0:.0f}s", flush=True)
    # complete-message forward over each slot's whole sequence (context + single-token steps)
    cms = []
    with torch.inference_mode():
        for s in range(n):
            ids = [t for tick in script for slot, chunk in tick if slot == s for t in chunk]
            x = torch.tensor([ids])
            hidden = clf(x, attention_mask=torch.ones_like(x), use_cache=False).last_hidden_state[0]
            cms.append(torch.stack([clf.readout(hidden, role)[0].float().softmax(-1)
                                    for role in ("user", "assistant")]).numpy())
            print(f"complete message {s} ({len(ids)} ids) done at {time.time() - t0:.0f}s", flush=True)
    out["cm_probs"] = np.concatenate(cms, axis=1)  # [role, sum of lengths, 3], slots in order
    np.savez_compressed(os.path.join(HERE, "golden_long.npz"), **out)
    print(f"wrote golden_long.npz in {time.time() - t0:.0f}s; tokens {out['stream_probs_user'].shape[0]}")


if __name__ == "__main__":
    main()
