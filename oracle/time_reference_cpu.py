"""CPU baseline of configuration C1, measured with the REFERENCE's own code beside this repository's CPU port.

Test infrastructure, run by hand in a container that has the reference checkout (root directory in $HSG_REFERENCE);
the reference does not travel to the GPU host, so the benchmark there times the port and this script ties the two
together on one set of host cores:

    HSG_REFERENCE=<reference checkout> python oracle/time_reference_cpu.py [--threads N] [--tokens 256] [--reps 3]

C1: batch 1, one message of 256 uniform-random token ids (seed 1), random-init weights (seed 0), fp32 on the CPU.
The reference side is its complete-message forward (the Classifier of src/hs_guard/runtime.py:54-75 over
transformers' Qwen3_5TextModel with its window patch, window_attention.py:34-100; runtime.py:136-145 without the
tokenizer, which has no bundle here) plus the role readout and softmax; the port side is oracle.stream.score_complete.
Both are timed warm (one untimed call first) with torch.set_num_threads(N). Prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "tests", "golden"))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=os.cpu_count() or 1)
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    from make_golden import reference_model  # checks $HSG_REFERENCE and applies the transformers mask shim
    from hs_guard_b200 import DEFAULT
    from hs_guard_b200 import weights as W
    from oracle.stream import Weights, score_complete

    torch.set_num_threads(args.threads)
    sd = W.random_state_dict(0)
    ids = np.random.Generator(np.random.PCG64(1)).integers(0, DEFAULT.vocab, args.tokens)
    clf = reference_model(sd)
    x = torch.tensor([ids.tolist()])

    def reference():
        with torch.inference_mode():
            hidden = clf(x, attention_mask=torch.ones_like(x), use_cache=False).last_hidden_state[0]
            return torch.stack([clf.readout(hidden, role)[0].float().softmax(-1) for role in ("user", "assistant")])

    w = Weights(sd, DEFAULT)

    def port():
        return score_complete(sd, DEFAULT, ids, w=w)

    out = {"config": "C1: batch 1, one message of %d uniform-random ids (seed 1), random-init weights (seed 0), fp32"
                     % args.tokens, "threads": args.threads, "host_cpus": os.cpu_count()}
    results = {}
    for name, fn in (("reference", reference), ("port", port)):
        first = fn()
        t0 = time.perf_counter()
        for _ in range(args.reps):
            fn()
        dt = (time.perf_counter() - t0) / args.reps
        results[name] = first
        out[name] = {"ms_per_message": dt * 1e3, "tokens_per_s": args.tokens / dt}
    out["port_over_reference_time"] = out["port"]["ms_per_message"] / out["reference"]["ms_per_message"]
    out["max_abs_dp"] = float((results["reference"] - results["port"]).abs().max())
    print(json.dumps(out))


if __name__ == "__main__":
    main()
