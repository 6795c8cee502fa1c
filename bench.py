"""Benchmark of the HS-Guard streaming step on B200 (workload C4 of the reference's headline metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Per GPU: 352 slots, each prefilled with 512, 2,048 or 8,000 uniform-random token ids (one third each, seed 4),
then single-token role=assistant steps (one token for every slot per step). One process per GPU (torchrun for
N > 1); each rank owns its own 352 slots and full weight replica, no collective on the data path ("weak" scaling).

Reported (rank 0, one JSON line):
- value: scored tokens/s of the whole job with the packed ticks already resident in HBM (graph replays timed with
  CUDA events, max over ranks); the per-tick working set (~10.8 GB) exceeds the 126 MB L2, so no flush is needed.
- e2e: the same metric through the public API (StreamingGuard.step with host lists: validation, packing, host->device
  copy, replay, device->host copy of the probabilities, 1 - p(safe)); latency_ms p50/P95 are of these steps.
- roofline: the dominant kernel (gated-delta-rule step) timed live with CUDA events in an eager tick.
- cpu_baseline: the CPU oracle port of the same step on this host's cores (bounded sample).
- complete_message: the reference's complete-message path (C1: one 256-id message) through MessageScorer on the GPU
  (batch 1 and 64) and through the CPU oracle port of the reference's forward on the host cores.
--impl reference times the CPU oracle port of the reference's step instead (the reference itself is Triton/CUDA-only
Python that is not shipped to the GPU host) and prints its own line.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "scored tokens/s/GPU at 352 slots; p50/P95 single-token step latency (ms)"
PUBLISHED_TOKENS_PER_S = 15075.6   # the reference's published minimum throughput, 1x L20, 352 streams
CONTEXTS = (512, 2048, 8000)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--slots", type=int, default=352)
    ap.add_argument("--contexts", default=",".join(map(str, CONTEXTS)))
    ap.add_argument("--cpu-slots", type=int, default=32)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="c4", choices=("c4", "c5", "c2", "c3"),
                    help="c4: single-token steps after prefill (the headline); c5: 64-token ticks with reassignment; "
                         "c2 / c3: the isolated gated-delta-rule step / ring-window decode of configs 2 and 3")
    ap.add_argument("--state-dtype", default="float16", choices=("float16", "float32"),
                    help="recurrent-state storage (float16 = the reference StreamingGuard's)")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def contexts_for(rank, slots, lens):
    rng = np.random.Generator(np.random.PCG64(4 + 1000 * rank))
    per = [lens[i % len(lens)] for i in range(slots)]
    rng.shuffle(per)
    return [[int(x) for x in rng.integers(0, 248320, n)] for n in per]


# ---- clocks -------------------------------------------------------------------------------------------------------
class Clocks:
    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, gpu_index):
        self.gpu, self.proc, self.path = gpu_index, None, f"/tmp/hsg_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu), "-lms", "200"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
            time.sleep(1.0)  # nvidia-smi needs a moment before its first sample
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            self.proc.wait(timeout=10)
            self.out.close()

    def summary(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "samples": len(sm),
                "reasons": sorted(reasons)}


# ---- CPU oracle port ------------------------------------------------------------------------------------------------
def cpu_oracle_rate(sd, slots, steps, warmup):
    """Tokens/s of the CPU oracle's single-token step (oracle.stream.StreamOracle: the reference's slot-engine
    algorithm in fp32 torch) on ``slots`` slots whose state is synthetic but full-size (full 512-column rings,
    random recurrent and conv state), i.e. the same per-step work as the GPU workload."""
    import torch
    from hs_guard_b200 import DEFAULT
    from oracle.stream import StreamOracle
    torch.set_num_threads(os.cpu_count() or 1)
    orc = StreamOracle(sd, DEFAULT, slots)
    g = torch.Generator().manual_seed(5)
    orc.rec.normal_(0, 0.02, generator=g)
    orc.conv.normal_(0, 1.0, generator=g)
    orc.ring_k.normal_(0, 1.0, generator=g)
    orc.ring_v.normal_(0, 1.0, generator=g)
    start = 2048
    for s in range(slots):
        for p in range(start - 512, start):
            orc.ring_pos[s, p % 512] = p
    orc.length[:] = start
    rng = np.random.default_rng(6)
    times = []
    for k in range(warmup + steps):
        req = [(s, [int(rng.integers(0, 248320))]) for s in range(slots)]
        t0 = time.perf_counter()
        orc.step(req)
        if k >= warmup:
            times.append(time.perf_counter() - t0)
    per_step = float(np.mean(times))
    return {"value": slots / per_step, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{slots} slots x {steps} single-token steps (after {warmup} warm-up) of the CPU oracle port "
                      f"(fp32 torch), full 512-column rings, context position {start}",
            "ms_per_step": per_step * 1e3}


def cpu_complete_message_rate(sd, n_tokens=256, reps=2):
    """C1: the CPU oracle port of the reference's complete-message forward (oracle.stream.score_complete, fp32 torch,
    all host threads) on one message of ``n_tokens`` uniform-random ids (seed 1)."""
    import torch
    from hs_guard_b200 import DEFAULT
    from oracle.stream import Weights, score_complete
    torch.set_num_threads(os.cpu_count() or 1)
    w = Weights(sd, DEFAULT)
    ids = np.random.Generator(np.random.PCG64(1)).integers(0, 248320, n_tokens)
    score_complete(sd, DEFAULT, ids, w=w)
    t0 = time.perf_counter()
    for _ in range(reps):
        score_complete(sd, DEFAULT, ids, w=w)
    dt = (time.perf_counter() - t0) / reps
    return {"value": n_tokens / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"batch 1, one message of {n_tokens} ids (seed 1), {reps} timed runs after 1 warm-up",
            "ms_per_message": dt * 1e3}


def gpu_complete_message_rate(sd, state_dtype, n_tokens=256, batch=1, reps=10):
    """The same complete-message scoring on the GPU through MessageScorer (fresh slots, 64-token ticks, probabilities
    copied to the host): ``batch`` messages of ``n_tokens`` ids scored side by side."""
    from hs_guard_b200.messages import MessageScorer
    scorer = MessageScorer(sd, max_slots=batch, state_dtype=state_dtype)
    rng = np.random.Generator(np.random.PCG64(1))
    seqs = [[int(x) for x in rng.integers(0, 248320, n_tokens)] for _ in range(batch)]
    for _ in range(3):
        scorer.probabilities(seqs)
    t0 = time.perf_counter()
    for _ in range(reps):
        scorer.probabilities(seqs)
    dt = (time.perf_counter() - t0) / reps
    scorer.close()
    return {"value": batch * n_tokens / dt, "unit": "tokens/s", "ms_per_batch": dt * 1e3,
            "sample": f"batch {batch} x {n_tokens} ids, {reps} timed batches (host wall clock, includes slot resets, "
                      "H2D of the ids and D2H of the probabilities)"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from hs_guard_b200 import weights as W
    sd = W.random_state_dict(0)
    cb = cpu_oracle_rate(sd, args.cpu_slots, args.steps, args.warmup)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cb["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"C4 single-token streaming step, CPU sample of {args.cpu_slots} slots "
                                   "(the reference path's algorithm, ported; host cores)",
                       "slots_per_gpu": args.slots},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- isolated kernels: configs 2 and 3 ------------------------------------------------------------------------------
class L2Flush:
    """Writes a 256 MB buffer (twice the 126 MB L2) so that the next kernel reads its inputs from HBM."""

    def __init__(self):
        import torch
        self.buf = torch.empty(64 << 20, dtype=torch.float32, device="cuda")

    def __call__(self, stream):
        import torch
        with torch.cuda.stream(stream):
            self.buf.fill_(1.0)


def hbm_peak():
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return peaks["hbm_gbs"], "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, "fallback"


def profile_traffic(key):
    """DRAM bytes per launch of a kernel from the committed ncu summaries (profiles/traffic.json), or None."""
    try:
        return json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))[key]["bytes_per_launch"]
    except (OSError, ValueError, KeyError):
        return None


def bench_c2(lib, steps=1000, reps=5, cold_samples=50):
    """Config 2: the isolated gated-delta-rule step (hsg_gdn_step, fp32 state) on 16 slots x 16 heads, dk = dv = 128,
    state ~ N(0, 0.02), q/k/v bf16 ~ N(0, 1) (the kernel L2-normalises q and k per head), raw a, b ~ N(0, 1) with
    A_log = dt_bias = 0 so that g = -softplus(a) and beta = sigmoid(b); ``steps`` consecutive single-token steps in
    one CUDA graph (seed 2). The state (16.8 MB) stays in L2 across graph steps, so the graph figure is per-step
    latency; ``cold`` times single steps after an L2 flush, the HBM-bound case the roofline fraction uses."""
    import torch
    from hs_guard_b200 import _lib
    n, H, D = 16, 16, 128
    g = torch.Generator(device="cuda").manual_seed(2)
    packed = torch.randn(steps, n, 1, 3 * H * D, device="cuda", generator=g).to(torch.bfloat16)
    a = torch.randn(steps, n, 1, H, device="cuda", generator=g)
    b = torch.randn(steps, n, 1, H, device="cuda", generator=g)
    state = torch.zeros(n + 1, H, D, D, device="cuda")
    state[:n] = torch.randn(n, H, D, D, device="cuda", generator=g) * 0.02
    zeros = torch.zeros(H, device="cuda")
    slots = torch.arange(n, dtype=torch.int64, device="cuda")
    lens = torch.ones(n, dtype=torch.int64, device="cuda")
    o = torch.empty(steps, n, 1, H, D, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()

    def step(t):
        _lib.check(lib.hsg_gdn_step(packed[t].data_ptr(), a[t].data_ptr(), b[t].data_ptr(), zeros.data_ptr(),
                                    zeros.data_ptr(), state.data_ptr(), _lib.HSG_STATE_F32, slots.data_ptr(),
                                    lens.data_ptr(), n, 1, n, o[t].data_ptr(), err.data_ptr(), stream.cuda_stream))
    with torch.cuda.stream(stream):
        for t in range(3):
            step(t)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream, capture_error_mode="relaxed"):
        for t in range(steps):
            step(t)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        graph.replay()
        start.record(stream)
        for _ in range(reps):
            graph.replay()
        end.record(stream)
    end.synchronize()
    graph_us = start.elapsed_time(end) * 1e3 / (reps * steps)
    flush = L2Flush()
    cold = []
    for t in range(cold_samples):
        flush(stream)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        step(t)
        s1.record(stream)
        s1.synchronize()
        cold.append(s0.elapsed_time(s1) * 1e3)
    assert int(err.item()) == 0, "device error in config 2"
    state_bytes = 2 * n * H * D * D * 4                      # read + write, fp32
    io_bytes = n * (3 * H * D * 2 + 2 * H * 4 + H * D * 4)   # q|k|v bf16, a, b, o fp32
    peak, src = hbm_peak()
    cold_us = float(np.median(cold))
    achieved = (state_bytes + io_bytes) / (cold_us * 1e-6) / 1e9
    return {"workload": "C2: gated-delta-rule single-token step, 16 slots x 16 heads, dk = dv = 128, fp32 state, "
                        f"{steps} consecutive steps in one CUDA graph, seed 2",
            "us_per_step_graph": graph_us, "us_per_step_cold": cold_us,
            "algorithmic_bytes_per_step": state_bytes + io_bytes,
            "roofline": {"kernel": "gdn_cols_kernel (fp32 state, isolated)", "bound": "hbm", "achieved": achieved,
                         "peak": peak, "unit": "GB/s", "frac": achieved / peak, "peak_source": src,
                         "traffic": profile_traffic("gdn_cols_c2"),
                         "timing": "median of single steps after an L2 flush"},
            "graph_gbs_l2_resident": (state_bytes + io_bytes) / (graph_us * 1e-6) / 1e9}


def c3_inputs(n=64, window=512, hkv=2, groups=4, dim=256, seed=3):
    """Config 3: 64 slots, rings [n+1][2][513][256] fp16 and the new key/value ~ N(0, 1), q ~ N(0, 1) for 4 query
    heads per KV head; per slot a write position ~ U[0, 512) and a filled length ~ U[1, 512] (rings wrap when the
    filled length exceeds the write position), one query token each. Returns device tensors and the filled lengths."""
    import torch
    r = np.random.Generator(np.random.PCG64(seed))
    f16 = lambda shape: torch.from_numpy(r.standard_normal(shape, dtype=np.float32)).to(torch.bfloat16).half().cuda()
    q = torch.from_numpy(r.standard_normal((n, hkv, groups, dim), dtype=np.float32)).to(torch.bfloat16).float().cuda()
    ring_k, ring_v = f16((n + 1, hkv, window + 1, dim)), f16((n + 1, hkv, window + 1, dim))
    new_k, new_v = f16((n, hkv, 1, dim)), f16((n, hkv, 1, dim))
    wp = r.integers(0, window, n)
    filled = r.integers(1, window + 1, n)
    ring_pos = np.full((n + 1, window + 1), -1, dtype=np.int64)
    starts = np.zeros(n, dtype=np.int64)
    for s in range(n):
        start = int(wp[s]) + (window if filled[s] > wp[s] else 0)
        starts[s] = start
        for p in range(start - int(filled[s]), start):
            ring_pos[s, p % window] = p
    dev = lambda x: torch.from_numpy(x).cuda()
    return (q, ring_k, ring_v, new_k, new_v, dev(ring_pos), dev(np.arange(n, dtype=np.int64)), dev(starts),
            dev(np.ones(n, dtype=np.int64))), filled


def bench_c3(lib, samples=50):
    """Config 3: the isolated ring-window GQA decode (hsg_ring_attention, one query token per slot, with the ring
    write) on 64 slots whose rings are partly filled and wrapped; each sample after an L2 flush (the rings, 67 MB,
    would otherwise stay in L2), CUDA events on the launching stream."""
    import torch
    from hs_guard_b200 import _lib
    (q, rk, rv, nk, nv, rp, slots, starts, lens), filled = c3_inputs()
    n = q.shape[0]
    out = torch.empty(n, 2, 4, 256, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.Stream()

    def call():
        _lib.check(lib.hsg_ring_attention(q.data_ptr(), rk.data_ptr(), rv.data_ptr(), nk.data_ptr(), nv.data_ptr(),
                                          rp.data_ptr(), slots.data_ptr(), starts.data_ptr(), lens.data_ptr(), n, 1,
                                          n, 1.0 / 16.0, out.data_ptr(), 1, err.data_ptr(), stream.cuda_stream))
    for _ in range(3):
        call()
    flush = L2Flush()
    times = []
    for _ in range(samples):
        flush(stream)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        call()
        s1.record(stream)
        s1.synchronize()
        times.append(s0.elapsed_time(s1) * 1e3)
    assert int(err.item()) == 0, "device error in config 3"
    us = float(np.median(times))
    filled_bytes = int(filled.sum()) * 2 * 2 * 256 * 2      # keys + values, 2 KV heads, 256 dims, fp16
    window_bytes = n * 2 * 2 * 512 * 256 * 2
    peak, src = hbm_peak()
    achieved = filled_bytes / (us * 1e-6) / 1e9
    return {"workload": "C3: ring-window GQA decode, 64 slots, window 512, 8 query / 2 KV heads, head_dim 256, "
                        "write position ~ U[0,512), filled ~ U[1,512] incl. wrapped rings, one query per slot, seed 3",
            "us_per_call": us, "filled_tokens_mean": float(filled.mean()),
            "algorithmic_bytes_filled": filled_bytes, "bytes_full_window": window_bytes,
            "roofline": {"kernel": "ring_decode_split_kernel (isolated; split-KV over clusters of 2 CTAs)", "bound": "hbm", "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_source": src,
                         "traffic": profile_traffic("ring_decode_c3"),
                         "timing": "median of calls after an L2 flush"},
            "full_window_frac": window_bytes / (us * 1e-6) / 1e9 / peak}


# ---- ours --------------------------------------------------------------------------------------------------------
def gdn_bytes_per_launch(nb, lb, state_elem=2, conv_history=True):
    """Algorithmic HBM bytes of one gated-delta-rule launch: per row, 16 heads x one 128 x 128 state tile read + write
    (``state_elem`` bytes per element: 32 KB fp16 / 64 KB fp32), the fp32 conv history (3 x 6144) read + write unless
    the input projection's epilogue keeps it (``conv_history`` False), the projection columns it reads (q|k|v|z|a|b)
    and its bf16 hi/lo output."""
    state = 16 * 128 * 128 * state_elem * 2
    conv = 3 * 6144 * 4 * 2 if conv_history else 0
    proj = lb * (6144 + 2048 + 32) * 4
    out = lb * 2048 * 2 * 2
    return nb * (state + conv + proj + out)


def gdn_reference_bytes(nb, lb, state_elem=2):
    """The same launch's bytes at the reference's storage types (bf16 conv history and projections, one bf16 output):
    the bound a kernel with the reference's layout would face. This engine keeps the conv history in fp32 and writes a
    hi/lo output pair for precision, so its own algorithmic bytes (gdn_bytes_per_launch) are larger."""
    state = 16 * 128 * 128 * state_elem * 2
    conv = 3 * 6144 * 2 * 2
    proj = lb * (6144 + 2048 + 32) * 2
    out = lb * 2048 * 2
    return nb * (state + conv + proj + out)


def tick_bytes(nb, lb, state_elem=2):
    """Algorithmic HBM bytes of one whole tick: bf16 weights once (non-embedding), per row the recurrent state
    (18 layers, read + write, ``state_elem`` bytes per element), fp32 conv history (read + write), the fp16 ring
    (6 layers x 2 heads x 512 x 256 x K,V read) and embedding rows."""
    weights = 498_113_344 * 2 + 2 * 512 * 1024 * 2
    per_row = 18 * (16 * 128 * 128 * state_elem * 2 + 3 * 6144 * 4 * 2) + 6 * 2 * 512 * 256 * 2 * 2 + lb * 1024 * 2
    return weights + nb * per_row


def device_steps(eng, S, K, Wm, rng, barrier, max_over_ranks):
    """K single-token ticks of all S slots as graph replays of packed ticks already resident in HBM (after Wm warm-up
    replays), CUDA events on the engine's stream, max over ranks: ms per tick. Advances the engine's lengths."""
    import torch
    from hs_guard_b200 import _lib
    from hs_guard_b200.pack import pack_inputs
    slots = np.arange(S, dtype=np.int64)
    staged = []
    length = eng.length.copy()
    for k in range(Wm + K):
        buf = np.zeros(S + 3 * S, dtype=np.int64)
        pack_inputs([[int(t)] for t in rng.integers(0, 248320, S)], slots, S, 1, length, S, buf)
        length[slots] += 1
        staged.append(torch.from_numpy(buf).cuda())
    L = eng._lib
    for k in range(Wm):
        _lib.check(L.hsg_launch(eng.handle, staged[k].data_ptr(), S, 1))
    _lib.check(L.hsg_synchronize(eng.handle))
    stream = torch.cuda.ExternalStream(L.hsg_stream(eng.handle))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    start.record(stream)
    for k in range(Wm, Wm + K):
        _lib.check(L.hsg_launch(eng.handle, staged[k].data_ptr(), S, 1))
    end.record(stream)
    end.synchronize()
    _lib.check(L.hsg_fetch(eng.handle, S, 1, None))
    eng.length[:] = length
    return max_over_ranks(start.elapsed_time(end) / K)


def gdn_roofline(eng, S, rng, state_elem, kernel):
    """The gated-delta-rule kernel of one eager single-token tick, timed live with CUDA events, against the
    algorithmic bytes of gdn_bytes_per_launch. Returns (roofline dict, per-kernel eager times)."""
    req = [[int(t)] for t in rng.integers(0, 248320, S)]
    _, prof = eng.profile_tick(req, np.arange(S, dtype=np.int64))
    gdn_ms, gdn_n = prof["gdn"]
    avg = gdn_ms / max(gdn_n, 1)
    peak, src = hbm_peak()
    nbytes = gdn_bytes_per_launch(S, 1, state_elem)
    achieved = nbytes / (avg * 1e-3) / 1e9
    traffic = None
    try:
        key = "gdn_step_c4_" + ("f16" if state_elem == 2 else "f32")
        traffic = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))[key]["bytes_per_launch"]
    except (OSError, ValueError, KeyError):
        pass
    ref_bytes = gdn_reference_bytes(S, 1, state_elem)
    return ({"kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
             "frac": achieved / peak, "peak_source": src, "traffic": traffic, "algorithmic_bytes": nbytes,
             "avg_launch_ms": avg, "reference_layout_bytes": ref_bytes,
             "frac_reference_layout": ref_bytes / (avg * 1e-3) / 1e9 / peak},
            {k: round(v[0], 4) for k, v in prof.items() if v[1]})


def c4_state_f32(eng16, sd, S, K, Wm, barrier, max_over_ranks):
    """C4 with the recurrent state stored in fp32 (HSG_FLAG_STATE_F32): an fp32-state engine takes over the fp16 run's
    prefilled pools (the state widened to fp32; a single-token tick's work does not depend on the values) and times K
    single-token ticks of all slots the same way as the headline, plus its delta-rule kernel against the fp32 bytes."""
    import torch
    from hs_guard_b200.engine import SlotEngine
    eng = SlotEngine(sd, S, state_dtype="float32")
    try:
        torch.cuda.synchronize()
        src, dst = eng16.pools(), eng.pools()
        for name in ("rec", "conv", "ring_k", "ring_v", "ring_pos"):
            dst[name].copy_(src[name])
        eng.length[:] = eng16.length
        torch.cuda.synchronize()
        rng = np.random.default_rng(200)
        ms = device_steps(eng, S, K, Wm, rng, barrier, max_over_ranks)
        roof, kernel_ms = gdn_roofline(eng, S, rng, 4, "gdn_step_kernel (fp32 state, fused conv + gated delta rule "
                                                       "+ gated norm)")
        step_bytes = tick_bytes(S, 1, 4)
        peak, _ = hbm_peak()
        return {"workload": "C4 with fp32 recurrent state: 352 slots after the 512/2048/8000-token prefill, "
                            "single-token steps", "value": S / (ms * 1e-3), "unit": "tokens/s", "ms_per_step": ms,
                "steps": K, "warmup": Wm, "gpu_launches": eng.launches_per_step(S, 1) * K, "roofline": roof,
                "step_roofline": {"bytes": step_bytes, "achieved_gbs": step_bytes / (ms * 1e-3) / 1e9,
                                  "frac": step_bytes / (ms * 1e-3) / 1e9 / peak},
                "kernel_ms_eager": kernel_ms}
    finally:
        eng.close()


def guarded(fn, *a, **k):
    """Run one of the default line's extra measurements; a failure is reported in its key, not hidden."""
    try:
        return fn(*a, **k)
    except Exception as exc:  # noqa: BLE001 -- the main measurement stands on its own
        return {"error": f"{type(exc).__name__}: {exc}"}


def run_ours(args):
    import torch
    rank, world, local = dist_env()
    barrier, max_over_ranks = dist_setup(local, world)
    from hs_guard_b200 import weights as W
    from hs_guard_b200.build import build
    from hs_guard_b200.engine import SlotEngine
    from hs_guard_b200.runtime import DEFAULT_METADATA, StreamingGuard

    if rank == 0:
        build()
    if world > 1:
        torch.distributed.barrier()
    S = args.slots
    sd = W.random_state_dict(0)
    eng = SlotEngine(sd, S, state_dtype=args.state_dtype)
    state_elem = 2 if args.state_dtype == "float16" else 4
    guard = StreamingGuard.from_engine(eng, DEFAULT_METADATA)
    lens = tuple(int(x) for x in args.contexts.split(","))
    t0 = time.perf_counter()
    eng.step(list(enumerate(contexts_for(rank, S, lens))))
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0

    rng = np.random.default_rng(100 + rank)
    K, Wm = args.steps, args.warmup
    # ---- device-resident ticks (value) ----
    clk = Clocks(local).__enter__()
    dev_ms = device_steps(eng, S, K, Wm, rng, barrier, max_over_ranks)
    launches = eng.launches_per_step(S, 1)

    # ---- end to end through StreamingGuard.step (e2e) ----
    lat = []
    for k in range(Wm + K):
        req = [(s, [int(t)]) for s, t in zip(range(S), rng.integers(0, 248320, S))]
        barrier() if k == Wm else None
        t0 = time.perf_counter()
        guard.step(req, role="assistant")
        if k >= Wm:
            lat.append((time.perf_counter() - t0) * 1e3)
    clk.__exit__(None, None, None)
    clocks = clk.summary()
    own = [float(np.mean(lat)), float(np.percentile(lat, 50)), float(np.percentile(lat, 95))]
    e2e_ms, p50, p95 = (max_over_ranks(x) for x in own)
    per_rank = None
    if world > 1:
        t = torch.tensor(own + [S / (own[0] * 1e-3), float(len(os.sched_getaffinity(0)))], dtype=torch.float64,
                         device="cuda")
        out = [torch.zeros_like(t) for _ in range(world)]
        torch.distributed.all_gather(out, t)
        per_rank = [{"rank": r, "e2e_ms": float(x[0]), "p50_ms": float(x[1]), "p95_ms": float(x[2]),
                     "e2e_tokens_per_s": float(x[3]), "host_cores_visible": int(x[4])} for r, x in enumerate(out)]

    # ---- live roofline of the dominant kernel (eager tick with per-kernel CUDA events) ----
    roofline, kernel_ms = gdn_roofline(eng, S, rng, state_elem,
                                       "gdn_tc_kernel (fused conv + gated delta rule + gated norm)"
                                       if state_elem == 2 else "gdn_step_kernel (fp32 state)")
    step_bytes = tick_bytes(S, 1, state_elem)
    hbm, _ = hbm_peak()

    cpu = complete = extras = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        extras = {"c2": guarded(bench_c2, eng._lib), "c3": guarded(bench_c3, eng._lib)}
        if state_elem == 2:
            extras["c4_f32"] = guarded(c4_state_f32, eng, sd, S, K, Wm, barrier, max_over_ranks)
        extras["c5"] = guarded(c5_measure, eng, S, 5, 3, rank, world, lens, barrier, max_over_ranks, local,
                               state_elem)
        cb = cpu_oracle_rate(sd, args.cpu_slots, 3, 1)
        cpu = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        eng.close()
        eng = None
        complete = {"gpu_batch1": gpu_complete_message_rate(sd, args.state_dtype),
                    "gpu_batch64": gpu_complete_message_rate(sd, args.state_dtype, batch=64, reps=5),
                    "cpu_port_batch1": cpu_complete_message_rate(sd)}

    if rank == 0:
        value = S * world / (dev_ms * 1e-3)
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K, "warmup": Wm,
            "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": value / world / PUBLISHED_TOKENS_PER_S,
            "dtype": f"f32 (norms, conv history, accumulation; {args.state_dtype} recurrent state; bf16 hi/lo "
                     "tensor-core operands; fp16 ring)",
            "data": "synthetic (uniform random token ids; random-init weights, seed 0)",
            "config": {"workload": "C4: full-model streaming, 352 slots per GPU prefilled with 512/2048/8000 "
                                   "random tokens (1/3 each, seed 4), then single-token role=assistant steps",
                       "slots_per_gpu": S, "contexts": list(lens), "parallelism": f"slot-sharded x{world}",
                       "l2": "no flush: each tick touches ~10.8 GB (> 126 MB L2)", "prefill_s": round(prefill_s, 2)},
            "latency_ms": {"p50": p50, "p95": p95, "device_per_step": dev_ms},
            "e2e": {"value": S * world / (e2e_ms * 1e-3), "unit": "tokens/s", "h2d_bytes_per_step": (S + 3 * S) * 8,
                    "d2h_bytes_per_step": 2 * S * 3 * 4 + 4},
            "gpu_launches": launches * K,
            "clocks": clocks,
            "roofline": roofline,
            "step_roofline": {"bytes": step_bytes, "achieved_gbs": step_bytes / (dev_ms * 1e-3) / 1e9,
                              "frac": step_bytes / (dev_ms * 1e-3) / 1e9 / hbm},
            "kernel_ms_eager": kernel_ms,
            "per_rank": per_rank,
            "cpu_baseline": cpu,
            "complete_message": complete,
        }
        if extras:
            line.update(extras)
        print(json.dumps(line), flush=True)
    if eng is not None:
        eng.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def c5_measure(eng, S, K, Wm, rank, world, lens, barrier, max_over_ranks, local, state_elem, e2e=True):
    """The C5 measurement on an engine: 64-token ticks over S slots, each slot's conversation 512, 2,048 or 8,000
    tokens long (one third each, seed 5 + 1000 rank), reset and reassigned when it ends or after 4,096 tokens; the
    resets (hsg_reset_slot) are inside the timed region. Returns the figures of the C5 line."""
    import torch
    from hs_guard_b200 import _lib
    from hs_guard_b200.pack import pack_inputs
    from hs_guard_b200.runtime import DEFAULT_METADATA, StreamingGuard
    LB, CAP = 64, 4096
    guard = StreamingGuard.from_engine(eng, DEFAULT_METADATA)
    rng = np.random.Generator(np.random.PCG64(5 + 1000 * rank))

    def conversation():
        return min(int(rng.choice(lens)), CAP) // LB * LB

    left = np.array([conversation() for _ in range(S)], dtype=np.int64)
    left = rng.integers(1, left // LB + 1) * LB  # staggered: each slot starts somewhere inside its first conversation
    slots = np.arange(S, dtype=np.int64)

    def plan(n):
        """n ticks: (slots reset before the tick, token chunks)."""
        out = []
        for _ in range(n):
            resets = np.nonzero(left == 0)[0]
            for s in resets:
                left[s] = conversation()
            out.append((resets.tolist(), rng.integers(0, 248320, (S, LB))))
            left[:] -= LB
        return out

    # ---- device-resident ticks (value) ----
    eng.reset()
    L = eng._lib
    ticks = plan(Wm + K)
    length = eng.length.copy()
    staged = []
    for resets, chunk in ticks:
        length[resets] = 0
        buf = np.zeros(S * LB + 3 * S, dtype=np.int64)
        pack_inputs(chunk.tolist(), slots, S, LB, length, S, buf)
        length += LB
        staged.append(torch.from_numpy(buf).cuda())

    def run_tick(k):
        for s in ticks[k][0]:
            _lib.check(L.hsg_reset_slot(eng.handle, int(s)))
        _lib.check(L.hsg_launch(eng.handle, staged[k].data_ptr(), S, LB))

    for k in range(Wm):
        run_tick(k)
    _lib.check(L.hsg_synchronize(eng.handle))
    stream = torch.cuda.ExternalStream(L.hsg_stream(eng.handle))
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = Clocks(local).__enter__()
    barrier()
    start.record(stream)
    for k in range(Wm, Wm + K):
        run_tick(k)
    end.record(stream)
    end.synchronize()
    _lib.check(L.hsg_fetch(eng.handle, S, LB, None))
    eng.length[:] = length
    dev_ms = max_over_ranks(start.elapsed_time(end) / K)
    n_resets = sum(len(t[0]) for t in ticks[Wm:])

    # ---- end to end: slot resets + StreamingGuard.step with host lists ----
    lat = []
    if e2e:
        for k, (resets, chunk) in enumerate(plan(Wm + K)):
            req = [(int(s), row) for s, row in zip(slots, chunk.tolist())]  # the caller's request list, as in C4
            if k == Wm:
                barrier()
            t0 = time.perf_counter()
            for s in resets:
                eng.reset_slot(s)
            guard.step(req, role="assistant")
            if k >= Wm:
                lat.append((time.perf_counter() - t0) * 1e3)
    clk.__exit__(None, None, None)
    e2e_ms = max_over_ranks(float(np.mean(lat))) if lat else None
    p50 = max_over_ranks(float(np.percentile(lat, 50))) if lat else None
    p95 = max_over_ranks(float(np.percentile(lat, 95))) if lat else None

    # ---- per-kernel CUDA events of one eager tick ----
    _, prof = eng.profile_tick(rng.integers(0, 248320, (S, LB)).tolist(), slots)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    tflops_peak, tsrc = (peaks["bf16_tflops_sustained"], "measured sustained") if "bf16_tflops_sustained" in peaks \
        else (1400.0, "fallback sustained")
    hbm, hsrc = hbm_peak()
    gemm_ms = sum(v[0] for k, v in prof.items() if k.startswith("gemm") or k == "head_gemm")
    gemm_n = sum(v[1] for k, v in prof.items() if k.startswith("gemm") or k == "head_gemm")
    gemm_flops = 2.0 * 498_113_344 * S * LB  # algorithmic (the hi/lo activation pair executes twice this)
    gdn_ms, gdn_n = prof["gdn"]
    # the chunked delta rule of a 64-token tick: tcgen05 (default) or the warp-MMA comparison (HSG_GDN_WY=0); with the
    # former the conv + SiLU runs in the input projection's epilogue unless HSG_GDN_CONV_GEMM=0
    wy = os.environ.get("HSG_GDN_WY", "1") != "0"
    pre = wy and os.environ.get("HSG_GDN_CONV_GEMM", "1") != "0"
    gdn_bytes = gdn_bytes_per_launch(S, LB, state_elem, conv_history=not pre)
    gdn_kernel = ("gdn_wy_kernel (tcgen05" + ("; conv + SiLU in the input projection's epilogue)" if pre else ")")
                  if wy else "gdn_chunk_kernel (warp-level mma.sync)")
    gdn_traffic = profile_traffic("gdn_wy_c5") if pre and S == 352 else None
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12
    tokens = S * LB * world
    return {
        "value": tokens / (dev_ms * 1e-3), "ms_per_step": dev_ms, "tokens_per_tick": S * LB,
        "resets_in_timed_ticks": n_resets, "clocks": clk.summary(),
        "latency_ms": {"p50": p50, "p95": p95, "device_per_step": dev_ms},
        "e2e": None if e2e_ms is None else {"value": tokens / (e2e_ms * 1e-3), "unit": "tokens/s",
                                            "h2d_bytes_per_step": (S * LB + 3 * S) * 8,
                                            "d2h_bytes_per_step": 2 * S * LB * 3 * 4 + 4},
        "gpu_launches": eng.launches_per_step(S, LB) * K,
        "roofline": {"kernel": "gemm_pc_kernel + gemm_tc_kernel (all projections of one tick)", "bound": "tensor",
                     "achieved": achieved, "peak": tflops_peak, "unit": "TFLOP/s", "frac": achieved / tflops_peak,
                     "peak_source": tsrc, "traffic": None, "algorithmic_flops": gemm_flops,
                     "tick_ms": gemm_ms, "launches": gemm_n},
        "gdn_chunk": {"kernel": gdn_kernel, "avg_launch_ms": gdn_ms / max(gdn_n, 1),
                      "algorithmic_bytes": gdn_bytes, "traffic": gdn_traffic,
                      "achieved_gbs": gdn_bytes / (gdn_ms / max(gdn_n, 1) * 1e-3) / 1e9,
                      "hbm_frac": gdn_bytes / (gdn_ms / max(gdn_n, 1) * 1e-3) / 1e9 / hbm, "peak_source": hsrc},
        "kernel_ms_eager": {k: round(v[0], 4) for k, v in prof.items() if v[1]},
    }


def dist_setup(local, world):
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())
    return barrier, max_over_ranks


def run_c5(args):
    """C5 per GPU: 352 slots stream 64-token ticks (the chunked delta-rule path) with slot reset and reassignment
    (c5_measure); a step is one tick of 352 x 64 tokens."""
    import torch
    rank, world, local = dist_env()
    barrier, max_over_ranks = dist_setup(local, world)
    from hs_guard_b200 import weights as W
    from hs_guard_b200.build import build
    from hs_guard_b200.engine import SlotEngine

    if rank == 0:
        build()
    if world > 1:
        torch.distributed.barrier()
    S = args.slots
    sd = W.random_state_dict(0)
    eng = SlotEngine(sd, S, state_dtype=args.state_dtype)
    state_elem = 2 if args.state_dtype == "float16" else 4
    lens = tuple(int(x) for x in args.contexts.split(","))
    r = c5_measure(eng, S, args.steps, args.warmup, rank, world, lens, barrier, max_over_ranks, local, state_elem)
    if rank == 0:
        line = {
            "metric": "scored tokens/s/GPU at 352 slots (C5: 64-token ticks)", "value": r["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": r["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": f"f32 (norms, conv history, accumulation; {args.state_dtype} recurrent state; bf16 hi/lo "
                     "tensor-core operands; fp16 ring)",
            "data": "synthetic (uniform random token ids; random-init weights, seed 0)",
            "config": {"workload": "C5: 64-token ticks over 352 slots per GPU, contexts 512/2048/8000 (seed 5), "
                                   "slot reset and reassignment at the end of a conversation or after 4096 tokens",
                       "slots_per_gpu": S, "tokens_per_tick": S * 64, "contexts": list(lens), "reassign_after": 4096,
                       "resets_in_timed_ticks": r["resets_in_timed_ticks"], "parallelism": f"slot-sharded x{world}",
                       "l2": "no flush: each tick touches > 10 GB (> 126 MB L2)"},
            "latency_ms": r["latency_ms"], "e2e": r["e2e"], "gpu_launches": r["gpu_launches"], "clocks": r["clocks"],
            "roofline": r["roofline"], "gdn_chunk": r["gdn_chunk"], "kernel_ms_eager": r["kernel_ms_eager"],
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def run_kernel_config(args):
    """One JSON line for config 2 or 3 on cuda:0 (rank 0 only): the same measurement as the default line's c2 / c3."""
    import torch
    rank, _, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    from hs_guard_b200 import _lib
    from hs_guard_b200.build import build
    build()
    r = (bench_c2 if args.workload == "c2" else bench_c3)(_lib.lib())
    us = r["us_per_step_graph"] if args.workload == "c2" else r["us_per_call"]
    line = {"metric": "us per step (config 2: gated-delta-rule step)" if args.workload == "c2"
            else "us per call (config 3: ring-window decode)", "value": us, "unit": "us", "n_gpus": 1,
            "higher_is_better": False, "dtype": "f32" if args.workload == "c2" else "f16 (fp32 softmax)",
            "data": "synthetic", "config": {"workload": r["workload"]}, "vs_baseline": None}
    line.update({k: v for k, v in r.items() if k != "workload"})
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "c5":
        run_c5(args)
    elif args.workload in ("c2", "c3"):
        run_kernel_config(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
