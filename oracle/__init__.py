"""CPU oracle for the HS-Guard slot-based streaming step -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU in fp32 (torch/numpy), the algorithm of the reference's streaming path so that
the CUDA engine can be checked against it. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import it, and only as the checker or as the timed CPU baseline; the product path
(``hs_guard_b200``) never imports, calls or falls back to anything here.

Modules:
- ``pack``: ``pack_inputs`` (reference ``src/hs_guard/engine/slot_engine_v7.py:7-25``), bit-exact integer layout.
- ``kernels``: the gated-delta-rule slot step (``engine/fused_kernels.py:140-211``), the ring-window attention
  contract (``engine/ring_attention_kernel.py:7-26``) and the causal-conv step (``fused_kernels.py:94-136``).
- ``stream``: the whole streaming engine (pools, tick, step splitting) following
  ``engine/bucketed_engine.py:22-132`` and ``engine/slot_engine_v7.py:117-167``, plus the complete-message scorer
  (``runtime.py:136-145`` with ``window_attention.py:34-53``).

Pinning: ``tests/golden/make_golden.py`` runs the reference itself (its pure-torch streaming engine and its
complete-message scorer on CPU, transformers' torch GDN) on seeded inputs and stores the outputs under
``tests/golden/``; ``tests/test_oracle_golden.py`` checks this oracle against those vectors.
"""
