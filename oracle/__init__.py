"""CPU oracle for the yalama token loop — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, what the reference computes on its hot path
(``ModelBase::Infer`` and ``ChatSession::Sample``), so that tests, the smoke
check and the benchmark's CPU baseline can check the CUDA engine against it.
Nothing in the product (``yalama_b200``) imports it; the engine fails loudly
when its CUDA library is missing instead of falling back to this code.

- ``oracle.numerics``: dtype rounding, the sampler's exp, Philox4x32-10.
- ``oracle.model``: the decoder forward with the reference's rounding points,
  KV-cache state machine and RoPE quirks.
- ``oracle.sampler``: greedy and top-k/temperature sampling.
- ``oracle/ref``: the recipe that compiles the reference's own model sources
  (LibTorch, CPU FP32 / CUDA FP16 / CUDA BF16) into ``oracle/_ref``; the
  restatement is pinned against it through ``tests/golden``.
"""
