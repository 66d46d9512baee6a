"""The roofline arithmetic of bench.py, on the CPU: algorithmic bytes per
decode token (weights + K/V at the mean context T + N/2) and FLOPs per
prefill (projections on every row, causal attention, last-row lm_head) for
each workload, against figures worked out by hand from the model shapes
(ModelBase.cpp's per-layer tensors: q/k/v/o, gate/up/down, two RMSNorm
weights, the optional bias and q/k-norm weights, the embedding and lm_head)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

# workload -> (GB per decode token at the mean context, TFLOP per prefill)
EXPECTED = {
    "qwen3-0.6b": (1.203, None),
    "llama3.2-3b": (6.499, 2.932),
    "qwen2.5-7b": (14.626, 120.4),
    "llama3.1-8b": (15.345, 29.7),
    "mistral-7b-v0.3": (14.563, 29.7),
    "llama3.1-70b": (140.43, 582.8),
}


@pytest.mark.parametrize("workload", sorted(EXPECTED))
def test_roofline_arithmetic(workload):
    import bench
    from yalama_b200 import synth
    preset, prompt, gen = bench.WORKLOADS[workload][:3]
    spec = synth.PRESETS[preset]
    gb, tf = EXPECTED[workload]
    got = bench.decode_bytes_per_token(spec, prompt + gen // 2, 1) / 1e9
    assert abs(got - gb) <= 0.0015 * gb, (got, gb)
    if tf is not None:
        got_tf = bench.prefill_flops(spec, prompt) / 1e12
        assert abs(got_tf - tf) <= 0.002 * tf, (got_tf, tf)


def test_tensor_parallel_shares():
    import bench
    from yalama_b200 import synth
    spec = synth.PRESETS["llama3.1-8b"]
    one = bench.decode_bytes_per_token(spec, 2560, 1)
    for tp in (2, 4, 8):
        assert bench.decode_bytes_per_token(spec, 2560, tp) == pytest.approx(one / tp)
    r = bench.prefill_roofline(spec, 2048, 80000.0, 8)
    assert r["flops_per_prefill_per_gpu"] == pytest.approx(bench.prefill_flops(spec, 2048) / 8)
    assert r["achieved_tflops"] == pytest.approx(r["flops_per_prefill_per_gpu"] * 80000.0 / 2048 / 1e12)
    assert r["frac"] == pytest.approx(r["achieved_tflops"] / r["peak_tflops"])


def test_prefill_attention_term_is_causal():
    # one layer, no projections: 4 D Hq T (T + 1) / 2 FLOPs (QK^T and PV over
    # keys 0..i for query i), plus the last-row lm_head 2 V H
    import bench
    from types import SimpleNamespace
    s = SimpleNamespace(hidden=0, head_dim=128, intermediate=0, vocab=0, heads=2, kv_heads=1, layers=1)
    assert bench.prefill_flops(s, 3) == 4 * 128 * 2 * 6
    s = SimpleNamespace(hidden=4, head_dim=128, intermediate=0, vocab=10, heads=0, kv_heads=0, layers=0)
    assert bench.prefill_flops(s, 100) == 2 * 10 * 4
