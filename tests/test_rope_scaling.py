"""The oracle's Llama-3 RoPE frequency scaling, pinned against an independent
implementation: Hugging Face transformers' ``_compute_llama3_parameters``
(transformers.modeling_rope_utils, in this image).

The reference parses the scaling fields (src/ConfigManager.cpp:443-463) but its
BuildRopeCache (src/models/ModelBase.cpp:372-394) uses plain theta only, so the
reference cannot pin the scaled variant; the engine's ``rope_scaling = 1`` table
is checked against this oracle on the GPU (tests/test_gpu_model.py)."""
import numpy as np
import pytest

from oracle.model import llama3_inv_freq, rope_tables
from yalama_b200 import synth

transformers = pytest.importorskip("transformers")


def hf_inv_freq(spec):
    from transformers import LlamaConfig
    from transformers.modeling_rope_utils import _compute_llama3_parameters
    cfg = LlamaConfig(hidden_size=spec.hidden, num_attention_heads=spec.heads, head_dim=spec.head_dim,
                      rope_theta=spec.rope_theta, max_position_embeddings=spec.max_pos,
                      rope_scaling=dict(spec.rope_scaling))
    inv, attention_factor = _compute_llama3_parameters(cfg, None)
    assert attention_factor == 1.0
    return inv.double().numpy()


def plain_inv_freq(spec):
    half = spec.head_dim // 2
    expo = (np.arange(half, dtype=np.float32) / np.float32(half)).astype(np.float32)
    return (1.0 / np.power(np.float64(np.float32(spec.rope_theta)), expo.astype(np.float64))).astype(np.float32)


@pytest.mark.parametrize("preset", ["llama3.2-3b", "llama3.1-8b", "llama3.1-70b"])
def test_llama3_inv_freq_matches_transformers(preset):
    spec = synth.PRESETS[preset]
    s = spec.rope_scaling
    ours = llama3_inv_freq(plain_inv_freq(spec), s["factor"], s["low_freq_factor"], s["high_freq_factor"],
                           s["original_max_position_embeddings"]).astype(np.float64)
    ref = hf_inv_freq(spec)
    # both round to FP32 after different operation orders: a few ulps
    np.testing.assert_allclose(ours, ref, rtol=2e-6, atol=0)
    # and the scaling really changes the low frequencies (wavelength > 8192 / 1)
    plain = plain_inv_freq(spec).astype(np.float64)
    wl = 2 * np.pi / plain
    low = wl > s["original_max_position_embeddings"] / s["low_freq_factor"]
    assert low.sum() > 20
    np.testing.assert_allclose(ours[low], plain[low] / s["factor"], rtol=2e-6)
    high = wl < s["original_max_position_embeddings"] / s["high_freq_factor"]
    np.testing.assert_array_equal(ours[high], plain[high])


def test_scaled_rope_table_follows_the_frequencies():
    spec = synth.PRESETS["llama3.1-8b"]
    cos, sin = rope_tables(spec.head_dim, 4096, spec.rope_theta, "f32", spec.rope_scaling)
    inv = hf_inv_freq(spec)
    pos = np.arange(4096, dtype=np.float64)[:, None]
    # angle error of FP32 inverse frequencies: pos x a few ulps
    tol = 4096 * np.max(inv) * 4e-7 + 1e-6
    np.testing.assert_allclose(cos[:, :64], np.cos(pos * inv[None, :]), atol=tol)
    np.testing.assert_allclose(sin[:, 64:], np.sin(pos * inv[None, :]), atol=tol)
