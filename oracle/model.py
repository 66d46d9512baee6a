"""Numpy restatement of the reference decoder forward — TEST INFRASTRUCTURE ONLY.

Follows ``ModelBase::Infer`` (``src/models/ModelBase.cpp:396-471``) step by
step, including the rounding to the storage dtype after every LibTorch op, the
fixed-size KV cache and its capacity rule, and the RoPE position quirk of the
decode branch. ``mode`` selects the storage dtype: ``"f32"`` reproduces the
reference compiled for CPU/FP32, ``"f16"`` the FP16 storage the engine uses,
``"bf16"`` the reference as shipped.

Reference quirks reproduced (all switchable):
- decode tokens are rotated at position ``slot - 1`` (``ModelBase.cpp:458-461,
  570-584``): after a prefill of T0 tokens ``last = T0 - 1``, the decode token
  is written to slot ``last + 1`` and rotated at ``last``;
- Llama-3 RoPE scaling is parsed but not applied (``ModelBase.cpp:372-394``);
  ``rope_scaling=True`` applies it as Llama 3.1 defines it;
- the decode capacity check tests ``last + 1 <= cap - last``
  (``ModelBase.cpp:570, 853-866``);
- a one-token prefill leaves ``last = 0``, so the next call is a prefill again.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Tuple

import numpy as np

from .numerics import ROUNDERS

OK = 0
SEQUENCE_LENGTH_EXCEEDED = 1
KV_CACHE_EXCEEDED = 2


def kv_capacity_tokens(kv_gb: int, kv_heads: int, head_dim: int, layers: int) -> int:
    """``ModelBase::InitKVCache`` (ModelBase.cpp:345-357): BF16-sized slots."""
    total = int(float(kv_gb) * 1024 * 1024 * 1024)
    per_token = 1 * kv_heads * head_dim * 2
    return (total // per_token) // layers // 2


def llama3_inv_freq(inv_freq: np.ndarray, factor: float, low: float, high: float, orig: int) -> np.ndarray:
    """Llama 3.1 frequency scaling, restated from its published definition
    (Meta's Llama 3.1 release; HF ``_compute_llama3_parameters``): wavelengths
    shorter than orig/high are kept, longer than orig/low are divided by the
    factor, and the band in between is interpolated smoothly."""
    inv = inv_freq.astype(np.float64)
    low_wl = orig / low
    high_wl = orig / high
    wl = 2.0 * math.pi / inv
    out = np.where(wl > low_wl, inv / factor, inv)
    smooth = (orig / wl - low) / (high - low)
    mid = (1.0 - smooth) * inv / factor + smooth * inv
    is_mid = (wl <= low_wl) & (wl >= high_wl)
    out = np.where(is_mid, mid, out)
    return out.astype(np.float32)


def rope_tables(head_dim: int, max_t: int, theta: float, mode: str,
                scaling: Optional[dict] = None) -> Tuple[np.ndarray, np.ndarray]:
    """``ModelBase::BuildRopeCache`` (ModelBase.cpp:372-394): FP32
    ``inv_freq = 1/theta^(i/half)``, ``freqs = pos x inv_freq``,
    ``cos/sin(cat(freqs, freqs))`` rounded to the storage dtype."""
    r = ROUNDERS[mode]
    half = head_dim // 2
    idx = np.arange(half, dtype=np.float32)
    expo = (idx / np.float32(half)).astype(np.float32)
    inv_freq = (1.0 / np.power(np.float64(np.float32(theta)), expo.astype(np.float64))).astype(np.float32)
    if scaling is not None:
        inv_freq = llama3_inv_freq(inv_freq, scaling["factor"], scaling["low_freq_factor"],
                                   scaling["high_freq_factor"], scaling["original_max_position_embeddings"])
    pos = np.arange(max_t, dtype=np.float32)
    freqs = (pos[:, None] * inv_freq[None, :]).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    cos = r(np.cos(emb.astype(np.float64)).astype(np.float32))
    sin = r(np.sin(emb.astype(np.float64)).astype(np.float32))
    return cos, sin


class OracleModel:
    """One model replica with its KV cache, driven like ``Model``
    (``src/models/Model.cpp:10-53``): ``begin_infer()`` then ``infer(ids)``."""

    def __init__(self, spec, weights: Dict[str, np.ndarray], mode: str = "f16", kv_gb: int = 2,
                 kv_enabled: bool = True, rope_scaling: bool = False, rope_compat: bool = True,
                 max_seq_len: Optional[int] = None):
        self.spec = spec
        self.mode = mode
        self.r = ROUNDERS[mode]
        self.W = {k: self.r(np.asarray(v, dtype=np.float32)) for k, v in weights.items()}
        self.kv_enabled = kv_enabled
        self.rope_compat = rope_compat
        self.cap = kv_capacity_tokens(kv_gb, spec.kv_heads, spec.head_dim, spec.layers)
        self.max_seq_len = spec.max_pos if max_seq_len is None else min(spec.max_pos, max_seq_len)
        scal = spec.rope_scaling if rope_scaling else None
        self.cos, self.sin = rope_tables(spec.head_dim, spec.max_pos, spec.rope_theta, mode, scal)
        self.lm_head = self.W.get("lm_head.weight", self.W["model.embed_tokens.weight"])
        self.ready = False
        self.last = 0
        self.K: List[np.ndarray] = []
        self.V: List[np.ndarray] = []

    # -- Model::BeginInfer (ModelBase.cpp:296-310)
    def begin_infer(self) -> None:
        self.ready = True
        self.last = 0
        s = self.spec
        self.K = [np.zeros((s.kv_heads, 0, s.head_dim), np.float32) for _ in range(s.layers)]
        self.V = [np.zeros((s.kv_heads, 0, s.head_dim), np.float32) for _ in range(s.layers)]

    def _ensure_slots(self, layer: int, n: int) -> None:
        have = self.K[layer].shape[1]
        if n > have:
            grow = max(n, 2 * have) - have
            pad = np.zeros((self.spec.kv_heads, grow, self.spec.head_dim), np.float32)
            self.K[layer] = np.concatenate([self.K[layer], pad], axis=1)
            self.V[layer] = np.concatenate([self.V[layer], pad], axis=1)

    # -- building blocks -------------------------------------------------
    def mm(self, x: np.ndarray, w: np.ndarray) -> np.ndarray:
        return self.r(np.asarray(x, np.float32) @ w.T)

    def rmsnorm(self, x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
        """``CalculateRMSNorm`` (ModelBase.cpp:724-736) and Qwen3's
        ``ApplyHeadDimRMSNorm`` (Qwen3Model.cpp:26-33)."""
        r = self.r
        sq = r(x * x)
        mean = r((sq.astype(np.float64).sum(-1, keepdims=True) / x.shape[-1]).astype(np.float32))
        denom = r((1.0 / np.sqrt(mean.astype(np.float64) + np.float64(np.float32(eps)))).astype(np.float32))
        return r(r(x * denom) * w)

    def rope(self, x: np.ndarray, start: int) -> np.ndarray:
        """``ApplyInferencingRope`` (ModelBase.cpp:784-820); x is [heads, T, D]."""
        r = self.r
        T, D = x.shape[1], x.shape[2]
        half = D // 2
        cos = self.cos[start:start + T][None]
        sin = self.sin[start:start + T][None]
        xcos = r(x * cos)
        rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
        xsin = r(rot * sin)
        return r(xcos + xsin)

    def sdpa(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool) -> np.ndarray:
        """``scaled_dot_product_attention`` with the GQA expansion of
        ``ExpandKV`` (ModelBase.cpp:671-707); scale 1/sqrt(D); q [Hq,T,D],
        k/v [Hkv,S,D]. Computed in float64, rounded to the storage dtype."""
        Hq, T, D = q.shape
        Hkv, S = k.shape[0], k.shape[1]
        rep = Hq // Hkv
        out = np.empty((Hq, T, D), np.float32)
        scale = 1.0 / math.sqrt(D)
        for h in range(Hq):
            g = h // rep
            s = (q[h].astype(np.float64) @ k[g].astype(np.float64).T) * scale
            if causal:
                # additive mask triu(ones(Tk,Tk),1) * -65504 sliced to Tq rows (:620-633)
                qi = np.arange(T)[:, None]
                kj = np.arange(S)[None, :]
                s = np.where(kj > qi, -np.inf, s)
            s = s - s.max(-1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(-1, keepdims=True)
            out[h] = (p @ v[g].astype(np.float64)).astype(np.float32)
        return self.r(out)

    # -- ModelBase::CalculateInferenceAttention (ModelBase.cpp:507-654)
    def attention(self, xn: np.ndarray, layer: int) -> Tuple[Optional[np.ndarray], bool]:
        s, W, r = self.spec, self.W, self.r
        p = f"model.layers.{layer}."
        T = xn.shape[0]
        D = s.head_dim
        q = self.mm(xn, W[p + "self_attn.q_proj.weight"])
        k = self.mm(xn, W[p + "self_attn.k_proj.weight"])
        v = self.mm(xn, W[p + "self_attn.v_proj.weight"])
        if s.qkv_bias:  # Qwen2_5Model.cpp:25-47
            q = r(q + W[p + "self_attn.q_proj.bias"])
            k = r(k + W[p + "self_attn.k_proj.bias"])
            v = r(v + W[p + "self_attn.v_proj.bias"])
        q = q.reshape(T, s.heads, D).transpose(1, 0, 2)
        k = k.reshape(T, s.kv_heads, D).transpose(1, 0, 2)
        v = v.reshape(T, s.kv_heads, D).transpose(1, 0, 2)
        if s.qk_norm:  # Qwen3Model.cpp:16-33
            q = self.rmsnorm(q, W[p + "self_attn.q_norm.weight"], s.rms_eps)
            k = self.rmsnorm(k, W[p + "self_attn.k_norm.weight"], s.rms_eps)

        if self.last == 0:  # KV cache disabled, or prefill (:539-543)
            q = self.rope(q, 0)
            k = self.rope(k, 0)
        causal = True
        if self.kv_enabled:
            if self.last == 0:  # prefill write (:547-565)
                if T > self.cap - self.last:
                    return None, False
                self._ensure_slots(layer, T)
                self.K[layer][:, :T] = k
                self.V[layer][:, :T] = v
            else:  # decode (:566-586)
                if self.last + 1 > self.cap - self.last:
                    return None, False
                if T != 1:
                    raise ValueError("decode takes one token")
                pos = self.last if self.rope_compat else self.last + 1
                q = self.rope(q, pos)
                k = self.rope(k, pos)
                slot = self.last + 1
                self._ensure_slots(layer, slot + 1)
                self.K[layer][:, slot] = k[:, 0]
                self.V[layer][:, slot] = v[:, 0]
                k = self.K[layer][:, :slot + 1]
                v = self.V[layer][:, :slot + 1]
                causal = False  # no mask on decode (:620)
        att = self.sdpa(q, k, v, causal)
        merged = att.transpose(1, 0, 2).reshape(T, s.heads * D)
        return self.mm(merged, W[p + "self_attn.o_proj.weight"]), True

    def ffn(self, x: np.ndarray, layer: int) -> np.ndarray:
        """``CalculateFFN`` (ModelBase.cpp:738-753): down(silu(gate) * up)."""
        r, W = self.r, self.W
        p = f"model.layers.{layer}.mlp."
        gate = self.mm(x, W[p + "gate_proj.weight"])
        up = self.mm(x, W[p + "up_proj.weight"])
        g64 = gate.astype(np.float64)
        act = r((g64 / (1.0 + np.exp(-g64))).astype(np.float32))
        h = r(act * up)
        return self.mm(h, W[p + "down_proj.weight"])

    def ensure_sequence_length(self, ids: np.ndarray, eos_per_prompt: List[int]) -> np.ndarray:
        """``EnsureSequenceLength`` (ModelBase.cpp:473-505): left-trim whole
        earlier prompts (or single tokens) until the ids fit."""
        while len(ids) > self.max_seq_len:
            if not eos_per_prompt:
                ids = ids[1:]
            else:
                drop = eos_per_prompt[0] + 1
                ids = ids[drop:]
                del eos_per_prompt[0]
                for i in range(len(eos_per_prompt)):
                    eos_per_prompt[i] -= drop
        return ids

    # -- ModelBase::Infer (ModelBase.cpp:396-471)
    def infer(self, ids, eos_per_prompt: Optional[List[int]] = None) -> Tuple[int, Optional[np.ndarray]]:
        """Returns (status, last-row logits). The reference returns all T rows
        of logits; ChatSession keeps only the last (ChatSession.cpp:136-138)."""
        if not self.ready:
            raise RuntimeError("Call BeginInfer() first")
        ids = np.asarray(ids, dtype=np.int64)
        ids = self.ensure_sequence_length(ids, eos_per_prompt if eos_per_prompt is not None else [])
        self.ids = ids  # Infer trims its in/out argument in place
        s, W, r = self.spec, self.W, self.r
        x = r(W["model.embed_tokens.weight"][ids])
        for layer in range(s.layers):
            p = f"model.layers.{layer}."
            xn = self.rmsnorm(x, W[p + "input_layernorm.weight"], s.rms_eps)
            att, ok = self.attention(xn, layer)
            if not ok:
                return KV_CACHE_EXCEEDED, None
            x = r(x + att)
            xn2 = self.rmsnorm(x, W[p + "post_attention_layernorm.weight"], s.rms_eps)
            x = r(x + self.ffn(xn2, layer))
        x = self.rmsnorm(x[-1:], W["model.norm.weight"], s.rms_eps)
        logits = self.mm(x, self.lm_head)[0]
        if self.kv_enabled:
            if self.last == 0:
                self.last = len(ids) - 1
            else:
                self.last += 1
        return OK, logits
