"""Seeded random-init model snapshots in the Hugging Face hub layout.

The reference loads a model from an HF hub directory: ``refs/main`` names a
snapshot hash, and ``snapshots/<hash>/`` holds ``config.json``,
``tokenizer_config.json`` (with ``eos_token``) and the ``*.safetensors`` shards
(``src/ConfigManager.cpp:320-342, 389-496``; shard discovery
``src/models/ModelBase.cpp:42-75``). Shards are accepted only when their header
contains ``"data_offsets"``, ``"__metadata__"`` and ``"format":"pt"`` with no
spaces (``ModelBase.cpp:63-66``). This module writes exactly that layout for
the model shapes the engine serves, with weights drawn from a counter-based
generator so every tensor element is reproducible from ``(seed, name, index)``
on any machine, in numpy here and in CUDA on the device
(``ylm_create`` with no snapshot directory uses the same generator).

Weights are ``N(0, std)`` (default 0.02) rounded to FP16-representable values,
RMSNorm and q/k-norm weights are 1.0, and Qwen2.5 biases are ``N(0, std)``.
"""
from __future__ import annotations

import dataclasses
import json
import os
import struct
from typing import Dict, Iterator, List, Optional, Tuple

import numpy as np

# model_type strings as config.json spells them (src/ConfigManager.cpp:410-421)
MODEL_TYPES = {"llama": 1, "mistral": 2, "qwen2": 3, "qwen3": 4}


@dataclasses.dataclass
class ModelSpec:
    """Architecture of a Llama-style decoder, as config.json describes it."""

    model_type: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: Optional[dict] = None
    tied: bool = False
    max_pos: int = 131072
    eos_token_id: int = 0

    @property
    def qkv_bias(self) -> bool:
        # Qwen2.5 adds q/k/v biases (src/models/Qwen2_5Model.cpp:16-47)
        return self.model_type == "qwen2"

    @property
    def qk_norm(self) -> bool:
        # Qwen3 adds per-head q/k RMSNorm (src/models/Qwen3Model.cpp:8-33)
        return self.model_type == "qwen3"

    def config_json(self) -> dict:
        cfg = {
            "model_type": self.model_type,
            "num_hidden_layers": self.layers,
            "hidden_size": self.hidden,
            "num_attention_heads": self.heads,
            "num_key_value_heads": self.kv_heads,
            "head_dim": self.head_dim,
            "intermediate_size": self.intermediate,
            "vocab_size": self.vocab,
            "rms_norm_eps": self.rms_eps,
            "rope_theta": self.rope_theta,
            "max_position_embeddings": self.max_pos,
            "tie_word_embeddings": self.tied,
            "eos_token_id": self.eos_token_id,
            "torch_dtype": "float16",
        }
        if self.rope_scaling is not None:
            cfg["rope_scaling"] = dict(self.rope_scaling)
        return cfg

    def tensor_shapes(self) -> List[Tuple[str, Tuple[int, ...]]]:
        """HF tensor names and shapes (names: src/models/ModelBase.cpp:239-253)."""
        H, D, I, V = self.hidden, self.head_dim, self.intermediate, self.vocab
        q, kv = self.heads * D, self.kv_heads * D
        out: List[Tuple[str, Tuple[int, ...]]] = [("model.embed_tokens.weight", (V, H))]
        for l in range(self.layers):
            p = f"model.layers.{l}."
            out += [
                (p + "input_layernorm.weight", (H,)),
                (p + "self_attn.q_proj.weight", (q, H)),
                (p + "self_attn.k_proj.weight", (kv, H)),
                (p + "self_attn.v_proj.weight", (kv, H)),
            ]
            if self.qkv_bias:
                out += [
                    (p + "self_attn.q_proj.bias", (q,)),
                    (p + "self_attn.k_proj.bias", (kv,)),
                    (p + "self_attn.v_proj.bias", (kv,)),
                ]
            if self.qk_norm:
                out += [
                    (p + "self_attn.q_norm.weight", (D,)),
                    (p + "self_attn.k_norm.weight", (D,)),
                ]
            out += [
                (p + "self_attn.o_proj.weight", (H, q)),
                (p + "post_attention_layernorm.weight", (H,)),
                (p + "mlp.gate_proj.weight", (I, H)),
                (p + "mlp.up_proj.weight", (I, H)),
                (p + "mlp.down_proj.weight", (H, I)),
            ]
        out.append(("model.norm.weight", (H,)))
        if not self.tied:
            out.append(("lm_head.weight", (V, H)))
        return out

    def n_params(self) -> int:
        return sum(int(np.prod(s)) for _, s in self.tensor_shapes())


_LLAMA3_SCALING = {
    "rope_type": "llama3",
    "factor": 32.0,
    "low_freq_factor": 1.0,
    "high_freq_factor": 4.0,
    "original_max_position_embeddings": 8192,
}

# Model shapes the engine is measured on (random-init, seeded).
PRESETS: Dict[str, ModelSpec] = {
    "qwen3-0.6b": ModelSpec("qwen3", 1024, 28, 16, 8, 128, 3072, 151936, 1e-6, 1e6,
                            tied=True, max_pos=40960, eos_token_id=151645),
    "llama3.2-3b": ModelSpec("llama", 3072, 28, 24, 8, 128, 8192, 128256, 1e-5, 5e5,
                             rope_scaling=_LLAMA3_SCALING, tied=True, eos_token_id=128009),
    "qwen2.5-7b": ModelSpec("qwen2", 3584, 28, 28, 4, 128, 18944, 152064, 1e-6, 1e6,
                            tied=False, max_pos=32768, eos_token_id=151645),
    "llama3.1-8b": ModelSpec("llama", 4096, 32, 32, 8, 128, 14336, 128256, 1e-5, 5e5,
                             rope_scaling=_LLAMA3_SCALING, tied=False, eos_token_id=128009),
    "mistral-7b-v0.3": ModelSpec("mistral", 4096, 32, 32, 8, 128, 14336, 32768, 1e-5, 1e6,
                                 tied=False, max_pos=32768, eos_token_id=2),
    "llama3.1-70b": ModelSpec("llama", 8192, 80, 64, 8, 128, 28672, 128256, 1e-5, 5e5,
                              rope_scaling=_LLAMA3_SCALING, tied=False, eos_token_id=128009),
}


def tiny_spec(model_type: str = "qwen3", layers: int = 2, hidden: int = 256, heads: int = 4,
              kv_heads: int = 2, intermediate: int = 512, vocab: int = 1000, **kw) -> ModelSpec:
    """Small model of a given family for CPU-speed parity cases (head_dim 128)."""
    base = dict(rms_eps=1e-6, rope_theta=1e6, tied=(model_type == "qwen3"), max_pos=4096,
                eos_token_id=vocab - 1)
    base.update(kw)
    return ModelSpec(model_type, hidden, layers, heads, kv_heads, 128, intermediate, vocab, **base)


# ---------------------------------------------------------------------------
# Counter-based N(0, std) generator (SplitMix64 hash + Box-Muller).
# SplitMix64's finaliser is the published one (Steele, Lea, Flood, "Fast
# splittable pseudorandom number generators", OOPSLA 2014; constants as in
# Vigna's public-domain splitmix64.c). Element i of tensor `name` under `seed`
# uses the two 64-bit hashes of counters 2i and 2i+1 in the stream keyed by
# mix(seed) ^ fnv1a64(name). The CUDA initialiser computes the same values.
# ---------------------------------------------------------------------------
_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
_GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def _mix64(z: np.ndarray) -> np.ndarray:
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def fnv1a64(s: str) -> int:
    h = 0xCBF29CE484222325
    for b in s.encode():
        h ^= b
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h


def stream_key(seed: int, name: str) -> int:
    with np.errstate(over="ignore"):
        s = _mix64(np.array([seed & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64))[0]
    return int(s) ^ fnv1a64(name)


def normal_values(seed: int, name: str, start: int, count: int, std: float = 0.02) -> np.ndarray:
    """Elements [start, start+count) of tensor `name`, as float16."""
    key = np.uint64(stream_key(seed, name))
    i = np.arange(start, start + count, dtype=np.uint64)
    with np.errstate(over="ignore"):
        c1 = key + (np.uint64(2) * i) * _GOLDEN
        c2 = key + (np.uint64(2) * i + np.uint64(1)) * _GOLDEN
        z1 = _mix64(c1)
        z2 = _mix64(c2)
    u1 = ((z1 >> np.uint64(11)).astype(np.float64) + 1.0) * (2.0 ** -53)  # (0, 1]
    u2 = (z2 >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)  # [0, 1)
    n = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (std * n).astype(np.float16)


def tensor_values(seed: int, name: str, shape: Tuple[int, ...], std: float = 0.02,
                  chunk: int = 1 << 24) -> np.ndarray:
    """Full tensor `name`: 1.0 for norm weights, seeded N(0, std) otherwise."""
    n = int(np.prod(shape))
    if name.endswith("norm.weight"):
        return np.ones(shape, dtype=np.float16)
    out = np.empty(n, dtype=np.float16)
    for s in range(0, n, chunk):
        c = min(chunk, n - s)
        out[s:s + c] = normal_values(seed, name, s, c, std)
    return out.reshape(shape)


def model_weights(spec: ModelSpec, seed: int = 0, std: float = 0.02) -> Dict[str, np.ndarray]:
    return {name: tensor_values(seed, name, shape, std) for name, shape in spec.tensor_shapes()}


# ---------------------------------------------------------------------------
# safetensors writer
# ---------------------------------------------------------------------------
_ST_DTYPES = {"F16": np.float16, "F32": np.float32, "BF16": None}


def _to_bf16_bytes(a: np.ndarray) -> bytes:
    f = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounded = (f + np.uint32(0x7FFF) + ((f >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return rounded.astype(np.uint16).tobytes()


def _encode(a: np.ndarray, dtype: str) -> bytes:
    if dtype == "BF16":
        return _to_bf16_bytes(a)
    return np.ascontiguousarray(a, dtype=_ST_DTYPES[dtype]).tobytes()


def write_safetensors(path: str, tensors: List[Tuple[str, Tuple[int, ...], "callable"]], dtype: str) -> None:
    """Write one shard. `tensors` holds (name, shape, producer) with producer()
    returning the array, so a large shard is generated one tensor at a time.

    The header is written compactly (``{"__metadata__":{"format":"pt"},...}``),
    padded with spaces to a multiple of 8 bytes, and never so that the data
    start lands on a page boundary: the reference's shard struct unmaps
    ``data`` on copy (include/safetensors.h:27-34), which only fails harmlessly
    while ``8 + header_len`` is not page aligned.
    """
    esize = {"F16": 2, "BF16": 2, "F32": 4}[dtype]
    header = {"__metadata__": {"format": "pt"}}
    off = 0
    for name, shape, _ in tensors:
        nbytes = int(np.prod(shape)) * esize
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    hb = json.dumps(header, separators=(",", ":")).encode()
    pad = (8 - len(hb) % 8) % 8
    hb += b" " * pad
    while (8 + len(hb)) % 4096 == 0:
        hb += b" " * 8
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name, shape, producer in tensors:
            a = producer()
            assert tuple(a.shape) == tuple(shape), (name, a.shape, shape)
            f.write(_encode(a, dtype))


def write_snapshot(root: str, spec: ModelSpec, seed: int = 0, dtype: str = "F16",
                   std: float = 0.02, shard_bytes: int = 4 << 30, fast: bool = False,
                   snapshot_hash: str = "0000000000000000000000000000000000000000") -> str:
    """Write an HF hub layout under `root`; return the snapshot directory.

    `fast=True` draws weights with numpy's PCG64 normal generator instead of
    the counter-based one (same distribution, much faster at billions of
    parameters); use it where only timing matters.
    """
    snap = os.path.join(root, "snapshots", snapshot_hash)
    os.makedirs(snap, exist_ok=True)
    os.makedirs(os.path.join(root, "refs"), exist_ok=True)
    with open(os.path.join(root, "refs", "main"), "w") as f:
        f.write(snapshot_hash)
    with open(os.path.join(snap, "config.json"), "w") as f:
        json.dump(spec.config_json(), f, indent=1)
    with open(os.path.join(snap, "tokenizer_config.json"), "w") as f:
        json.dump({"eos_token": "<eos>", "bos_token": None}, f)

    esize = {"F16": 2, "BF16": 2, "F32": 4}[dtype]
    rng = np.random.default_rng(seed) if fast else None

    def producer(name, shape):
        def make():
            if fast and not name.endswith("norm.weight"):
                return (rng.standard_normal(shape, dtype=np.float32) * np.float32(std))
            return tensor_values(seed, name, shape, std)
        return make

    shards: List[List] = [[]]
    size = 0
    for name, shape in spec.tensor_shapes():
        nb = int(np.prod(shape)) * esize
        if shards[-1] and size + nb > shard_bytes:
            shards.append([])
            size = 0
        shards[-1].append((name, shape, producer(name, shape)))
        size += nb
    n = len(shards)
    for i, sh in enumerate(shards):
        fname = "model.safetensors" if n == 1 else f"model-{i + 1:05d}-of-{n:05d}.safetensors"
        write_safetensors(os.path.join(snap, fname), sh, dtype)
    return snap


def read_safetensors(path: str) -> Dict[str, np.ndarray]:
    """Read a shard written by write_safetensors (F16/F32/BF16) as float32."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        s, e = meta["data_offsets"]
        raw = data[s:e]
        if meta["dtype"] == "BF16":
            a = (np.frombuffer(raw, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            a = np.frombuffer(raw, dtype=_ST_DTYPES[meta["dtype"]]).astype(np.float32)
        out[name] = a.reshape(meta["shape"])
    return out


def write_ids(path: str, ids) -> None:
    np.asarray(ids, dtype=np.int64).tofile(path)


def prompt_ids(seed: int, n: int, vocab: int) -> np.ndarray:
    """Prompt of n token ids uniform over [0, vocab), from the seed."""
    return np.random.default_rng(seed + 0x5EED).integers(0, vocab, size=n, dtype=np.int64)
