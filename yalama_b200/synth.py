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


TILE_PERIOD = 16777213  # 2**24 - 3, prime


def tiled_values(block: np.ndarray, start: int, shape: Tuple[int, ...]) -> np.ndarray:
    """`block` read cyclically from `start` into an array of `shape` (float32)."""
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    p = block.size
    pos, src = 0, start % p
    while pos < n:
        c = min(n - pos, p - src)
        out[pos:pos + c] = block[src:src + c]
        pos += c
        src = 0
    return out.reshape(shape)


def round_bf16(a: np.ndarray) -> np.ndarray:
    """float32 values rounded to BF16 (nearest even), as float32."""
    f = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((f + np.uint32(0x7FFF) + ((f >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)) << np.uint32(16)
    return r.view(np.float32)


def write_snapshot(root: str, spec: ModelSpec, seed: int = 0, dtype: str = "F16",
                   std: float = 0.02, shard_bytes: int = 4 << 30, fast: bool = False,
                   snapshot_hash: str = "0000000000000000000000000000000000000000",
                   through_bf16: bool = False) -> str:
    """Write an HF hub layout under `root`; return the snapshot directory.

    `through_bf16=True` rounds every value to BF16 before it is stored as
    `dtype` (an F16 snapshot then holds exactly what a BF16 one decodes to).

    `fast=True` fills the weights from one block of ``TILE_PERIOD`` N(0, std)
    values (numpy PCG64 from the seed), each tensor reading the block
    cyclically from its own offset, instead of the counter-based generator:
    the same distribution, written at disk speed for billions of parameters.
    The period is prime, so no two rows of a power-of-two-wide (or any
    shorter-than-the-period) matrix repeat. Use it where every consumer loads
    the same file (timing, or parity between two loaders of the snapshot).
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
    block = None
    if fast:
        block = np.random.default_rng(seed).standard_normal(TILE_PERIOD, dtype=np.float32) * np.float32(std)

    def producer(name, shape):
        def make():
            if fast and not name.endswith("norm.weight"):
                v = tiled_values(block, fnv1a64(name) % TILE_PERIOD, shape)
            else:
                v = tensor_values(seed, name, shape, std)
            return round_bf16(v).reshape(v.shape) if through_bf16 else v
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


# ---------------------------------------------------------------------------
# Byte-level BPE tokenizer fixture (tokenizer.json / tokenizer_config.json)
# ---------------------------------------------------------------------------
# Special tokens per family, as the reference's chat templates spell them
# (include/chat_templates/*ChatTemplateProvider.h); the last one is the EOS.
SPECIAL_TOKENS = {
    "llama": ["<|begin_of_text|>", "<|end_of_text|>", "<|start_header_id|>", "<|end_header_id|>",
              "<|reserved_special_token_0|>", "<|eot_id|>"],
    "qwen": ["<|endoftext|>", "<|im_start|>", "<think>", "</think>", "<|im_end|>"],
}

_SAMPLE_TEXT = (
    "The engine streams every weight matrix once per token, and the attention reads the cached keys "
    "and values of the context. A persistent kernel keeps one block on each multiprocessor, so the "
    "next projection starts while the previous one is finishing. Tokens are generated one at a time: "
    "the model reads the prompt, then answers with the most likely word, again and again, until it "
    "reaches the end of the text or the length limit."
)


def byte_alphabet() -> List[str]:
    """The byte-level BPE alphabet: byte b -> a printable character (bytes
    33-126, 161-172, 174-255 map to themselves, the others to 256 + n in
    order), the mapping the reference's TokenizerBase::BuildByteEncoder
    builds (src/tokenizer/TokenizerBase.cpp:17-63)."""
    safe = set(range(33, 127)) | set(range(161, 173)) | set(range(174, 256))
    out, n = [], 0
    for b in range(256):
        if b in safe:
            out.append(chr(b))
        else:
            out.append(chr(256 + n))
            n += 1
    return out


def train_merges(text: str, n_merges: int) -> List[Tuple[str, str]]:
    """Greedy BPE merges (most frequent adjacent pair first, ties by first
    occurrence) over the words of `text` in the byte alphabet, a space
    attached to the following word as 'Ġ'."""
    alpha = byte_alphabet()
    words: List[List[str]] = []
    for i, w in enumerate(text.split(" ")):
        b = (" " + w if i else w).encode()
        words.append([alpha[c] for c in b])
    merges: List[Tuple[str, str]] = []
    for _ in range(n_merges):
        counts: Dict[Tuple[str, str], int] = {}
        order: Dict[Tuple[str, str], int] = {}
        for w in words:
            for a, b in zip(w, w[1:]):
                counts[(a, b)] = counts.get((a, b), 0) + 1
                order.setdefault((a, b), len(order))
        if not counts:
            break
        best = max(counts, key=lambda p: (counts[p], -order[p]))
        if counts[best] < 2:
            break
        merges.append(best)
        for j, w in enumerate(words):
            out, k = [], 0
            while k < len(w):
                if k + 1 < len(w) and (w[k], w[k + 1]) == best:
                    out.append(w[k] + w[k + 1])
                    k += 2
                else:
                    out.append(w[k])
                    k += 1
            words[j] = out
    return merges


def write_tokenizer(snap: str, spec: ModelSpec, family: str = "llama", n_merges: int = 200) -> Dict[str, int]:
    """Write tokenizer.json (byte-level BPE: the 256 byte characters as ids
    0-255, merges learned from a fixed sample text as the next ids, the
    family's special tokens as the last ids of the vocabulary) and a
    tokenizer_config.json naming the EOS and carrying a chat template. Returns
    the special tokens' ids. The vocabulary fits in spec.vocab."""
    specials = SPECIAL_TOKENS[family]
    merges = train_merges(_SAMPLE_TEXT, n_merges)
    vocab: Dict[str, int] = {c: i for i, c in enumerate(byte_alphabet())}
    for a, b in merges:
        if a + b not in vocab:
            vocab[a + b] = len(vocab)
    if len(vocab) + len(specials) > spec.vocab:
        raise ValueError("vocabulary too small for the tokenizer fixture")
    sp = {t: spec.vocab - len(specials) + i for i, t in enumerate(specials)}
    tok = {
        "version": "1.0",
        "added_tokens": [{"id": i, "content": t, "single_word": False, "lstrip": False, "rstrip": False,
                          "normalized": False, "special": True} for t, i in sp.items()],
        "model": {"type": "BPE", "vocab": vocab, "merges": [f"{a} {b}" for a, b in merges]},
    }
    with open(os.path.join(snap, "tokenizer.json"), "w") as f:
        json.dump(tok, f, ensure_ascii=False)
    eos = specials[-1]
    with open(os.path.join(snap, "tokenizer_config.json"), "w") as f:
        json.dump({"eos_token": eos, "bos_token": specials[0] if family == "llama" else None,
                   "chat_template": "{% for m in messages %}{{ m.content }}{% endfor %}"}, f)
    cfg_path = os.path.join(snap, "config.json")
    cfg = json.load(open(cfg_path))
    cfg["eos_token_id"] = sp[eos]
    with open(cfg_path, "w") as f:
        json.dump(cfg, f, indent=1)
    return sp


# ---------------------------------------------------------------- large BPE tokenizers
# A tokenizer.json with tens of thousands of merges and a text to encode with
# it, for checking and timing the host BPE encoder on long prompts. The merge
# table is built from a seeded lexicon of syllable words (pairwise, level by
# level, most frequent words first), so merges nest the way trained ones do;
# the text draws those words with Zipf frequencies, with punctuation, digits,
# newlines and multi-byte characters, and optional special tokens.
_SYL_CONS = ["b", "c", "d", "f", "g", "h", "j", "k", "l", "m", "n", "p", "r", "s", "t", "v", "w", "z",
             "ch", "sh", "th", "st", "tr", "pl"]
_SYL_VOWS = ["a", "e", "i", "o", "u", "ai", "ea", "ou", "é", "ü", "ø"]


def _lexicon(rng: np.random.Generator, n_words: int) -> List[str]:
    seen, out = set(), []
    while len(out) < n_words:
        k = int(rng.integers(1, 5))
        w = ""
        for _ in range(k):
            w += _SYL_CONS[int(rng.integers(len(_SYL_CONS)))] + _SYL_VOWS[int(rng.integers(len(_SYL_VOWS)))]
            if rng.random() < 0.3:
                w += _SYL_CONS[int(rng.integers(len(_SYL_CONS)))]
        if rng.random() < 0.02:
            w += "中"  # a 3-byte character
        if w not in seen:
            seen.add(w)
            out.append(w)
    return out


def _symbols(text: str, family: str) -> List[str]:
    """The base symbols the reference's tokenizer splits `text` into before BPE:
    byte-alphabet characters (Llama, Qwen) or UTF-8 characters with '▁' for
    a space (Mistral)."""
    if family == "mistral":
        return list(text.replace(" ", "▁"))
    alpha = byte_alphabet()
    return [alpha[b] for b in text.encode()]


def bpe_tokenizer(family: str, n_merges: int, seed: int = 0, n_words: int = 20000):
    """(vocab {token: id}, merges ["a b"], special {token: id}, lexicon)."""
    rng = np.random.default_rng(seed)
    lex = _lexicon(rng, n_words)
    if family == "mistral":
        base = sorted(set("".join(lex)) | set(" ,.?!:;'\n0123456789-") - {" "}) + ["▁"]
        vocab: Dict[str, int] = {"<unk>": 0}
        for c in base:
            vocab.setdefault(c, len(vocab))
    else:
        vocab = {c: i for i, c in enumerate(byte_alphabet())}
    merges: List[str] = []
    have = set()
    for w in lex:
        for form in (" " + w, w):
            s = _symbols(form, family)
            while len(s) > 1 and len(merges) < n_merges:
                nxt = []
                for i in range(0, len(s), 2):
                    if i + 1 < len(s):
                        key = s[i] + " " + s[i + 1]
                        if key not in have:
                            have.add(key)
                            merges.append(key)
                            vocab.setdefault(s[i] + s[i + 1], len(vocab))
                        nxt.append(s[i] + s[i + 1])
                    else:
                        nxt.append(s[i])
                s = nxt
        if len(merges) >= n_merges:
            break
    specials = SPECIAL_TOKENS["qwen" if family == "qwen" else "llama"]
    sp = {t: len(vocab) + i for i, t in enumerate(specials)}
    return vocab, merges, sp, lex


def write_bpe_tokenizer(folder: str, family: str, n_merges: int, seed: int = 0) -> Dict[str, int]:
    """Write `folder`/tokenizer.json (the layout LoadFromJson reads,
    src/tokenizer/TokenizerBase.cpp:65-208). Returns the special tokens' ids."""
    vocab, merges, sp, _ = bpe_tokenizer(family, n_merges, seed)
    tok = {
        "version": "1.0",
        "added_tokens": [{"id": i, "content": t, "single_word": False, "lstrip": False, "rstrip": False,
                          "normalized": False, "special": True} for t, i in sp.items()],
        "model": {"type": "BPE", "vocab": vocab, "merges": merges},
    }
    os.makedirs(folder, exist_ok=True)
    with open(os.path.join(folder, "tokenizer.json"), "w", encoding="utf-8") as f:
        json.dump(tok, f, ensure_ascii=False)
    return sp


def bpe_text(family: str, n_bytes: int, seed: int = 0, specials_every: int = 0, n_merges: int = 0) -> str:
    """About `n_bytes` of text in the lexicon of bpe_tokenizer(family, seed);
    a special token of the family after every `specials_every` words (0: none)."""
    rng = np.random.default_rng(seed + 1)
    lex = _lexicon(np.random.default_rng(seed), 20000)
    p = 1.0 / (np.arange(len(lex)) + 10.0)
    p /= p.sum()
    specials = SPECIAL_TOKENS["qwen" if family == "qwen" else "llama"]
    out, size, nw = [], 0, 0
    picks, rolls, k = np.empty(0, np.int64), np.empty(0), 0
    while size < n_bytes:
        if k == len(picks):
            picks, rolls, k = rng.choice(len(lex), size=4096, p=p), rng.random(4096), 0
        w, r = lex[int(picks[k])], float(rolls[k])
        k += 1
        if r < 0.05:
            w += ","
        elif r < 0.08:
            w += "."
        elif r < 0.09:
            w += "?\n"
        elif r < 0.10:
            w = str(int(rng.integers(0, 100000)))
        out.append(w)
        size += len(w.encode()) + 1
        nw += 1
        if specials_every and nw % specials_every == 0:
            out.append(specials[int(rng.integers(len(specials)))])
    return " ".join(out)
