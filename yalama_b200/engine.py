"""Python binding of the engine's C ABI (include/yalama_b200.h), via ctypes.

The classes mirror the reference's host interface for the token loop:

- ``Model`` is the static facade of ``src/models/Model.cpp:10-53``
  (``Init`` / ``BeginInfer`` / ``Infer``) returning a ``GenerationResult``
  (``include/GenerationResult.h:6-11``) with the last-row logits;
- ``Engine`` is the handle behind it (one per GPU / tensor-parallel rank), with
  ``sample`` (``ChatSession::Sample``, ``src/ChatSession.cpp:560-593``),
  ``decode`` (one-launch Infer + Sample) and ``generate`` (the token loop of
  ``ChatSession::Generate``, ``src/ChatSession.cpp:113-230``, on token ids).

The library is required: if ``libyalama_b200.so`` is missing or fails to load,
every entry raises instead of computing anything another way.
"""
from __future__ import annotations

import ctypes
import enum
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libyalama_b200.so")


class Status(enum.IntEnum):
    OK = 0
    SEQUENCE_LENGTH_EXCEEDED = 1
    KV_CACHE_EXCEEDED = 2
    INVALID_PROMPT = 3
    CANCELED = 4
    GPU_QUEUE_TIMED_OUT = 5
    INVALID_ARG = 16
    NOT_READY = 17
    LOAD_ERROR = 18
    CUDA_ERROR = 19
    DEVICE_TIMEOUT = 20
    COMM_ERROR = 21
    UNSUPPORTED = 22


# GenerationError (include/enums/GenerationError.h:1-8) are the first six statuses
GENERATION_ERRORS = {Status.OK, Status.SEQUENCE_LENGTH_EXCEEDED, Status.KV_CACHE_EXCEEDED,
                     Status.INVALID_PROMPT, Status.CANCELED, Status.GPU_QUEUE_TIMED_OUT}

MODEL_TYPES = {"llama": 1, "mistral": 2, "qwen2": 3, "qwen3": 4}


class ModelConfig(ctypes.Structure):
    _fields_ = [
        ("model_type", ctypes.c_int32),
        ("num_layers", ctypes.c_int32),
        ("hidden_size", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("intermediate_size", ctypes.c_int32),
        ("tie_word_embeddings", ctypes.c_int32),
        ("vocab_size", ctypes.c_int64),
        ("rms_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("rope_factor", ctypes.c_float),
        ("rope_low_freq", ctypes.c_float),
        ("rope_high_freq", ctypes.c_float),
        ("rope_orig_max_pos", ctypes.c_int32),
        ("max_position_embeddings", ctypes.c_int32),
        ("eos_ids", ctypes.c_int32 * 8),
        ("n_eos", ctypes.c_int32),
    ]


class EngineOptions(ctypes.Structure):
    _fields_ = [
        ("device", ctypes.c_int32),
        ("kv_cache_gb", ctypes.c_int32),
        ("kv_cache_enabled", ctypes.c_int32),
        ("rope_compat", ctypes.c_int32),
        ("rope_scaling", ctypes.c_int32),
        ("use_cuda_graph", ctypes.c_int32),
        ("use_pdl", ctypes.c_int32),
        ("tp_rank", ctypes.c_int32),
        ("tp_size", ctypes.c_int32),
        ("nccl_id", ctypes.c_void_p),
        ("init_seed", ctypes.c_uint64),
        ("init_std", ctypes.c_double),
        ("zero_kv_on_begin", ctypes.c_int32),
        ("prefill_tensor_cores", ctypes.c_int32),
        ("decode_persistent", ctypes.c_int32),
        ("wait_limit_us", ctypes.c_int32),
    ]


class Sampling(ctypes.Structure):
    _fields_ = [
        ("greedy", ctypes.c_int32),
        ("top_k", ctypes.c_int32),
        ("temperature", ctypes.c_float),
        ("seed", ctypes.c_uint64),
        ("masked_ids", ctypes.POINTER(ctypes.c_int64)),
        ("n_masked", ctypes.c_int32),
    ]


class YlmError(RuntimeError):
    def __init__(self, status: int, where: str, message: str):
        self.status = Status(status) if status in Status._value2member_map_ else status
        super().__init__(f"{where}: {self.status!r}: {message}")


_lib = None
_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)
_I64P = ctypes.POINTER(ctypes.c_int64)
_F32P = ctypes.POINTER(ctypes.c_float)
_F64P = ctypes.POINTER(ctypes.c_double)

# exported symbol -> (restype, argtypes)
SIGNATURES = {
    "ylm_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "ylm_last_error": (ctypes.c_char_p, []),
    "ylm_options_default": (ctypes.c_int, [ctypes.POINTER(EngineOptions)]),
    "ylm_config_from_json": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ModelConfig)]),
    "ylm_resolve_snapshot": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int32]),
    "ylm_nccl_unique_id": (ctypes.c_int, [_P]),
    "ylm_create": (ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(ModelConfig), ctypes.POINTER(EngineOptions),
                                  ctypes.POINTER(_P)]),
    "ylm_destroy": (ctypes.c_int, [_P]),
    "ylm_begin_infer": (ctypes.c_int, [_P]),
    "ylm_infer": (ctypes.c_int, [_P, _I64P, _I32P, _I32P, _I32P]),
    "ylm_logits": (ctypes.c_int, [_P, _P, ctypes.c_int32]),
    "ylm_logits_device": (ctypes.c_int, [_P, ctypes.POINTER(_P), _I64P]),
    "ylm_set_sampling": (ctypes.c_int, [_P, ctypes.POINTER(Sampling)]),
    "ylm_sample": (ctypes.c_int, [_P, ctypes.c_int32, _I64P]),
    "ylm_decode": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int32, _I64P]),
    "ylm_generate": (ctypes.c_int, [_P, _I64P, ctypes.c_int32, ctypes.c_int32, _I64P, ctypes.c_int32, _I64P, _I32P,
                                    _F64P, _F64P]),
    "ylm_set_draw": (ctypes.c_int, [_P, ctypes.c_float]),
    "ylm_last_topk": (ctypes.c_int, [_P, _I64P, _F32P, _I32P, _F32P]),
    "ylm_info": (ctypes.c_int, [_P, _I32P, _I32P, _I32P]),
    "ylm_time_decode": (ctypes.c_int, [_P, ctypes.c_int32, _F64P]),
    "ylm_last_prefill_ms": (ctypes.c_int, [_P, _F64P]),
    "ylm_decode_path": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_int32)]),
    "ylm_time_segment": (ctypes.c_int, [_P, ctypes.c_int32, ctypes.c_int32, _F64P, _F64P]),
    "ylm_exchange_stats": (ctypes.c_int, [_P, ctypes.c_int32, _F64P, _F64P, _F64P]),
    "ylm_time_allreduce": (ctypes.c_int, [_P, ctypes.c_int32, _F64P]),
    "ylm_set_attention_path": (ctypes.c_int, [ctypes.c_int32]),
    "ylm_debug_drop_output": (ctypes.c_int, [_P, ctypes.c_int32]),
    "ylm_k_gemv": (ctypes.c_int, [_P, ctypes.c_int32, ctypes.c_int32, _P, _P, _P]),
    "ylm_k_gemm": (ctypes.c_int, [_P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _P, ctypes.c_int32, _P]),
    "ylm_k_prefill_attention": (ctypes.c_int, [_P, _P, _P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                               ctypes.c_int32, _P, ctypes.c_int32, _P]),
    "ylm_k_decode_attention": (ctypes.c_int, [_P, _P, _P, ctypes.c_float, _P, _P, ctypes.c_int32, _P, _P,
                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_int32, _P, _P]),
    "ylm_k_decode_attention_noalloc": (ctypes.c_int, [_P, _P, _P, ctypes.c_float, _P, _P, ctypes.c_int32, _P, _P,
                                                      ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                                      ctypes.c_int32, _P, _P]),
    "ylm_k_sample": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_float, _P,
                                    ctypes.c_float, _I64P, _I64P, _F32P, _P]),
}


def lib() -> ctypes.CDLL:
    """Load the engine library (raises when it is missing: there is no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m yalama_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class split_attention:
    """Context manager: the split-K decode-attention kernel for every launch
    (and CUDA graph captured) inside the block, process-wide."""

    def __enter__(self):
        check(lib().ylm_set_attention_path(1), "ylm_set_attention_path")
        return self

    def __exit__(self, *exc):
        lib().ylm_set_attention_path(0)
        return False


def check(status: int, where: str) -> None:
    if status != 0:
        raise YlmError(status, where, lib().ylm_last_error().decode(errors="replace"))


def _i64(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


def config_from_spec(spec) -> ModelConfig:
    """ModelConfig from a yalama_b200.synth.ModelSpec (or anything with its fields)."""
    c = ModelConfig()
    c.model_type = MODEL_TYPES[spec.model_type]
    c.num_layers = spec.layers
    c.hidden_size = spec.hidden
    c.num_heads = spec.heads
    c.num_kv_heads = spec.kv_heads
    c.head_dim = spec.head_dim
    c.intermediate_size = spec.intermediate
    c.tie_word_embeddings = int(spec.tied)
    c.vocab_size = spec.vocab
    c.rms_eps = spec.rms_eps
    c.rope_theta = spec.rope_theta
    rs = spec.rope_scaling or {}
    c.rope_factor = rs.get("factor", 1.0)
    c.rope_low_freq = rs.get("low_freq_factor", 1.0)
    c.rope_high_freq = rs.get("high_freq_factor", 1.0)
    c.rope_orig_max_pos = rs.get("original_max_position_embeddings", spec.max_pos)
    c.max_position_embeddings = spec.max_pos
    c.eos_ids[0] = spec.eos_token_id
    c.n_eos = 1
    return c


def config_from_json(path: str) -> ModelConfig:
    c = ModelConfig()
    check(lib().ylm_config_from_json(path.encode(), ctypes.byref(c)), "ylm_config_from_json")
    return c


def resolve_snapshot(hf_root: str) -> str:
    buf = ctypes.create_string_buffer(4096)
    check(lib().ylm_resolve_snapshot(hf_root.encode(), buf, len(buf)), "ylm_resolve_snapshot")
    return buf.value.decode()


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    check(lib().ylm_nccl_unique_id(buf), "ylm_nccl_unique_id")
    return buf.raw


def default_options(**kw) -> EngineOptions:
    o = EngineOptions()
    check(lib().ylm_options_default(ctypes.byref(o)), "ylm_options_default")
    for k, v in kw.items():
        if not hasattr(o, k):
            raise TypeError(f"unknown engine option {k}")
        setattr(o, k, v)
    return o


@dataclass
class GenerationResult:
    """include/GenerationResult.h:6-11 (Logits holds the last row only)."""
    Logits: Optional[np.ndarray]
    IsSuccess: bool
    Error: Status


class Engine:
    """One engine (one GPU / tensor-parallel rank)."""

    def __init__(self, snapshot_dir: Optional[str], config: ModelConfig, nccl_id: Optional[bytes] = None, **options):
        self._h = _P()
        self._nccl = ctypes.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
        opt = default_options(**options)
        if self._nccl is not None:
            opt.nccl_id = ctypes.cast(self._nccl, ctypes.c_void_p)
        self.config = config
        self.vocab = int(config.vocab_size)
        self._masked = None
        check(lib().ylm_create(snapshot_dir.encode() if snapshot_dir else None, ctypes.byref(config),
                               ctypes.byref(opt), ctypes.byref(self._h)), "ylm_create")

    def close(self) -> None:
        if self._h:
            lib().ylm_destroy(self._h)
            self._h = _P()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- Model facade
    def begin_infer(self) -> None:
        check(lib().ylm_begin_infer(self._h), "ylm_begin_infer")

    def infer(self, ids: Sequence[int], eos_per_prompt: Optional[List[int]] = None):
        """Model::Infer: returns (status, trimmed ids). Raises on non-GenerationError failures."""
        a = _i64(ids).copy()
        n = ctypes.c_int32(a.size)
        eos = np.asarray(eos_per_prompt or [], dtype=np.int32).copy()
        ne = ctypes.c_int32(eos.size)
        st = lib().ylm_infer(self._h, _ptr(a, ctypes.c_int64), ctypes.byref(n),
                             _ptr(eos, ctypes.c_int32) if eos.size else None, ctypes.byref(ne))
        if st not in GENERATION_ERRORS:
            check(st, "ylm_infer")
        if eos_per_prompt is not None:
            eos_per_prompt[:] = [int(v) for v in eos[:ne.value]]
        return Status(st), a[:n.value]

    def logits(self, as_float32: bool = True) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32 if as_float32 else np.float16)
        check(lib().ylm_logits(self._h, out.ctypes.data_as(_P), int(as_float32)), "ylm_logits")
        return out

    def logits_device(self):
        p = _P()
        v = ctypes.c_int64()
        check(lib().ylm_logits_device(self._h, ctypes.byref(p), ctypes.byref(v)), "ylm_logits_device")
        return p.value, v.value

    # -- sampling
    def set_sampling(self, greedy: bool = True, top_k: int = 40, temperature: float = 0.6, seed: int = 0,
                     masked_ids: Optional[Sequence[int]] = None) -> None:
        s = Sampling()
        s.greedy = int(greedy)
        s.top_k = top_k
        s.temperature = temperature
        s.seed = seed
        self._masked = _i64(masked_ids if masked_ids is not None else [])
        s.masked_ids = _ptr(self._masked, ctypes.c_int64) if self._masked.size else None
        s.n_masked = self._masked.size
        check(lib().ylm_set_sampling(self._h, ctypes.byref(s)), "ylm_set_sampling")

    def set_draw(self, u: float) -> None:
        check(lib().ylm_set_draw(self._h, u), "ylm_set_draw")

    def sample(self, greedy: bool) -> int:
        out = ctypes.c_int64()
        check(lib().ylm_sample(self._h, int(greedy), ctypes.byref(out)), "ylm_sample")
        return out.value

    def decode(self, token: int, greedy: bool):
        out = ctypes.c_int64()
        st = lib().ylm_decode(self._h, int(token), int(greedy), ctypes.byref(out))
        if st not in GENERATION_ERRORS:
            check(st, "ylm_decode")
        return Status(st), out.value

    def last_topk(self):
        ids = np.zeros(64, np.int64)
        probs = np.zeros(64, np.float32)
        k = ctypes.c_int32()
        u = ctypes.c_float()
        check(lib().ylm_last_topk(self._h, _ptr(ids, ctypes.c_int64), _ptr(probs, ctypes.c_float), ctypes.byref(k),
                                  ctypes.byref(u)), "ylm_last_topk")
        return ids[:k.value], probs[:k.value], u.value

    def generate(self, prompt: Sequence[int], max_new: int, eos_ids: Sequence[int] = ()) -> dict:
        p = _i64(prompt)
        eos = _i64(list(eos_ids))
        out = np.zeros(max(1, max_new), np.int64)
        n = ctypes.c_int32()
        t_first = ctypes.c_double()
        t_dec = ctypes.c_double()
        st = lib().ylm_generate(self._h, _ptr(p, ctypes.c_int64), p.size, max_new,
                                _ptr(eos, ctypes.c_int64) if eos.size else None, eos.size,
                                _ptr(out, ctypes.c_int64), ctypes.byref(n), ctypes.byref(t_first), ctypes.byref(t_dec))
        if st not in GENERATION_ERRORS:
            check(st, "ylm_generate")
        return {"status": Status(st), "ids": out[:n.value].copy(), "first_token_ms": t_first.value,
                "decode_ms": t_dec.value}

    def info(self) -> dict:
        cap, last, mx = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        check(lib().ylm_info(self._h, ctypes.byref(cap), ctypes.byref(last), ctypes.byref(mx)), "ylm_info")
        return {"kv_capacity": cap.value, "last_kv_index": last.value, "max_seq_len": mx.value}

    def last_prefill_ms(self) -> float:
        ms = ctypes.c_double()
        check(lib().ylm_last_prefill_ms(self._h, ctypes.byref(ms)), "ylm_last_prefill_ms")
        return ms.value

    def time_decode(self, iters: int) -> float:
        ms = ctypes.c_double()
        st = lib().ylm_time_decode(self._h, iters, ctypes.byref(ms))
        check(st, "ylm_time_decode")
        return ms.value

    def time_segment(self, layer: int, iters: int):
        """(ms per launch, weight bytes) of one persistent GEMV segment."""
        ms, nb = ctypes.c_double(), ctypes.c_double()
        check(lib().ylm_time_segment(self._h, layer, iters, ctypes.byref(ms), ctypes.byref(nb)), "ylm_time_segment")
        return ms.value, nb.value

    def exchange_stats(self, reset: bool = False) -> dict:
        """Device time in the fused all-reduce exchanges (tensor parallel)."""
        w, n, t = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
        check(lib().ylm_exchange_stats(self._h, int(reset), ctypes.byref(w), ctypes.byref(n), ctypes.byref(t)),
              "ylm_exchange_stats")
        return {"wait_ms": w.value, "exchanges": n.value, "tokens": t.value}

    def reset_exchange_stats(self) -> None:
        self.exchange_stats(reset=True)

    def time_allreduce(self, iters: int) -> Optional[float]:
        """ms per decode step of the step's 2L NCCL all-reduces alone (None at tp = 1)."""
        ms = ctypes.c_double()
        st = lib().ylm_time_allreduce(self._h, iters, ctypes.byref(ms))
        if st == Status.UNSUPPORTED:
            return None
        check(st, "ylm_time_allreduce")
        return ms.value

    def debug_drop_output(self, layer: int) -> None:
        """Test support: the persistent path writes `layer`'s SwiGLU activation
        elsewhere, so the down projection's bounded wait expires (-1 restores)."""
        check(lib().ylm_debug_drop_output(self._h, layer), "ylm_debug_drop_output")

    def decode_persistent(self) -> bool:
        """True when decode steps run as one cooperative kernel."""
        v = ctypes.c_int32()
        check(lib().ylm_decode_path(self._h, ctypes.byref(v)), "ylm_decode_path")
        return bool(v.value)


class Model:
    """Static facade of the reference's Model (src/models/Model.cpp:10-53)."""

    _engine: Optional[Engine] = None

    @classmethod
    def Init(cls, snapshot_dir: Optional[str], config: ModelConfig, **options) -> None:
        if cls._engine is not None:
            cls._engine.close()
        cls._engine = Engine(snapshot_dir, config, **options)

    @classmethod
    def _ensure(cls) -> Engine:
        if cls._engine is None:
            raise RuntimeError("You must explicitly call Init() function at program startup once before "
                               "calling any other functions")
        return cls._engine

    @classmethod
    def BeginInfer(cls) -> None:
        cls._ensure().begin_infer()

    @classmethod
    def Infer(cls, tokenVectors: List[int], eosPerPrompt: List[int]) -> GenerationResult:
        e = cls._ensure()
        st, trimmed = e.infer(tokenVectors, eosPerPrompt)
        tokenVectors[:] = [int(t) for t in trimmed]
        if st != Status.OK:
            return GenerationResult(None, False, st)
        return GenerationResult(e.logits(), True, Status.OK)
