"""Sampling contract of the engine, restated on the CPU — TEST INFRASTRUCTURE ONLY.

Mirrors ``ChatSession::Sample`` (``src/ChatSession.cpp:560-593``) and the
first-token rule at ``ChatSession.cpp:140`` (the first generated token is
always greedy):

- greedy: ``argmax`` over the last-row logits, lowest index among ties;
- top-k: logits times ``1/temp`` rounded to FP16 (the working dtype),
  every masked special id set to ``-1e9`` (``-inf`` in FP16), the K largest
  values in descending order with ties broken by the lower index (what
  ``torch::topk`` returns sorted), softmax over them rounded to FP16, and a
  categorical draw. The reference draws with ``torch::multinomial``; the engine
  draws by inverse CDF from one uniform ``u`` per call (Philox4x32-10, see
  ``oracle.numerics``), so given the same logits and the same ``u`` the
  engine and this function pick the same id bit for bit.
"""
from __future__ import annotations

from typing import Iterable, Optional, Tuple

import numpy as np

from .numerics import F32, exp_rn, round_f16


def greedy(logits: np.ndarray) -> int:
    return int(np.argmax(np.asarray(logits, np.float32)))


def topk_candidates(logits: np.ndarray, k: int, temp: float,
                    masked: Optional[Iterable[int]] = None) -> Tuple[np.ndarray, np.ndarray]:
    """Scaled FP16 values and ids of the top-k, in sampling order."""
    inv_t = F32(1.0) / F32(temp)
    scaled = round_f16(np.asarray(logits, np.float32) * inv_t)
    if masked is not None:
        m = np.asarray(list(masked), dtype=np.int64)
        if m.size:
            scaled[m] = -np.inf
    idx = np.arange(scaled.shape[0], dtype=np.int64)
    order = np.lexsort((idx, -scaled))[:k]
    return scaled[order].astype(np.float32), order.astype(np.int64)


def topk_probs(vals: np.ndarray) -> np.ndarray:
    """Softmax over the sorted top-k values: exp_rn of (v - max), a sequential
    FP32 sum, an FP32 division, rounded to FP16."""
    with np.errstate(invalid="ignore"):
        d = (vals - vals[0]).astype(np.float32)
    d = np.where(np.isnan(d), np.float32(-np.inf), d)
    e = exp_rn(d)
    s = F32(0.0)
    for v in e:
        s = F32(s + v)
    return round_f16((e / s).astype(np.float32))


def draw(probs: np.ndarray, ids: np.ndarray, u: float) -> int:
    """Inverse-CDF pick: first i whose running FP32 sum exceeds u * total."""
    total = F32(0.0)
    for p in probs:
        total = F32(total + F32(p))
    target = F32(F32(u) * total)
    c = F32(0.0)
    last_pos = 0
    for i, p in enumerate(probs):
        if p > 0:
            last_pos = i
        c = F32(c + F32(p))
        if c > target:
            return int(ids[i])
    return int(ids[last_pos])


def sample_topk(logits: np.ndarray, k: int, temp: float, u: float,
                masked: Optional[Iterable[int]] = None) -> int:
    vals, ids = topk_candidates(logits, k, temp, masked)
    return draw(topk_probs(vals), ids, u)
