"""Numeric building blocks of the oracle — TEST INFRASTRUCTURE ONLY.

Rounding to the storage dtype mirrors LibTorch's behaviour for FP16/BF16
tensors: every elementwise op and every matmul computes in FP32 and rounds its
result to the storage dtype (the reference chains such ops, e.g.
``src/models/ModelBase.cpp:731-735``).

``exp_rn`` and ``philox4x32_10`` are the exact arithmetic the engine's sampler
kernel performs (same FP32 operations in the same order, no fused multiply-add),
so sampling can be compared bit for bit.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def round_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    f = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (f + np.uint32(0x7FFF) + ((f >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def round_f32(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


ROUNDERS = {"f16": round_f16, "bf16": round_bf16, "f32": round_f32}


# ---------------------------------------------------------------------------
# exp for the sampler's softmax: Cody-Waite range reduction (ln 2 split in two
# parts as in Cephes' expf: 0.693359375 and -2.12194440e-4) and the degree-7
# Taylor polynomial of e^r on |r| <= ln2/2, evaluated by Horner, every step a
# separately rounded FP32 operation. Inputs are <= 0 (logit minus the maximum).
# ---------------------------------------------------------------------------
_LOG2E = F32(1.44269504088896341)
_C1 = F32(0.693359375)
_C2 = F32(-2.12194440e-4)
_INV_FACT = [F32(1.0 / f) for f in (5040.0, 720.0, 120.0, 24.0, 6.0, 2.0, 1.0, 1.0)]


def exp_rn(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        n = np.rint(x * _LOG2E).astype(np.float32)
        r = (x - n * _C1).astype(np.float32)
        r = (r - n * _C2).astype(np.float32)
        p = _INV_FACT[0]
        for c in _INV_FACT[1:]:
            p = (p * r).astype(np.float32)
            p = (p + c).astype(np.float32)
        ni = np.clip(n, -126, 0).astype(np.int32)
        scale = ((ni + 127).astype(np.uint32) << np.uint32(23)).view(np.float32)
        out = (p * scale).astype(np.float32)
    return np.where(x < F32(-87.0), F32(0.0), out).astype(np.float32)


# ---------------------------------------------------------------------------
# Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy
# as 1, 2, 3", SC 2011). The sampler draws one uniform per sampling call:
# counter = (call index lo, hi, 0, 0), key = (seed lo, seed hi); word 0 of the
# output gives u = (2*(x0 >> 9) + 1) * 2^-24, exactly representable, in (0, 1).
# ---------------------------------------------------------------------------
_PH_M0 = 0xD2511F53
_PH_M1 = 0xCD9E8D57
_PH_W0 = 0x9E3779B9
_PH_W1 = 0xBB67AE85
_U32 = 0xFFFFFFFF


def philox4x32_10(counter, key):
    c = [int(v) & _U32 for v in counter]
    k0, k1 = int(key[0]) & _U32, int(key[1]) & _U32
    for rnd in range(10):
        p0 = _PH_M0 * c[0]
        p1 = _PH_M1 * c[2]
        hi0, lo0 = (p0 >> 32) & _U32, p0 & _U32
        hi1, lo1 = (p1 >> 32) & _U32, p1 & _U32
        c = [hi1 ^ c[1] ^ k0, lo1, hi0 ^ c[3] ^ k1, lo0]
        if rnd < 9:
            k0 = (k0 + _PH_W0) & _U32
            k1 = (k1 + _PH_W1) & _U32
    return c


def sampler_uniform(seed: int, call_index: int) -> np.float32:
    ctr = (call_index & _U32, (call_index >> 32) & _U32, 0, 0)
    key = (seed & _U32, (seed >> 32) & _U32)
    x0 = philox4x32_10(ctr, key)[0]
    return F32((2 * (x0 >> 9) + 1) * (2.0 ** -24))
