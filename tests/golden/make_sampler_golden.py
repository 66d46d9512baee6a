"""Generate the sampler fixtures in this directory from the reference's own ops.

``ChatSession::Sample`` (src/ChatSession.cpp:560-593) picks the next id with
LibTorch: ``argmax`` (greedy), or ``logits / Temp``, masked special ids set to
-1e9, ``torch::topk(K)``, ``torch::softmax`` and ``torch::multinomial``. The
harness mode ``ref_harness --sample-fixture`` (oracle/ref/ref_harness.cpp)
runs exactly those ops up to the draw on given FP16 logit rows. With the
LibTorch CUDA FP16 build (``oracle/_ref/ref_gpu_f16``, on a GPU) it gives what
the reference computes on the device; the CPU build gives LibTorch's CPU
kernels. The fixture stores, per parameter set and row, the argmax id, the
top-k ids in LibTorch's order, their FP16 values and their FP16 softmax
probabilities. The logit rows are not stored: ``logit_rows()`` regenerates them
from the counter-based generator in yalama_b200.synth, bit for bit.

    python tests/golden/make_sampler_golden.py --binary oracle/_ref/ref_gpu_f16 \
        --out tests/golden/sampler_torch_cuda.npz
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from yalama_b200 import synth  # noqa: E402

VOCAB = 128256
# masked special ids (ChatSession.cpp:41-61 builds the list from the tokenizer)
MASKED = [7, 128000, 128001, 128006, 128007, 128009, 100, 5000]
# (K, temperature)
PARAMS = [(40, 0.6), (64, 1.0), (5, 0.05), (2, 0.7), (1, 0.6)]


def _to_bf16_f16(a: np.ndarray) -> np.ndarray:
    """Round float32 to BF16 (nearest even), then hold it as FP16."""
    f = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((f + np.uint32(0x7FFF) + ((f >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)) << np.uint32(16)
    return r.view(np.float32).astype(np.float16)


def logit_rows() -> np.ndarray:
    """FP16 logit rows [R, VOCAB] with few, many and total ties."""
    rows = []
    for r in range(4):  # N(0, 2): few ties
        rows.append(synth.normal_values(17, f"sampler.row{r}", 0, VOCAB, 2.0))
    for r in range(4):  # the same through BF16 (the reference's storage type): heavy ties at the top
        v = synth.normal_values(19, f"sampler.bf{r}", 0, VOCAB, 3.0).astype(np.float32)
        rows.append(_to_bf16_f16(v))
    for r in range(2):  # multiples of 0.25: ties everywhere
        v = synth.normal_values(23, f"sampler.q{r}", 0, VOCAB, 1.5).astype(np.float32)
        rows.append((np.round(v * 4) / 4).astype(np.float16))
    rows.append(np.zeros(VOCAB, np.float16))  # all equal
    v = synth.normal_values(29, "sampler.masktop", 0, VOCAB, 2.0).astype(np.float32)
    v[MASKED] = 12.0  # the masked ids are the largest
    rows.append(v.astype(np.float16))
    return np.stack(rows)


def parse(path: str, n_rows: int, k: int) -> dict:
    raw = open(path, "rb").read()
    per = 8 + 8 * k + 2 * k + 2 * k
    assert len(raw) == per * n_rows, (len(raw), per, n_rows)
    g = np.zeros(n_rows, np.int64)
    ids = np.zeros((n_rows, k), np.int64)
    vals = np.zeros((n_rows, k), np.uint16)
    probs = np.zeros((n_rows, k), np.uint16)
    for r in range(n_rows):
        o = r * per
        g[r] = np.frombuffer(raw, np.int64, 1, o)[0]
        ids[r] = np.frombuffer(raw, np.int64, k, o + 8)
        vals[r] = np.frombuffer(raw, np.uint16, k, o + 8 + 8 * k)
        probs[r] = np.frombuffer(raw, np.uint16, k, o + 8 + 10 * k)
    return {"greedy": g, "ids": ids, "vals": vals, "probs": probs}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--binary", default=os.path.join(ROOT, "oracle", "_ref", "ref_gpu_f16"))
    ap.add_argument("--out", default=os.path.join(HERE, "sampler_torch_cuda.npz"))
    a = ap.parse_args()
    rows = logit_rows()
    out = {"params": np.array(PARAMS, dtype=np.float64), "masked": np.array(MASKED, np.int64),
           "vocab": np.int64(VOCAB), "binary": os.path.basename(a.binary)}
    with tempfile.TemporaryDirectory() as tmp:
        fin = os.path.join(tmp, "in.bin")
        with open(fin, "wb") as f:
            f.write(np.array([rows.shape[0], VOCAB], np.int64).tobytes())
            f.write(rows.view(np.uint16).tobytes())
        mask = os.path.join(tmp, "mask.bin")
        synth.write_ids(mask, MASKED)
        for i, (k, t) in enumerate(PARAMS):
            fout = os.path.join(tmp, f"out{i}.bin")
            r = subprocess.run([a.binary, "--sample-fixture", fin, fout, "--topk", str(k), "--temp", str(t),
                                "--mask", mask], capture_output=True, text=True, timeout=600)
            if r.returncode != 0:
                raise SystemExit(r.stderr[-2000:])
            res = parse(fout, rows.shape[0], k)
            for key, v in res.items():
                out[f"p{i}_{key}"] = v
    np.savez_compressed(a.out, **out)
    print(json.dumps({"out": a.out, "rows": int(rows.shape[0]), "params": PARAMS}))


if __name__ == "__main__":
    main()
