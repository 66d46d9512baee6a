"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference's own model code, compiled for CPU/FP32 by
``oracle/ref/Makefile`` (``oracle/_ref/ref_cpu_f32``), on small seeded
random-init models written by ``yalama_b200.synth`` and stores, per case, the
last-row logits of every step and the greedy ids it chose. Needs the reference
sources to build the binary (``make -C oracle/ref``); the fixtures it writes
are committed so the tests need neither.

    python tests/golden/make_golden.py [--ref oracle/_ref/ref_cpu_f32]
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
sys.path.insert(0, ROOT)

from yalama_b200 import synth  # noqa: E402

# name -> (spec kwargs, prompt length, decode steps, harness flags)
CASES = {
    # Qwen3 family: per-head q/k RMSNorm, tied embeddings, Hq*D != hidden
    "qwen3_tiny": (dict(model_type="qwen3"), 16, 6, []),
    # Qwen2.5 family: q/k/v biases, untied lm_head
    "qwen2_tiny": (dict(model_type="qwen2", tied=False), 16, 6, []),
    # Llama family: llama3 rope_scaling present in config.json (the reference ignores it)
    "llama_tiny": (dict(model_type="llama", tied=False, rope_theta=5e5, heads=8, kv_heads=2,
                        rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                                      "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}),
                   24, 6, []),
    # Mistral family, MHA-like grouping (Hq == Hkv)
    "mistral_tiny": (dict(model_type="mistral", tied=False, heads=2, kv_heads=2), 8, 4, []),
    # KV cache disabled: every call recomputes the whole sequence with a causal mask
    "qwen3_nokv": (dict(model_type="qwen3"), 8, 4, ["--nokv"]),
    # one-token prompt: the decode branch is never entered (last stays 0)
    "llama_prompt1": (dict(model_type="llama", tied=True), 1, 4, []),
    # sequence longer than max_position_embeddings (512, the smallest the reference
    # accepts, ModelBase.cpp:330-332) without a KV cache: left trim one token per step
    "qwen2_trim": (dict(model_type="qwen2", max_pos=512), 508, 8, ["--nokv"]),
    # KV capacity: 64 layers x 8 KV heads -> cap = 2^30/(8*128*2)/64/2 = 4096 slots;
    # prefill 2048 leaves last=2047, decode 1 fits (2048 <= 4096-2047), decode 2 fails
    "llama_kvcap": (dict(model_type="llama", layers=64, hidden=128, heads=8, kv_heads=8,
                         intermediate=128, vocab=256, tied=True), 2048, 3, ["--kvgb", "1"]),
}


def run_case(ref: str, name: str, work: str) -> dict:
    kw, n_prompt, n_decode, flags = CASES[name]
    spec = synth.tiny_spec(**kw)
    root = os.path.join(work, name)
    synth.write_snapshot(root, spec, seed=0, dtype="F32")
    prompt = synth.prompt_ids(0, n_prompt, spec.vocab)
    pfile = os.path.join(work, name + "_prompt.bin")
    synth.write_ids(pfile, prompt)
    out = os.path.join(work, name + "_out.bin")
    cmd = [ref, "--model", root, "--prompt", pfile, "--decode", str(n_decode), "--out", out,
           "--threads", "4"] + (flags if "--kvgb" in flags else flags + ["--kvgb", "1"])
    res = subprocess.run(cmd, capture_output=True, text=True, check=True)
    summary = json.loads(res.stdout.strip().splitlines()[-1])
    rows, ids = [], []
    with open(out, "rb") as f:
        while True:
            b = f.read(8)
            if not b:
                break
            v = int(np.frombuffer(b, np.int64)[0])
            rows.append(np.frombuffer(f.read(4 * v), np.float32).copy())
            ids.append(int(np.frombuffer(f.read(8), np.int64)[0]))
    np.savez_compressed(
        os.path.join(HERE, name + ".npz"),
        logits=np.stack(rows) if rows else np.zeros((0, spec.vocab), np.float32),
        ids=np.asarray(ids, np.int64),
        prompt=prompt,
        error=np.int64(summary["error"]),
        spec=json.dumps({k: v for k, v in kw.items()}),
        flags=json.dumps(flags),
    )
    return {"case": name, "steps": len(ids), "error": summary["error"]}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.path.join(ROOT, "oracle", "_ref", "ref_cpu_f32"))
    ap.add_argument("--cases", nargs="*", default=list(CASES))
    a = ap.parse_args()
    with tempfile.TemporaryDirectory() as work:
        for name in a.cases:
            print(run_case(a.ref, name, work))


if __name__ == "__main__":
    main()
