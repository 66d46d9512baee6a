#!/usr/bin/env python
"""Batch-1 FP16 decode benchmark of the yalama B200 engine.

Default workload (one "step" = one request): a Llama-3.1-8B-shaped FP16 model
(hidden 4096, 32 layers, 32 Q / 8 KV heads, head_dim 128, intermediate 14336,
vocab 128256, untied lm_head), random-init N(0, 0.02) weights from a seed, a
2048-token uniform-random prompt, then 1024 greedily generated tokens. Other
shapes run with ``--workload`` (see WORKLOADS). Synthetic data: no checkpoint or
dataset is read.

  value   decode tok/s with everything resident in HBM: the 1023 decode steps of
          each request run as back-to-back CUDA-graph launches (one graph per
          token: the whole forward + on-device sampling), timed with CUDA events
          on the engine stream; max over ranks.
  e2e     the same tok/s through the C ABI's token loop (ylm_generate) with
          host buffers: the prompt copied in from host memory and every token id
          read back to the host, timed per the reference's own definition
          ((generated - 1) / sum of per-token times).

At N > 1 the model is tensor-parallel over the N GPUs of the node (strong
scaling: the same request, split), and the line carries the per-token time
spent in the all-reduce exchanges. Weights (16 GB) far exceed the 126 MB L2, so
no flush is needed between timed steps. At N = 1 the line also carries the
Llama-3.2-3B top-k 40 / temperature 0.6 workload as an extra key.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--workload NAME]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# name -> (model preset, prompt tokens, generated tokens, top_k (0 = greedy), temperature,
#          KV cache GB: the reference's --kvcachesizeingb; its capacity rule (EnsureKVCapacity,
#          src/models/ModelBase.cpp:853-866) needs 3 GB for a 4096 + 512 request at 70B)
WORKLOADS = {
    "llama3.1-8b": ("llama3.1-8b", 2048, 1024, 0, 0.6, 2),
    "llama3.2-3b": ("llama3.2-3b", 512, 256, 40, 0.6, 2),
    "qwen3-0.6b": ("qwen3-0.6b", 32, 128, 0, 0.6, 2),
    "qwen2.5-7b": ("qwen2.5-7b", 8192, 512, 0, 0.6, 2),
    "mistral-7b-v0.3": ("mistral-7b-v0.3", 2048, 1024, 0, 0.6, 2),
    "llama3.1-70b": ("llama3.1-70b", 4096, 512, 0, 0.6, 3),
}
DEFAULT_WORKLOAD = "llama3.1-8b"
EXTRA_WORKLOAD = "llama3.2-3b"
SEEDS = {"weight_seed": 0, "prompt_seed": 0, "sample_seed": 1234}
METRIC = "batch-1 FP16 decode tok/s"
# the CPU reference runs a bounded sample: this many prompt tokens at most, then a few decode tokens
CPU_SAMPLE_PROMPT = 128
REF_CPU = os.path.join(ROOT, "oracle", "_ref", "ref_cpu_f32")
REF_GPU = os.path.join(ROOT, "oracle", "_ref", "ref_gpu_f16")
REF_GPU_BF16 = os.path.join(ROOT, "oracle", "_ref", "ref_gpu_bf16")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peaks():
    """Dense 16-bit tensor-core rate (TF/s): burst and sustained, measured with
    a cuBLAS bf16 GEMM on this kind of GPU (FP16 runs at the same dense rate)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        if d.get("bf16_tflops"):
            burst = float(d["bf16_tflops"])
            return burst, float(d.get("bf16_tflops_sustained") or burst), "measured"
    return 1590.0, 1400.0, "fallback"


def prefill_flops(spec, T):
    """Algorithmic FLOPs of one T-token prefill as the engine computes it: the
    four projections on every row, causal attention (QK^T and PV over keys
    0..i for query i) and the lm_head on the last row only."""
    H, D, I, V = spec.hidden, spec.head_dim, spec.intermediate, spec.vocab
    proj = H * (spec.heads + 2 * spec.kv_heads) * D + spec.heads * D * H + 3 * H * I
    attn = 4 * D * spec.heads * T * (T + 1) // 2
    return spec.layers * (2 * T * proj + attn) + 2 * V * H


def prefill_roofline(spec, T, tok_s, tp):
    burst, sustained, kind = tensor_peaks()
    fl = prefill_flops(spec, T) / tp
    achieved = fl * tok_s / T / 1e12
    return {"flops_per_prefill_per_gpu": fl, "achieved_tflops": achieved, "peak_tflops": burst,
            "frac": achieved / burst, "frac_of_sustained": achieved / sustained, "peak_kind": kind,
            "note": "FP16 tensor-core FLOPs (projections on all rows, causal attention, last-row lm_head) "
                    "over CUDA-event prefill time, against the cuBLAS bf16 burst rate (sustained beside it)"}


def profile_traffic(name):
    """traffic (bytes per launch) recorded from an ncu capture under profiles/."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


class Clocks:
    """nvidia-smi clock/throttle samples taken during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.f = None

    def start(self):
        try:
            self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.flush()
        rows = [l.strip().split(", ") for l in open(self.f.name) if l.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        load = [s for s in sm if mx and s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def args_():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", "--preset", dest="workload", default=DEFAULT_WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--prompt", type=int, default=0, help="override the workload's prompt length")
    ap.add_argument("--decode", type=int, default=0, help="override the workload's generated tokens")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the extra top-k workload at N = 1")
    ap.add_argument("--e2e-requests", type=int, default=2)
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (small cases for profiler captures; not a bench number)")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--decode-path", default="persistent", choices=["persistent", "per-op"],
                    help="persistent GEMV segments (default) or the per-op graph")
    ap.add_argument("--kernels", action="store_true",
                    help="time the prefill kernels alone (tcgen05 GEMM beside cuBLAS, causal attention) and exit")
    a = ap.parse_args()
    preset, prompt, decode, top_k, temp, kv_gb = WORKLOADS[a.workload]
    a.preset = preset
    a.kv_gb = kv_gb
    a.prompt = a.prompt or prompt
    a.decode = a.decode or decode
    a.top_k, a.temperature = top_k, temp
    return a


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def sampling_desc(top_k, temp):
    return "greedy" if top_k == 0 else f"top-k {top_k}, temperature {temp} (first token greedy)"


# ---------------------------------------------------------------- host resources
def host_mem_available():
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return None


def scratch_dir(need_bytes):
    """A folder with room for a snapshot of `need_bytes` (RAM-backed /dev/shm
    only when it leaves at least twice that in host memory)."""
    env = os.environ.get("YLM_BENCH_TMP")
    if env:
        return env
    mem = host_mem_available() or 0
    try:
        if shutil.disk_usage("/dev/shm").free > need_bytes * 1.2 and mem > need_bytes * 4:
            return "/dev/shm"
    except OSError:
        pass
    d = tempfile.gettempdir()
    if shutil.disk_usage(d).free < need_bytes * 1.2:
        raise RuntimeError(f"no room for a {need_bytes / 2**30:.1f} GiB snapshot in {d}")
    return d


def snapshot_bytes(spec, esize):
    return spec.n_params() * esize


# ---------------------------------------------------------------- reference runs
def write_snapshot(tmp, spec, dtype):
    from yalama_b200 import synth
    root = os.path.join(tmp, f"model_{dtype}")
    synth.write_snapshot(root, spec, seed=SEEDS["weight_seed"], dtype=dtype, fast=True)
    return root


def run_reference_binary(binary, root, prompt_file, n_decode, warmup, top_k, temp, threads=None, timeout=1800):
    cmd = [binary, "--model", root, "--prompt", prompt_file, "--decode", str(n_decode), "--warmup", str(warmup),
           "--topk", str(top_k), "--temp", str(temp), "--seed", str(SEEDS["sample_seed"])]
    if threads:
        cmd += ["--threads", str(threads)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"{os.path.basename(binary)} failed: {r.stderr[-400:]}")
    return json.loads(r.stdout.strip().splitlines()[-1])


def cpu_reference(spec, prompt_len, n_decode, warmup, top_k, temp):
    """The reference's own forward (LibTorch, CPU, FP32) on this host's cores,
    on a bounded sample: at most CPU_SAMPLE_PROMPT prompt tokens, then
    `warmup` untimed and `n_decode` timed decode tokens."""
    from yalama_b200 import synth
    threads = os.cpu_count() or 1
    p = min(prompt_len, CPU_SAMPLE_PROMPT)
    need = snapshot_bytes(spec, 4)
    mem = host_mem_available()
    if os.path.exists(REF_CPU):
        # the reference clones every tensor out of the mapped shard: the file's
        # pages plus a private copy must fit in host memory
        if mem is not None and mem < need * 2.5:
            raise RuntimeError(f"host memory {mem / 2**30:.0f} GiB < 2.5 x the {need / 2**30:.0f} GiB FP32 weights")
        with tempfile.TemporaryDirectory(dir=scratch_dir(need)) as tmp:
            pf = os.path.join(tmp, "prompt.bin")
            synth.write_ids(pf, synth.prompt_ids(SEEDS["prompt_seed"], p, spec.vocab))
            root = write_snapshot(tmp, spec, "F32")
            res = run_reference_binary(REF_CPU, root, pf, n_decode + warmup, warmup, top_k, temp, threads)
        kind = "reference"
    else:
        res = cpu_port(spec, p, n_decode, warmup)
        kind = "port"
    sample = (f"{res['timed_tokens']} timed decode tokens ({warmup} untimed) after a {p}-token prefill of the "
              f"same {spec.hidden}-wide {spec.layers}-layer model, {sampling_desc(top_k, temp)}, FP32; decode is "
              f"bound by the FP32 weight stream, which the shorter context leaves unchanged")
    return res, kind, threads, sample


def cpu_port(spec, prompt_len, n_decode, warmup):
    """Fallback when the reference binary is absent: the numpy restatement."""
    import numpy as np
    from yalama_b200 import synth
    from oracle.model import OracleModel
    rng = np.random.default_rng(SEEDS["weight_seed"])
    w = {n: (np.ones(s, np.float32) if n.endswith("norm.weight")
             else rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)) for n, s in spec.tensor_shapes()}
    m = OracleModel(spec, w, mode="f32")
    m.begin_infer()
    ids = synth.prompt_ids(SEEDS["prompt_seed"], prompt_len, spec.vocab)
    t0 = time.perf_counter()
    _, lg = m.infer(ids)
    first = time.perf_counter() - t0
    tt = 0.0
    for i in range(n_decode + warmup):
        t0 = time.perf_counter()
        _, lg = m.infer([int(np.argmax(lg))])
        if i >= warmup:
            tt += time.perf_counter() - t0
    return {"tokens_per_second": n_decode / tt, "first_token_s": first, "decode_s": tt, "timed_tokens": n_decode,
            "threads": os.cpu_count()}


def bench_reference(a):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from yalama_b200 import synth
    spec = synth.PRESETS[a.preset]
    try:
        res, kind, threads, sample = cpu_reference(spec, a.prompt, a.steps, a.warmup, a.top_k, a.temperature)
    except Exception as ex:
        print(json.dumps({"impl": "reference", "unavailable": f"reference CPU path could not run: {str(ex)[:200]}"}),
              flush=True)
        return
    v = res["tokens_per_second"]
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1000.0 / v if v else None,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, uniform-random prompt ids)",
            "config": {"workload": workload_desc(a, spec),
                       "path": "reference LibTorch CPU path (ModelBase::Infer + ChatSession::Sample)"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def workload_desc(a, spec):
    return (f"{a.preset}-shaped FP16{f' ({a.layers} layers)' if a.layers else ''}, batch 1, prompt {a.prompt}, "
            f"{a.decode} generated tokens, {sampling_desc(a.top_k, a.temperature)}"
            f"{f', KV cache {a.kv_gb} GB' if a.kv_gb != 2 else ''}")


def gpu_reference(spec, prompt, top_k, temp):
    """The reference's LibTorch CUDA builds on this GPU: FP16 (the storage type
    of this engine) and BF16 (the reference as shipped), 128 timed decode
    tokens after the full prompt, wall clock per token as ChatSession times it."""
    from yalama_b200 import synth
    out = {}
    need = snapshot_bytes(spec, 2)
    with tempfile.TemporaryDirectory(dir=scratch_dir(need * 2)) as tmp:
        pf = os.path.join(tmp, "prompt.bin")
        synth.write_ids(pf, prompt)
        for key, binary, dtype in (("reference_gpu_fp16", REF_GPU, "F16"), ("reference_gpu_bf16", REF_GPU_BF16, "BF16")):
            if not os.path.exists(binary):
                continue
            try:
                root = write_snapshot(tmp, spec, dtype)
                res = run_reference_binary(binary, root, pf, 128 + 4, 4, top_k, temp)
                shutil.rmtree(root, ignore_errors=True)
                out[key] = {"value": res["tokens_per_second"], "unit": "tok/s",
                            "first_token_ms": res["first_token_s"] * 1e3, "load_s": res.get("load_s"),
                            "sample": f"{res['timed_tokens']} decode tokens (4 untimed) after the {len(prompt)}-token "
                                      f"prefill, {sampling_desc(top_k, temp)}, LibTorch CUDA "
                                      f"{dtype} on this GPU (wall clock per token, as ChatSession times it)"}
            except Exception as ex:
                out[key] = {"value": None, "error": str(ex)[:300]}
    return out


# ---------------------------------------------------------------- host BPE encode
TOKENIZER_BENCH = os.path.join(ROOT, "yalama_b200", "host", "_build", "tokenizer_bench")


def host_bpe_encode(n_bytes=32000, n_merges=50000):
    """The prompt-encoding step before the token loop: a 32 KB Qwen-family
    prompt (one BPE piece) with a 50k-merge synthetic tokenizer, encoded by the
    reference's QwenTokenizer and by its FastBpe wrapper (ids compared), median
    wall time of each on one host core."""
    if not os.path.exists(TOKENIZER_BENCH):
        return {"value": None, "error": "tokenizer_bench not built (it needs the reference sources at build time)"}
    from yalama_b200 import synth
    with tempfile.TemporaryDirectory() as tmp:
        synth.write_bpe_tokenizer(tmp, "qwen", n_merges, seed=0)
        tp = os.path.join(tmp, "prompt.txt")
        with open(tp, "w", encoding="utf-8") as f:
            f.write(synth.bpe_text("qwen", n_bytes, seed=0))
        r = subprocess.run([TOKENIZER_BENCH, "--model", tmp, "--family", "qwen", "--text", tp, "--reps", "5",
                            "--ref-reps", "1"], capture_output=True, text=True, timeout=300)
    if r.returncode != 0:
        return {"value": None, "error": r.stderr[-300:]}
    res = json.loads(r.stdout.strip().splitlines()[-1])
    return {"value": res["fast_ms"], "unit": "ms", "reference_ms": res["ref_ms"], "tokens": res["tokens"],
            "ids_equal_reference": res["equal"],
            "sample": f"{res['bytes']}-byte synthetic prompt, {n_merges}-merge byte-level BPE, Qwen family "
                      "(whole text one piece), EncodeWithoutChatTemplate, BPE cache cleared per run"}


# ---------------------------------------------------------------- our engine
def segment_roofline(eng, spec, hbm_peak, peak_kind):
    """The dominant kernel of the persistent path: one decode GEMV segment (a
    middle layer's O, gate-up, down and the next layer's QKV) timed alone with
    CUDA events on the engine stream, back to back; its weights (436 MB for the
    8B shape) exceed L2, so every launch streams them from HBM. Algorithmic
    bytes = the segment's weights."""
    ms, wbytes = eng.time_segment(spec.layers // 2, 48)
    achieved = wbytes / (ms * 1e-3) / 1e9
    return {"kernel": "decode_segment_kernel (O + gate-up + down + next QKV of one layer, FP16)",
            "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "peak_kind": peak_kind, "traffic": profile_traffic(f"decode_segment_{spec_name(spec)}.txt"),
            "algorithmic_bytes": wbytes, "avg_launch_us": ms * 1e3}


def spec_name(spec):
    from yalama_b200 import synth
    for k, v in synth.PRESETS.items():
        if v.hidden == spec.hidden and v.vocab == spec.vocab and v.model_type == spec.model_type:
            return k
    return "custom"


def decode_bytes_per_token(spec, ctx, tp):
    """Weights + KV read per decode token per GPU (algorithmic)."""
    H, D, I, V = spec.hidden, spec.head_dim, spec.intermediate, spec.vocab
    per_layer = H * spec.heads * D + 2 * H * spec.kv_heads * D + spec.heads * D * H + 3 * H * I + 2 * H
    if spec.qkv_bias:
        per_layer += (spec.heads + 2 * spec.kv_heads) * D
    if spec.qk_norm:
        per_layer += 2 * D
    w = 2 * (spec.layers * per_layer + V * H + H)
    kv = 2 * spec.layers * spec.kv_heads * D * 2 * ctx
    return (w + kv) / tp


def run_workload(a, rank, world, local, pg, nccl_id, spec, steps, warmup, e2e_requests, with_roofline):
    """Time `steps` requests of the workload (after `warmup`); returns a dict of
    the measured numbers, identical on every rank (max over ranks)."""
    import torch
    from yalama_b200 import engine as E
    from yalama_b200 import synth

    cfg = E.config_from_spec(spec)
    eng = E.Engine(None, cfg, nccl_id=nccl_id, device=local, tp_rank=rank, tp_size=world,
                   init_seed=SEEDS["weight_seed"], decode_persistent=int(a.decode_path == "persistent"),
                   kv_cache_gb=a.kv_gb)
    greedy = a.top_k == 0
    eng.set_sampling(greedy=greedy, top_k=a.top_k or 40, temperature=a.temperature, seed=SEEDS["sample_seed"])
    prompt = synth.prompt_ids(SEEDS["prompt_seed"], a.prompt, spec.vocab)
    n_dec = a.decode - 1

    def request():
        eng.begin_infer()
        st, _ = eng.infer(prompt)
        assert st == E.Status.OK, st
        pf = eng.last_prefill_ms()
        eng.sample(True)
        ms = eng.time_decode(n_dec)
        return pf, ms * n_dec

    def barrier():
        if pg:
            pg.barrier()
        torch.cuda.synchronize()

    for _ in range(warmup):
        request()
    barrier()
    clocks = Clocks(local)
    clocks.start()
    t_wall = time.perf_counter()
    pf_ms, dec_ms = 0.0, 0.0
    eng.reset_exchange_stats()
    for _ in range(steps):
        p, d = request()
        pf_ms += p
        dec_ms += d
    barrier()
    wall = time.perf_counter() - t_wall
    clk = clocks.stop()
    xstats = eng.exchange_stats()
    tm = torch.tensor([pf_ms, dec_ms, xstats["wait_ms"], xstats["tokens"]], dtype=torch.float64)
    if pg:
        pg.all_reduce(tm, op=pg.ReduceOp.MAX)
    pf_ms, dec_ms = float(tm[0]), float(tm[1])
    r = {"value": steps * n_dec / (dec_ms / 1e3), "prefill_tok_s": steps * a.prompt / (pf_ms / 1e3),
         "ms_per_step": (pf_ms + dec_ms) / steps, "ms_per_token": dec_ms / (steps * n_dec), "wall": wall,
         "clocks": clk, "persistent": eng.decode_persistent()}
    if world > 1:
        r["exchange_wait_ms_per_token"] = float(tm[2]) / max(1.0, float(tm[3]))

    e2e_tps = []
    for _ in range(e2e_requests):
        barrier()
        g = eng.generate(prompt, a.decode, eos_ids=[])
        n = len(g["ids"])
        t = torch.tensor([g["decode_ms"]], dtype=torch.float64)
        if pg:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_tps.append((n - 1) / (float(t[0]) / 1e3))
    r["e2e"] = statistics.median(e2e_tps) if e2e_tps else None
    if world > 1:
        r["allreduce_nccl_ms_per_token"] = eng.time_allreduce(32)
    if with_roofline and r["persistent"] and world == 1:
        r["roofline"] = segment_roofline(eng, spec, *peaks())
    eng.close()
    del eng
    return r


def bench_ours(a):
    import torch
    from yalama_b200 import tp as TP
    from yalama_b200 import synth

    rank, world, local = dist_env()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    pg = None
    nccl_id = None
    if world > 1:
        import torch.distributed as dist
        import datetime
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        pg = dist
        nccl_id = TP.share_nccl_id(pg, rank)
    spec = synth.PRESETS[a.preset]
    if a.layers:
        import dataclasses
        spec = dataclasses.replace(spec, layers=a.layers)

    r = run_workload(a, rank, world, local, pg, nccl_id, spec, a.steps, a.warmup, a.e2e_requests,
                     not a.no_roofline)
    hbm, peak_kind = peaks()
    ctx = a.prompt + a.decode // 2
    bpt = decode_bytes_per_token(spec, ctx, world)
    ms_tok = r["ms_per_token"]
    step_roof = {"bytes_per_token_per_gpu": bpt, "mean_context": ctx, "ms_per_token": ms_tok,
                 "achieved_gbs": bpt / (ms_tok * 1e-3) / 1e9, "peak_gbs": hbm,
                 "frac": bpt / (ms_tok * 1e-3) / 1e9 / hbm, "frac_of_8000": bpt / (ms_tok * 1e-3) / 1e9 / 8000.0,
                 "peak_kind": peak_kind}

    extra = None
    if world == 1 and not a.no_extra and not a.layers and a.workload != EXTRA_WORKLOAD:
        b = argparse.Namespace(**vars(a))
        b.preset, b.prompt, b.decode, b.top_k, b.temperature, b.kv_gb = WORKLOADS[EXTRA_WORKLOAD]
        espec = synth.PRESETS[b.preset]
        er = run_workload(b, rank, world, local, pg, nccl_id, espec, 2, 1, 1, False)
        ebpt = decode_bytes_per_token(espec, b.prompt + b.decode // 2, 1)
        extra = {"workload": workload_desc(b, espec), "value": er["value"], "unit": "tok/s",
                 "ms_per_token": er["ms_per_token"], "prefill_tok_s": er["prefill_tok_s"],
                 "decode_roofline_frac": ebpt / (er["ms_per_token"] * 1e-3) / 1e9 / hbm,
                 "prefill_roofline_frac": prefill_roofline(espec, b.prompt, er["prefill_tok_s"], 1)["frac"],
                 "e2e": er["e2e"], "steps": 2, "warmup": 1}

    if rank != 0:
        if pg:
            pg.barrier()
        return
    # decode launches per token: persistent path = one GEMV segment per layer
    # plus one, attention per layer, and a sampler launch only for top-k (a
    # greedy pick runs in the lm_head epilogue); per-op graph = QKV, attention,
    # O, gate-up, down per layer (+ residual adds with tensor parallelism),
    # lm_head, sampler; NCCL's all-reduce / all-gather kernels are not counted
    if r["persistent"]:
        launches_per_token = 2 * spec.layers + 1 + (1 if a.top_k else 0)
    else:
        launches_per_token = spec.layers * (5 if world == 1 else 7) + 2
    n_dec = a.decode - 1
    prefill_launches = 1 + spec.layers * 8 + 1
    gpu_launches = a.steps * (prefill_launches + 1 + n_dec * launches_per_token)
    calls = 2 + (a.decode - 1)
    h2d = a.prompt * 8 + 64 * calls
    d2h = 64 * calls
    line = {"metric": METRIC, "value": r["value"], "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random-init N(0,0.02) weights, uniform-random prompt ids)",
            "config": {"workload": workload_desc(a, spec), "parallelism": f"tp{world}",
                       "decode_path": "persistent GEMV segments" if r["persistent"] else "per-op graph",
                       "l2": f"weights {bpt * world / 1e9:.1f} GB >> 126 MB L2 (no flush needed)",
                       "timing": "CUDA events on the engine stream; value = decode tokens / decode time"},
            "prefill_tok_s": r["prefill_tok_s"],
            "prefill_roofline": prefill_roofline(spec, a.prompt, r["prefill_tok_s"], world),
            "decode_roofline": step_roof, "roofline": r.get("roofline"),
            "e2e": {"value": r["e2e"], "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "ylm_generate (C ABI), host prompt in, host ids out, per-token sync"},
            "gpu_launches": gpu_launches, "wall_s_timed": r["wall"], "clocks": r["clocks"]}
    if world > 1:
        line["allreduce"] = {
            "exchange_wait_ms_per_token": r["exchange_wait_ms_per_token"],
            "nccl_ms_per_token": r["allreduce_nccl_ms_per_token"],
            "count_per_token": 2 * spec.layers, "bytes_each": spec.hidden * 2,
            "note": "exchange_wait: device time (%globaltimer) from a segment's first partial store to the "
                    "arrival of every peer's partials, summed over the step's exchanges (block 0); nccl: "
                    "2L back-to-back NCCL all-reduces of [hidden] FP16 in a CUDA graph on the same ranks"}
    if extra:
        line["extra_" + EXTRA_WORKLOAD.replace(".", "_").replace("-", "_")] = extra
    if world == 1 and not a.no_cpu_baseline:
        try:
            res, kind, threads, sample = cpu_reference(spec, a.prompt, 4, 1, a.top_k, a.temperature)
            line["cpu_baseline"] = {"value": res["tokens_per_second"], "unit": "tok/s", "cores": threads,
                                    "kind": kind, "sample": sample}
        except Exception as ex:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": str(ex)[:300]}
    if world == 1 and not a.layers:
        line["host_bpe_encode"] = host_bpe_encode()
    if world == 1 and not a.no_ref_gpu and not a.layers:
        from yalama_b200 import synth as sy
        try:
            line.update(gpu_reference(spec, sy.prompt_ids(SEEDS["prompt_seed"], a.prompt, spec.vocab), a.top_k,
                                      a.temperature))
        except Exception as ex:
            line["reference_gpu_fp16"] = {"value": None, "error": str(ex)[:300]}
    print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()


# ---------------------------------------------------------------- prefill kernels alone
GEMM_SHAPES = [(2048, 6144, 4096), (2048, 4096, 4096), (2048, 28672, 4096), (2048, 4096, 14336), (8192, 4608, 3584),
               (512, 16384, 3072)]
ATTN_SHAPES = [(2048, 32, 8), (8192, 28, 4), (512, 24, 8)]


def bench_kernels():
    """The prefill kernels through their C-ABI entry points on random FP16
    inputs, CUDA events on the launching stream, after 3 warm-up launches: the
    tcgen05 GEMM (ylm_k_gemm) at the Llama-3.1-8B, Qwen2.5-7B and Llama-3.2-3B
    projection shapes beside cuBLAS (torch.matmul, the same FP16 operands), and
    the causal attention (ylm_k_prefill_attention, tcgen05 and mma.sync). Order
    of attention launches: per shape 3 + 10 tcgen05, then 3 + 10 mma.sync."""
    import torch
    from yalama_b200 import engine as E
    L = E.lib()
    st = lambda: ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())

    def timed(fn, n):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    out = {"attention": [], "gemm": []}
    for T, hq, hkv in ATTN_SHAPES:
        q = torch.randn(T, hq * 128, device="cuda", dtype=torch.float16)
        kc = torch.randn(hkv, T, 128, device="cuda", dtype=torch.float16)
        vc = torch.randn(hkv, T, 128, device="cuda", dtype=torch.float16)
        o = torch.empty(T, hq * 128, device="cuda", dtype=torch.float16)
        flops = 4 * hq * 128 * T * T / 2
        row = {"T": T, "hq": hq, "hkv": hkv}
        for name, tc in (("tcgen05", 1), ("mma_sync", 0)):
            ms = timed(lambda: E.check(L.ylm_k_prefill_attention(ptr(q), ptr(kc), ptr(vc), T, hq, hkv, T, ptr(o), tc,
                                                                 st()), "attention"), 10)
            row[name + "_tflops"] = round(flops / (ms * 1e-3) / 1e12, 1)
        out["attention"].append(row)
    for T, N, K in GEMM_SHAPES:
        a = torch.randn(T, K, device="cuda", dtype=torch.float16) * 0.1
        w = torch.randn(N, K, device="cuda", dtype=torch.float16) * 0.1
        c = torch.empty(T, N, device="cuda", dtype=torch.float16)
        t_own = timed(lambda: E.check(L.ylm_k_gemm(ptr(a), ptr(w), T, N, K, ptr(c), 1, st()), "gemm"), 20)
        t_lib = timed(lambda: torch.matmul(a, w.t()), 20)
        f = 2 * T * N * K
        out["gemm"].append({"T": T, "N": N, "K": K, "tcgen05_tflops": round(f / (t_own * 1e-3) / 1e12, 1),
                            "cublas_tflops": round(f / (t_lib * 1e-3) / 1e12, 1)})
    print(json.dumps({"kernels": out, "unit": "TFLOP/s (FP16 in, FP32 accumulate)",
                      "timing": "CUDA events, 3 warm-up launches, mean of 10 (attention) / 20 (GEMM)"}), flush=True)


def main():
    a = args_()
    if a.kernels:
        bench_kernels()
        return
    if a.impl == "reference":
        bench_reference(a)
    else:
        bench_ours(a)


if __name__ == "__main__":
    main()
