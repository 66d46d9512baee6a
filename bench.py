#!/usr/bin/env python
"""Batch-1 FP16 decode benchmark of the yalama B200 engine.

Workload (one "step" = one request): a Llama-3.2-3B-shaped FP16 model
(hidden 3072, 28 layers, 24 Q / 8 KV heads, head_dim 128, intermediate 8192,
vocab 128256, tied embeddings), random-init N(0, 0.02) weights from a seed,
a 512-token uniform-random prompt, then 256 generated tokens with top-k 40 and
temperature 0.6 (the first token greedy, as the reference's token loop does).
Synthetic data: no checkpoint or dataset is read.

  value   decode tok/s with everything resident in HBM: the 255 decode steps of
          each request run as back-to-back CUDA-graph launches (one graph per
          token: the whole forward + on-device sampling), timed with CUDA events
          on the engine stream; max over ranks.
  e2e     the same tok/s through the C ABI's token loop (ylm_generate) with
          host buffers: the prompt copied in from host memory and every token id
          read back to the host, timed per the reference's own definition
          ((generated - 1) / sum of per-token times).

At N > 1 the model is tensor-parallel over the N GPUs of the node (strong
scaling: the same request, split). Weights (6.4 GB) far exceed the 126 MB L2,
so no flush is needed between timed steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = {"preset": "llama3.2-3b", "prompt": 512, "decode": 256, "top_k": 40, "temperature": 0.6,
            "weight_seed": 0, "prompt_seed": 0, "sample_seed": 1234}
METRIC = "batch-1 FP16 decode tok/s"
REF_CPU = os.path.join(ROOT, "oracle", "_ref", "ref_cpu_f32")
REF_GPU = os.path.join(ROOT, "oracle", "_ref", "ref_gpu_f16")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


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
    ap.add_argument("--preset", default=WORKLOAD["preset"])
    ap.add_argument("--prompt", type=int, default=WORKLOAD["prompt"])
    ap.add_argument("--decode", type=int, default=WORKLOAD["decode"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true")
    ap.add_argument("--e2e-requests", type=int, default=2)
    ap.add_argument("--layers", type=int, default=0,
                    help="override the layer count (small cases for profiler captures; not a bench number)")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--decode-path", default="persistent", choices=["persistent", "per-op"],
                    help="persistent GEMV segments (default) or the per-op graph")
    return ap.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# ---------------------------------------------------------------- reference runs
def write_snapshot(tmp, spec, dtype):
    from yalama_b200 import synth
    root = os.path.join(tmp, f"model_{dtype}")
    synth.write_snapshot(root, spec, seed=WORKLOAD["weight_seed"], dtype=dtype, fast=True)
    return root


def run_reference_binary(binary, root, prompt_file, n_decode, warmup, threads=None, timeout=1800):
    cmd = [binary, "--model", root, "--prompt", prompt_file, "--decode", str(n_decode), "--warmup", str(warmup),
           "--topk", str(WORKLOAD["top_k"]), "--temp", str(WORKLOAD["temperature"]), "--seed",
           str(WORKLOAD["sample_seed"])]
    if threads:
        cmd += ["--threads", str(threads)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    if r.returncode != 0:
        raise RuntimeError(f"{os.path.basename(binary)} failed: {r.stderr[-400:]}")
    return json.loads(r.stdout.strip().splitlines()[-1])


def cpu_reference(spec, n_decode, warmup):
    """The reference's own forward (LibTorch, CPU, FP32) on this host's cores."""
    from yalama_b200 import synth
    threads = os.cpu_count() or 1
    with tempfile.TemporaryDirectory(dir=os.environ.get("YLM_BENCH_TMP")) as tmp:
        pf = os.path.join(tmp, "prompt.bin")
        synth.write_ids(pf, synth.prompt_ids(WORKLOAD["prompt_seed"], WORKLOAD["prompt"], spec.vocab))
        if os.path.exists(REF_CPU):
            root = write_snapshot(tmp, spec, "F32")
            res = run_reference_binary(REF_CPU, root, pf, n_decode + warmup, warmup, threads)
            kind = "reference"
        else:
            res = cpu_port(spec, n_decode, warmup)
            kind = "port"
    return res, kind, threads


def cpu_port(spec, n_decode, warmup):
    """Fallback when the reference binary is absent: the numpy restatement."""
    import numpy as np
    from yalama_b200 import synth
    from oracle.model import OracleModel
    rng = np.random.default_rng(WORKLOAD["weight_seed"])
    w = {n: (np.ones(s, np.float32) if n.endswith("norm.weight")
             else rng.standard_normal(s, dtype=np.float32) * np.float32(0.02)) for n, s in spec.tensor_shapes()}
    m = OracleModel(spec, w, mode="f32")
    m.begin_infer()
    ids = synth.prompt_ids(WORKLOAD["prompt_seed"], WORKLOAD["prompt"], spec.vocab)
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
    res, kind, threads = cpu_reference(spec, a.steps, a.warmup)
    v = res["tokens_per_second"]
    sample = (f"{res['timed_tokens']} decode tokens after a {WORKLOAD['prompt']}-token prefill "
              f"({a.warmup} untimed warm-up tokens), top-k 40 / temperature 0.6, FP32")
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "tok/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1000.0 / v if v else None,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random-init weights, uniform-random prompt ids)",
            "config": {"workload": f"{a.preset} batch-1 decode, prompt {WORKLOAD['prompt']}, top-k 40, temp 0.6",
                       "path": "reference LibTorch CPU path (ModelBase::Infer + ChatSession::Sample)"},
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- our engine
def gemv_roofline(spec, hbm_peak, peak_kind):
    """The dominant kernel (gate-up GEMV, [2I, H]) timed alone with CUDA events on
    the launching stream; 4 weight copies rotate so every launch streams from HBM."""
    import numpy as np
    import torch
    from yalama_b200 import engine as E
    n, k = 2 * spec.intermediate, spec.hidden
    ws = [(torch.randn(n, k, device="cuda", dtype=torch.float16) * 0.02) for _ in range(4)]
    x = torch.randn(k, device="cuda", dtype=torch.float16)
    y = torch.empty(n, device="cuda", dtype=torch.float16)
    s = torch.cuda.current_stream()
    sp = ctypes.c_void_p(s.cuda_stream)
    L = E.lib()
    for i in range(8):
        E.check(L.ylm_k_gemv(ctypes.c_void_p(ws[i % 4].data_ptr()), n, k, ctypes.c_void_p(x.data_ptr()),
                             ctypes.c_void_p(y.data_ptr()), sp), "gemv")
    iters = 64
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda._sleep(1000000)  # keep the stream busy while the launches are queued
    a.record(s)
    for i in range(iters):
        L.ylm_k_gemv(ctypes.c_void_p(ws[i % 4].data_ptr()), n, k, ctypes.c_void_p(x.data_ptr()),
                     ctypes.c_void_p(y.data_ptr()), sp)
    b.record(s)
    b.synchronize()
    ms = a.elapsed_time(b) / iters
    alg = n * k * 2 + k * 2 + n * 2
    achieved = alg / (ms * 1e-3) / 1e9
    del ws
    return {"kernel": f"gemv_kernel (gate-up shape {n}x{k}, FP16)", "bound": "hbm", "achieved": achieved,
            "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak, "peak_kind": peak_kind,
            "traffic": profile_traffic("gemv_gateup_llama3.2-3b.txt"), "algorithmic_bytes": alg,
            "avg_launch_us": ms * 1e3}


def segment_roofline(eng, spec, hbm_peak, peak_kind):
    """The dominant kernel of the persistent path: one decode GEMV segment (a
    middle layer's O, gate-up, down and the next layer's QKV, one cooperative
    launch) timed alone with CUDA events on the engine stream, back to back;
    its weights (201 MB for the 3B shape) exceed L2, so every launch streams
    them from HBM. Algorithmic bytes = the segment's weights."""
    ms, wbytes = eng.time_segment(spec.layers // 2, 48)
    achieved = wbytes / (ms * 1e-3) / 1e9
    return {"kernel": "decode_segment_kernel (O + gate-up + down + next QKV of one layer, FP16)",
            "bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "peak_kind": peak_kind, "traffic": profile_traffic("decode_segment_llama3.2-3b.txt"),
            "algorithmic_bytes": wbytes, "avg_launch_us": ms * 1e3}


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


def bench_ours(a):
    import numpy as np
    import torch
    from yalama_b200 import engine as E
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
    cfg = E.config_from_spec(spec)
    eng = E.Engine(None, cfg, nccl_id=nccl_id, device=local, tp_rank=rank, tp_size=world,
                   init_seed=WORKLOAD["weight_seed"], decode_persistent=int(a.decode_path == "persistent"))
    eng.set_sampling(greedy=False, top_k=WORKLOAD["top_k"], temperature=WORKLOAD["temperature"],
                     seed=WORKLOAD["sample_seed"])
    prompt = synth.prompt_ids(WORKLOAD["prompt_seed"], a.prompt, spec.vocab)
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

    for _ in range(a.warmup):
        request()
    barrier()
    clocks = Clocks(local)
    clocks.start()
    t_wall = time.perf_counter()
    pf_ms, dec_ms = 0.0, 0.0
    for _ in range(a.steps):
        p, d = request()
        pf_ms += p
        dec_ms += d
    barrier()
    wall = time.perf_counter() - t_wall
    clk = clocks.stop()
    tm = torch.tensor([pf_ms, dec_ms], dtype=torch.float64)
    if pg:
        pg.all_reduce(tm, op=pg.ReduceOp.MAX)
    pf_ms, dec_ms = float(tm[0]), float(tm[1])
    value = a.steps * n_dec / (dec_ms / 1e3)
    prefill_tps = a.steps * a.prompt / (pf_ms / 1e3)

    # e2e: the C-ABI token loop with host buffers
    e2e_tps = []
    for _ in range(a.e2e_requests):
        barrier()
        r = eng.generate(prompt, a.decode, eos_ids=[])
        n = len(r["ids"])
        t = torch.tensor([r["decode_ms"]], dtype=torch.float64)
        if pg:
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
        e2e_tps.append((n - 1) / (float(t[0]) / 1e3))
    e2e_v = statistics.median(e2e_tps) if e2e_tps else None
    # bytes crossing the host boundary per request: prompt in, 64-byte step state in/out per call
    calls = 2 + (a.decode - 1)
    h2d = a.prompt * 8 + 64 * calls
    d2h = 64 * calls

    hbm, peak_kind = peaks()
    ctx = a.prompt + a.decode // 2
    bpt = decode_bytes_per_token(spec, ctx, world)
    ms_tok = dec_ms / (a.steps * n_dec)
    persistent = eng.decode_persistent()
    seg_roof = None
    if persistent and world == 1 and not a.no_roofline:
        seg_roof = segment_roofline(eng, spec, *peaks())
    step_roof = {"bytes_per_token_per_gpu": bpt, "ms_per_token": ms_tok,
                 "achieved_gbs": bpt / (ms_tok * 1e-3) / 1e9, "peak_gbs": hbm,
                 "frac": bpt / (ms_tok * 1e-3) / 1e9 / hbm, "frac_of_8000": bpt / (ms_tok * 1e-3) / 1e9 / 8000.0,
                 "peak_kind": peak_kind}
    eng.close()
    del eng

    if rank != 0:
        if pg:
            pg.barrier()
        return
    roof = seg_roof
    if roof is None and world == 1 and not a.no_roofline:
        roof = gemv_roofline(spec, hbm, peak_kind)
    # decode launches per token: persistent path = one GEMV segment per layer
    # plus one, attention per layer, sampler; per-op graph = QKV, attention,
    # O, gate-up, down per layer (+ residual adds with tensor parallelism),
    # lm_head, sampler; NCCL's all-reduce / all-gather kernels are not counted
    if persistent:
        launches_per_token = 2 * spec.layers + 2
    else:
        launches_per_token = spec.layers * (5 if world == 1 else 7) + 2
    prefill_launches = 1 + spec.layers * 8 + 1
    gpu_launches = a.steps * (prefill_launches + 1 + n_dec * launches_per_token)
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": (pf_ms + dec_ms) / a.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded random-init N(0,0.02) weights, uniform-random prompt ids)",
            "config": {"workload": f"{a.preset}-shaped FP16{f' ({a.layers} layers)' if a.layers else ''}, batch 1, prompt {a.prompt}, {a.decode} generated tokens, "
                                   f"top-k {WORKLOAD['top_k']}, temperature {WORKLOAD['temperature']}",
                       "parallelism": f"tp{world}", "decode_path": "persistent GEMV segments" if persistent else "per-op graph",
                       "l2": "weights 6.4 GB >> 126 MB L2 (no flush needed)",
                       "timing": "CUDA events on the engine stream; value = decode tokens / decode time"},
            "prefill_tok_s": prefill_tps, "decode_roofline": step_roof, "roofline": roof,
            "e2e": {"value": e2e_v, "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "ylm_generate (C ABI), host prompt in, host ids out, per-token sync"},
            "gpu_launches": gpu_launches, "wall_s_timed": wall, "clocks": clk}
    if world == 1 and not a.no_cpu_baseline:
        try:
            res, kind, threads = cpu_reference(spec, 4, 1)
            line["cpu_baseline"] = {"value": res["tokens_per_second"], "unit": "tok/s", "cores": threads,
                                    "kind": kind,
                                    "sample": f"{res['timed_tokens']} decode tokens after a {a.prompt}-token "
                                              f"prefill (1 warm-up token), FP32, same model shape"}
        except Exception as ex:  # the baseline is reported, never required
            line["cpu_baseline"] = {"value": None, "error": str(ex)[:300]}
    if world == 1 and not a.no_ref_gpu and os.path.exists(REF_GPU):
        try:
            from yalama_b200 import synth as sy
            with tempfile.TemporaryDirectory(dir=os.environ.get("YLM_BENCH_TMP")) as tmp:
                pf = os.path.join(tmp, "prompt.bin")
                sy.write_ids(pf, prompt)
                root = write_snapshot(tmp, spec, "F16")
                res = run_reference_binary(REF_GPU, root, pf, 32 + 3, 3)
            line["reference_gpu_fp16"] = {"value": res["tokens_per_second"], "unit": "tok/s",
                                          "first_token_ms": res["first_token_s"] * 1e3,
                                          "sample": "32 decode tokens after the 512-token prefill, top-k 40, "
                                                    "LibTorch CUDA FP16 on this GPU (wall clock per token)"}
        except Exception as ex:
            line["reference_gpu_fp16"] = {"value": None, "error": str(ex)[:300]}
    print(json.dumps(line), flush=True)
    if pg:
        pg.barrier()


def main():
    a = args_()
    if a.impl == "reference":
        bench_reference(a)
    else:
        bench_ours(a)


if __name__ == "__main__":
    main()
