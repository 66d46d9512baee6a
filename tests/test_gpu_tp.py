"""Tensor parallelism on 2, 4 and 8 GPUs: one process per GPU, one engine each
(rank r holds 1/tp of every projection), through the C ABI.

With two ranks the all-reduce of FP16 partials is one correctly rounded FP16
addition per element whichever side computes it, so the persistent path (the
all-reduce inside the GEMV segments, over NVLink peer memory) and the per-op
graph (NCCL all-reduce, then a residual add) agree bit for bit. With more
ranks NCCL's FP16 reduction order differs from the segments' (FP32 sum in rank
order, one rounding), so there both paths are held to the logit tolerance of
the oracle's single-device FP16 forward."""
import os
import socket

import numpy as np
import pytest

from oracle.model import OracleModel
from oracle import sampler as S
from yalama_b200 import synth

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-2
# every shape divides by 8 ranks: KV heads, intermediate size and vocabulary
FAMILIES = {
    "llama": dict(model_type="llama", tied=False, rope_theta=5e5, heads=8, kv_heads=8, vocab=1024),
    "qwen3": dict(model_type="qwen3", heads=16, kv_heads=8, vocab=1024),
    "qwen2": dict(model_type="qwen2", tied=False, heads=8, kv_heads=8, vocab=1024),
}
PROMPT_LEN, STEPS = 40, 12


def gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    from yalama_b200 import engine as E
    from yalama_b200 import tp as TP
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    try:
        for fam, kw in FAMILIES.items():
            spec = synth.tiny_spec(**kw)
            cfg = E.config_from_spec(spec)
            prompt = synth.prompt_ids(5, PROMPT_LEN, spec.vocab)
            for persistent in (0, 1):
                eng = TP.tp_engine(dist, rank, world, cfg, init_seed=0, decode_persistent=persistent)
                assert eng.decode_persistent() == bool(persistent)
                eng.begin_infer()
                st, _ = eng.infer(prompt)
                assert st == E.Status.OK
                rows, toks = [eng.logits()], []
                for _ in range(STEPS):
                    tok = S.greedy(rows[-1])
                    toks.append(tok)
                    st, _ = eng.infer([tok])
                    assert st == E.Status.OK
                    rows.append(eng.logits())
                # the advance-mode decode loop (graph replays)
                assert eng.time_decode(6) > 0
                loop = eng.logits()
                # greedy token loops: on the persistent path each rank's best
                # candidate crosses over peer memory instead of a logits gather,
                # and the logits are gathered only when read
                eng.set_sampling(greedy=True)
                gen = eng.generate(prompt, STEPS)
                assert gen["status"] == E.Status.OK
                eng.begin_infer()
                st, _ = eng.infer(prompt)
                assert st == E.Status.OK
                seq = [eng.sample(True)]
                for _ in range(3):
                    st, nxt = eng.decode(seq[-1], True)
                    assert st == E.Status.OK
                    seq.append(nxt)
                dec_logits = eng.logits()
                if rank == 0:
                    np.savez(os.path.join(out_dir, f"{fam}_{persistent}.npz"), rows=np.stack(rows),
                             toks=np.array(toks), loop=loop, gen=gen["ids"], seq=np.array(seq),
                             dec_logits=dec_logits)
                eng.close()
                dist.barrier()
    finally:
        dist.destroy_process_group()


def oracle_worst(kw, rows, toks):
    spec = synth.tiny_spec(**kw)
    orc = OracleModel(spec, synth.model_weights(spec, 0), mode="f16", kv_gb=2)
    orc.begin_infer()
    ids = list(synth.prompt_ids(5, PROMPT_LEN, spec.vocab))
    worst = 0.0
    for i, row in enumerate(rows):
        _, lo = orc.infer(ids)
        worst = max(worst, float(np.max(np.abs(row - lo))))
        if i < len(toks):
            ids = [int(toks[i])]
    return worst


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_persistent_and_per_op_match_oracle(world, tmp_path):
    if gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.start_processes(_rank_main, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for fam, kw in FAMILIES.items():
        p = np.load(tmp_path / f"{fam}_1.npz")
        g = np.load(tmp_path / f"{fam}_0.npz")
        if world == 2:
            np.testing.assert_array_equal(p["rows"], g["rows"])
            np.testing.assert_array_equal(p["toks"], g["toks"])
            np.testing.assert_array_equal(p["loop"], g["loop"])
        for name, r in (("persistent", p), ("per-op", g)):
            # the greedy loops pick the argmax of the same logits, on every rank
            np.testing.assert_array_equal(r["gen"], r["toks"])
            np.testing.assert_array_equal(r["seq"], r["toks"][:4])
            np.testing.assert_array_equal(r["dec_logits"], r["rows"][3])
            worst = oracle_worst(kw, r["rows"], r["toks"])
            print(f"{fam} tp{world} {name}: max |logit diff| vs oracle = {worst:.3e}")
            assert worst < LOGIT_TOL


# Llama-3.1-70B width, one layer: at 8 ranks each GPU holds one KV head and
# eight query heads, 3584 of the 28672 intermediate rows, 16032 vocabulary rows
WIDE = dict(preset="llama3.1-70b", layers=1, prompt=300, steps=6)


def _wide_rank_main(rank, world, port, root, out_dir):
    import dataclasses
    import datetime
    import torch.distributed as dist
    from yalama_b200 import engine as E
    from yalama_b200 import tp as TP
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=300))
    try:
        spec = dataclasses.replace(synth.PRESETS[WIDE["preset"]], layers=WIDE["layers"])
        snap = E.resolve_snapshot(root)
        prompt = synth.prompt_ids(21, WIDE["prompt"], spec.vocab)
        for persistent in (0, 1):
            # every rank slices its share of each tensor straight from the snapshot
            eng = TP.tp_engine(dist, rank, world, E.config_from_spec(spec), snapshot_dir=snap,
                               decode_persistent=persistent)
            eng.begin_infer()
            st, _ = eng.infer(prompt)
            assert st == E.Status.OK
            rows, toks = [eng.logits()], []
            for _ in range(WIDE["steps"]):
                tok = S.greedy(rows[-1])
                toks.append(tok)
                st, _ = eng.infer([tok])
                assert st == E.Status.OK
                rows.append(eng.logits())
            if rank == 0:
                np.savez(os.path.join(out_dir, f"wide_{persistent}.npz"), rows=np.stack(rows), toks=np.array(toks))
            eng.close()
            dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 8])
def test_tp_snapshot_slices_at_70b_width(world, tmp_path):
    if gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    import dataclasses
    import torch.multiprocessing as mp
    from yalama_b200 import engine as E
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    spec = dataclasses.replace(synth.PRESETS[WIDE["preset"]], layers=WIDE["layers"])
    root = str(tmp_path / "model")
    synth.write_snapshot(root, spec, seed=0, dtype="F16", fast=True)
    mp.start_processes(_wide_rank_main, args=(world, free_port(), root, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    # the same snapshot on one GPU, fed the same tokens
    one = E.Engine(E.resolve_snapshot(root), E.config_from_spec(spec), device=0)
    prompt = synth.prompt_ids(21, WIDE["prompt"], spec.vocab)
    for persistent in (0, 1):
        z = np.load(tmp_path / f"wide_{persistent}.npz")
        one.begin_infer()
        one.infer(prompt)
        worst = float(np.max(np.abs(one.logits() - z["rows"][0])))
        for i, tok in enumerate(z["toks"]):
            one.infer([int(tok)])
            worst = max(worst, float(np.max(np.abs(one.logits() - z["rows"][i + 1]))))
        print(f"70b width tp{world} persistent={persistent}: max |logit diff| vs one GPU = {worst:.3e}")
        assert worst < LOGIT_TOL
    one.close()
