"""Tensor-parallel host logic on CPU: two gloo ranks share the NCCL unique id,
and every rank rejects a tensor-parallel shape before touching a device
(KV heads, intermediate size and vocabulary must divide by tp; the rank must
lie in [0, tp))."""
import json
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from yalama_b200 import engine as E
from yalama_b200 import synth
from yalama_b200 import tp as TP


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nid = TP.share_nccl_id(dist, rank)
        open(os.path.join(out_dir, f"id{rank}"), "wb").write(nid)
        results = []
        # KV heads 3 do not split over 2 ranks
        spec = synth.tiny_spec("llama", layers=1, heads=3, kv_heads=3)
        for kw in (dict(tp_rank=rank, tp_size=world), dict(tp_rank=world, tp_size=world),
                   dict(tp_rank=-1, tp_size=world)):
            c = E.config_from_spec(spec if kw["tp_rank"] == rank else synth.tiny_spec("llama", layers=1))
            try:
                E.Engine(None, c, nccl_id=nid, **kw)
                results.append("created")
            except E.YlmError as ex:
                results.append(int(ex.status))
        # vocabulary not divisible by tp
        c = E.config_from_spec(synth.tiny_spec("llama", layers=1, vocab=1001))
        try:
            E.Engine(None, c, nccl_id=nid, tp_rank=rank, tp_size=world)
            results.append("created")
        except E.YlmError as ex:
            results.append(int(ex.status))
        open(os.path.join(out_dir, f"st{rank}"), "w").write(json.dumps(results))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_share_id_and_validate_shapes(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    ids = [open(tmp_path / f"id{r}", "rb").read() for r in range(world)]
    assert len(ids[0]) == 128 and ids[0] == ids[1]
    for r in range(world):
        st = json.loads(open(tmp_path / f"st{r}").read())
        assert st == [int(E.Status.INVALID_ARG)] * 4, (r, st)


def test_shape_rejection_needs_no_process_group():
    # rejected before any device or communicator is touched
    c = E.config_from_spec(synth.tiny_spec("llama", layers=1, heads=3, kv_heads=3))
    with pytest.raises(E.YlmError) as ei:
        E.Engine(None, c, tp_rank=0, tp_size=2)
    assert ei.value.status == E.Status.INVALID_ARG
    assert "tensor parallel" in str(ei.value)
