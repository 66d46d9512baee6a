"""Tensor-parallel engines: one process per GPU, one engine per process.

The reference runs a model on one GPU (src/models/ModelBase.cpp:129 moves every
weight to the one CUDA device); this engine adds Megatron-style tensor
parallelism: each rank is its own process holding 1/tp of every projection
(Q/K/V heads, O columns, gate/up rows, down columns, lm_head rows) and an
NCCL communicator.
The decode step's all-reduces run inside the persistent GEMV segments over
NVLink peer memory; prefill all-reduces and the logits all-gather are NCCL.

A process group (gloo is enough) carries the NCCL unique id from rank 0 to
every rank; nothing else of the data path uses it.
"""
from typing import Optional

from . import engine as E


def share_nccl_id(pg, rank: int) -> bytes:
    """Rank 0 makes the NCCL unique id; every rank returns the same 128 bytes."""
    obj = [E.nccl_unique_id() if rank == 0 else None]
    pg.broadcast_object_list(obj, src=0)
    nid = obj[0]
    if not isinstance(nid, (bytes, bytearray)) or len(nid) != 128:
        raise RuntimeError("NCCL unique id broadcast failed")
    return bytes(nid)


def tp_engine(pg, rank: int, world: int, config: E.ModelConfig, snapshot_dir: Optional[str] = None,
              device: Optional[int] = None, **options) -> E.Engine:
    """This rank's engine of a `world`-way tensor-parallel model.

    `pg` is an initialised torch.distributed module or group wrapper with
    broadcast_object_list (world > 1 only). Every rank must call this with the
    same config and options; each then makes the same engine calls in the
    same order (a decode step of one rank waits for its peers' partials)."""
    nid = share_nccl_id(pg, rank) if world > 1 else None
    return E.Engine(snapshot_dir, config, nccl_id=nid, device=rank if device is None else device,
                    tp_rank=rank, tp_size=world, **options)
