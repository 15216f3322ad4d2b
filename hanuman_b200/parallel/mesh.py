"""Process-group setup and the (data, expert) device mesh.

One process per GPU (torchrun).  ``init_distributed`` reads RANK /
LOCAL_RANK / WORLD_SIZE / MASTER_* from the environment, binds the local GPU
and initialises NCCL (gloo on CPU) with a bounded timeout so that a rank that
never arrives ends the collective with an error instead of a hang.  The mesh
mirrors model/sharding.py:12-30 of the reference: axes ``("data", "expert")``
with ``data * expert == world``.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class DistCtx:
    rank: int
    world: int
    local_rank: int
    device: torch.device
    backend: str
    data: int = 1
    expert: int = 1
    mesh: object = None

    def barrier(self):
        if self.backend == "nccl":
            dist.barrier(device_ids=[self.local_rank])
        else:
            dist.barrier()

    def max_scalar(self, x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_scalar(self, x: float) -> float:
        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def shutdown(self):
        if dist.is_initialized():
            dist.destroy_process_group()


def init_distributed(timeout_s: float = 120.0, expert: int = 1) -> Optional[DistCtx]:
    """Initialise from torchrun variables; None when WORLD_SIZE is 1/unset."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return None
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
        backend = "nccl"
    else:
        dev = torch.device("cpu")
        backend = "gloo"
    kw = {}
    if backend == "nccl":
        kw["device_id"] = dev
    dist.init_process_group(backend=backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)
    ctx = DistCtx(rank, world, local, dev, backend, data=world // expert, expert=expert)
    if backend == "nccl":
        from torch.distributed.device_mesh import init_device_mesh
        ctx.mesh = init_device_mesh("cuda", (ctx.data, ctx.expert),
                                    mesh_dim_names=("data", "expert"))
    return ctx
