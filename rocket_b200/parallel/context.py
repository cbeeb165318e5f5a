"""Process-group plumbing: one process per GPU, ``torch.distributed`` over NCCL.

TP (attention heads, dense-MLP intermediate, vocab) and EP (routed experts)
both span the whole node here, as in the headline serving config (EP8 + TP8).  The
collectives below are the unfused NCCL path; the fused kernels in
``parallel/fused.py`` replace the hot ones.

Reference counterpart: the 2-rank RDMA fabric and ExpertParallel
(engines/glm5-moe-nvfp4-2b/src/fabric/{fabric.h,expert_parallel.h}); on one
NVSwitch node NCCL takes the transport's place.
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


class ParallelCtx:
    def __init__(self, rank: int = 0, world: int = 1, device=None, group=None):
        self.rank = rank
        self.world = world
        self.tp = world
        self.ep = world
        self.tp_rank = rank
        self.ep_rank = rank
        self.group = group
        self.device = torch.device(device) if device is not None else torch.device("cuda", 0)

    @property
    def enabled(self) -> bool:
        return self.world > 1

    def with_layout(self, tp: int, ep: int) -> "ParallelCtx":
        """A context over the same process group with attention / dense / vocab split
        `tp` ways and routed experts `ep` ways.  Each is 1 (replicated on every rank) or
        the world size; tp = ep = 1 on several ranks means the default tp = ep = world.
        tp = 1, ep = world is the exact-parity layout: attention replicated, experts
        expert parallel."""
        if tp == 1 and ep == 1:
            tp = ep = self.world
        for name, v in (("tp", tp), ("ep", ep)):
            if v not in (1, self.world):
                raise ValueError(f"{name}={v}: must be 1 or the world size {self.world}")
        c = ParallelCtx(self.rank, self.world, self.device, self.group)
        c.tp, c.ep = tp, ep
        c.tp_rank = self.rank if tp > 1 else 0
        c.ep_rank = self.rank if ep > 1 else 0
        return c

    def all_reduce(self, t: torch.Tensor):
        if self.world > 1:
            dist.all_reduce(t, group=self.group)
        return t

    def all_reduce_max(self, t: torch.Tensor):
        if self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return t

    def all_gather_into(self, out: torch.Tensor, inp: torch.Tensor):
        if self.world > 1:
            dist.all_gather_into_tensor(out, inp, group=self.group)
        else:
            out.copy_(inp)
        return out

    def broadcast(self, t: torch.Tensor, src: int = 0):
        if self.world > 1:
            dist.broadcast(t, src=src, group=self.group)
        return t

    def barrier(self):
        if self.world > 1:
            dist.barrier(group=self.group)

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())

    def shard(self, n: int, what: str = "") -> tuple[int, int]:
        """[lo, hi) of a tensor-parallel dimension for this rank (must divide evenly)."""
        if n % self.tp:
            raise ValueError(f"{what or 'dimension'} {n} not divisible by {self.tp} ranks")
        s = n // self.tp
        return self.tp_rank * s, (self.tp_rank + 1) * s


def init_from_env(timeout_s: float = 120.0) -> ParallelCtx:
    """Create the NCCL process group from torchrun's environment (or a 1-GPU ctx)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        dev = torch.device("cuda", local)
    else:
        dev = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = dev
        dist.init_process_group(**kw)
    return ParallelCtx(rank, world, dev, None)
