"""Data-parallel gradient synchronisation over one flat gradient buffer.

Backends:

* ``"p2p"`` (CUDA, world > 1): the fused peer-memory all-reduce kernel over
  NVLink/NVSwitch (`autodrive_b200.parallel.p2p`), which reduces, averages,
  computes the global gradient norm, clips and applies Adam in one launch.
* ``"nccl"``: ``torch.distributed.all_reduce`` on the flat buffer followed
  by the fused clip+Adam kernels (the baseline path).
* ``"gloo"``: CPU ranks (tests and CPU plumbing runs).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class GradientSync:
    def __init__(self, optimizer, world: int, backend: str = "auto"):
        self.opt = optimizer
        self.world = world
        dev = optimizer.flat.flat.device
        if backend == "auto":  # the fused peer-memory kernel is the multi-GPU product path
            backend = "p2p" if dev.type == "cuda" else "gloo"
        if world > 1 and backend == "p2p":
            from .p2p import FusedAllReduceAdam
            self.fused = FusedAllReduceAdam(optimizer)
        else:
            self.fused = None
        self.backend = backend if world > 1 else "local"

    def step(self) -> torch.Tensor:
        """Average gradients across ranks, clip by global norm, apply Adam."""
        if self.world > 1:
            if self.fused is not None:
                return self.fused.step()
            self.opt.flat.sync_grads()
            g = self.opt.flat.grad
            dist.all_reduce(g, op=dist.ReduceOp.SUM)
            g.div_(self.world)
        return self.opt.step()


def sync_parameters(module: torch.nn.Module, world: int) -> None:
    """Broadcast rank 0's parameters so every replica starts identical."""
    if world <= 1:
        return
    for p in module.parameters():
        dist.broadcast(p.data, src=0)
