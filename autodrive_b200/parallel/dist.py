"""Process-group bootstrap: one process per GPU under torchrun.

Mirrors frc_defense/tensor_training_runtime.py:109-146: WORLD_SIZE/RANK/
LOCAL_RANK from the environment, ``init_process_group`` on NCCL for CUDA
ranks (gloo for CPU ranks), plus a separate gloo control group for barriers
so rank-0-only work (evaluation, checkpoint publication) never spins GPUs.
Groups are given a finite timeout so a missing rank ends its peers with an
error instead of hanging.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist

_CONTROL_GROUP = None
_CONTROL_OWNED = False


@dataclass
class DistState:
    device: torch.device
    rank: int
    world: int
    created: bool
    local_rank: int = 0

    @property
    def distributed(self) -> bool:
        return self.world > 1

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def resolve_device(requested) -> torch.device:
    dev = torch.device(requested)
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError(f"Requested accelerator {str(requested)!r} is unavailable; refusing CPU fallback")
    return dev


def distributed_state(device="cuda", timeout_s: float | None = None) -> DistState:
    """Initialise (or adopt) the torchrun process group and select the local device."""
    global _CONTROL_GROUP, _CONTROL_OWNED
    timeout = datetime.timedelta(seconds=float(timeout_s or os.environ.get("AD_PG_TIMEOUT_S", 900)))
    if dist.is_available() and dist.is_initialized():
        rank, world = dist.get_rank(), dist.get_world_size()
        local = int(os.environ.get("LOCAL_RANK", "0"))
        dev = resolve_device(device)
        if world > 1 and dev.type == "cuda":
            dev = torch.device("cuda", local)
            torch.cuda.set_device(dev)
        if world > 1 and _CONTROL_GROUP is None:
            _CONTROL_GROUP = dist.new_group(backend="gloo", timeout=timeout)
            _CONTROL_OWNED = True
        return DistState(dev, rank, world, False, local)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world <= 1:
        return DistState(resolve_device(device), 0, 1, False, 0)
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = resolve_device(device)
    if dev.type == "cuda":
        if local >= torch.cuda.device_count():
            raise RuntimeError(f"LOCAL_RANK={local} is outside the visible GPU set")
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", timeout=timeout, device_id=dev)
    else:
        dist.init_process_group("gloo", timeout=timeout)
    if dist.get_world_size() != world:
        raise RuntimeError(f"torchrun WORLD_SIZE={world} but the process group has {dist.get_world_size()} ranks")
    _CONTROL_GROUP = dist.new_group(backend="gloo", timeout=timeout)
    _CONTROL_OWNED = True
    return DistState(dev, dist.get_rank(), world, True, local)


def control_group():
    return _CONTROL_GROUP


def barrier() -> None:
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier(group=_CONTROL_GROUP)


def teardown(state: DistState) -> None:
    """Destroy only the groups this process created."""
    global _CONTROL_GROUP, _CONTROL_OWNED
    if _CONTROL_OWNED and dist.is_initialized() and _CONTROL_GROUP is not None:
        dist.destroy_process_group(_CONTROL_GROUP)
    _CONTROL_GROUP, _CONTROL_OWNED = None, False
    if state.created and dist.is_initialized():
        dist.destroy_process_group()


def all_reduce_(tensor: torch.Tensor, op: str = "sum") -> torch.Tensor:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return tensor
    ops = {"sum": dist.ReduceOp.SUM, "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}
    dist.all_reduce(tensor, op=ops[op])
    return tensor


def broadcast_object(obj, src: int = 0):
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return obj
    holder = [obj]
    dist.broadcast_object_list(holder, src=src, group=_CONTROL_GROUP)
    return holder[0]
