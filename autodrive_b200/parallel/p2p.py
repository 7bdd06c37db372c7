"""Fused peer-memory all-reduce + clip + Adam for data-parallel training.

Every rank re-homes its flat gradient and parameter buffers into one
IPC-exported device region (`csrc/comm_ops.cu`); IPC handles are exchanged
over the gloo control group. One cooperative kernel per optimizer step then
reduce-scatters gradients with NVLink peer loads, all-reduces the shard norms
for the global clip, applies Adam to the owned shard and all-gathers the new
parameters with peer stores. Waits on peers are bounded: a rank that stops
participating makes the others raise `PeerCommError` instead of hanging.

Two modes, chosen by buffer size: buffers up to ``oneshot_bytes`` (4 MB) use a
one-shot kernel (each rank reads every peer's whole gradient, reduces it,
takes the global norm locally and applies Adam to the whole buffer: two
cross-rank barriers, no parameter traffic); larger ones use the two-shot
reduce-scatter / sharded Adam / parameter all-gather kernel, whose optimizer
moments are meaningful for the owned shard only (ZeRO-1 layout).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import require_extension
from ..utils import launches
from . import dist as pdist


class PeerCommError(RuntimeError):
    pass


ONESHOT_BYTES = 4 << 20  # buffers up to 4 MB: one-shot all-reduce (latency bound)


class FusedAllReduceAdam:
    def __init__(self, optimizer, max_wait_iters: int = 1 << 24, check_every: int = 1,
                 oneshot_bytes: int = ONESHOT_BYTES):
        self.ext = require_extension()
        self.opt = optimizer
        grouped = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size() if grouped else 1
        self.rank = dist.get_rank() if grouped else 0
        flat = optimizer.flat
        if flat.flat.device.type != "cuda":
            raise RuntimeError("the peer-memory all-reduce needs CUDA ranks")
        n = flat.flat.numel()
        self.comm = self.ext.peer_comm_create(n, self.world, self.rank, int(oneshot_bytes))
        self.mode = "one-shot" if self.comm.oneshot else "two-shot"
        handle = self.ext.peer_comm_ipc_handle(self.comm)
        handles = [handle]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=pdist.control_group())
        self.ext.peer_comm_open(self.comm, handles)
        grad, param = self.ext.peer_comm_buffers(self.comm)
        param.copy_(flat.flat)
        grad.zero_()
        flat.rehome(param, grad)
        padded = self.comm.n_padded
        self.m = torch.zeros(padded, device=param.device)
        self.v = torch.zeros(padded, device=param.device)
        self.max_wait_iters = int(max_wait_iters)
        self.check_every = max(1, int(check_every))
        self.steps = 0
        self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._status_event = None
        torch.cuda.synchronize(param.device)
        pdist.barrier()

    def step(self) -> torch.Tensor:
        opt = self.opt
        opt.flat.sync_grads()
        opt.step_count += 1
        launches.add(1)
        self.ext.peer_comm_step(self.comm, self.m, self.v, opt.last_norm, opt.step_count, opt.lr,
                                opt.betas[0], opt.betas[1], opt.eps, opt.weight_decay, opt.max_grad_norm,
                                self.max_wait_iters)
        self.steps += 1
        if self.steps % self.check_every == 0:
            self.check(block=False)
        return opt.last_norm

    def stats_allreduce(self, sums: torch.Tensor, maxes: torch.Tensor | None = None) -> None:
        """In-place cross-rank sum of `sums` and max of `maxes` (float64, <= 16
        values in total) in one small peer-memory kernel."""
        self.ext.peer_stats_allreduce(self.comm, sums, maxes, self.max_wait_iters)

    def broadcast_parameters(self, root: int = 0) -> None:
        """Copy rank `root`'s parameters into every rank's parameters (peer stores)."""
        self.ext.peer_broadcast_params(self.comm, int(root), self.max_wait_iters)

    def check(self, block: bool = True) -> None:
        """Raise PeerCommError if a step gave up waiting on a peer. Non-blocking
        checks read the status copied after an earlier step (no host sync on
        the hot path); a blocking check waits for the latest step."""
        if block:
            code = int(self.comm.status.item())
        else:
            code = 0
            if self._status_event is not None and self._status_event.query():
                code = int(self._status_host[0])
            self._status_host.copy_(self.comm.status, non_blocking=True)
            if self._status_event is None:
                self._status_event = torch.cuda.Event()
            self._status_event.record()
        if code:
            # the word is cleared so a caller that recovers (or a later check)
            # sees only new expiries
            self.comm.status.zero_()
            phase = {1: "gradients-ready", 2: "norm exchange", 4: "completion", 8: "stats exchange",
                     16: "parameter broadcast"}.get(code, str(code))
            raise PeerCommError(f"peer all-reduce wait expired in the {phase} barrier on rank {self.rank}")
