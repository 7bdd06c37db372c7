"""Gradient all-reduce + clip + Adam sweep over bucket sizes (multi-GPU).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 --master-port 29519 \
        -m autodrive_b200.bench.comm_bench --sizes 65536,1048576,16777216,268435456

For each gradient size (bytes of fp32) and each path, the time of one
optimizer step on the device (CUDA events, median of ``--iters`` after
``--warmup``, max over ranks):

* ``nccl``       torch.distributed all_reduce (sum) + divide + fused clip/Adam
* ``oneshot``    the fused peer-memory kernel, one-shot mode
* ``twoshot``    the fused peer-memory kernel, reduce-scatter/all-gather mode

Reported bus bandwidth is 2(W-1)/W x bytes / time (the all-reduce convention);
the NVLink roofline is the bytes each rank must move across NVLink at the
measured 770 GB/s per direction: two-shot (and NCCL ring) 2(W-1)/W x bytes,
one-shot (W-1) x bytes, against which ``roofline_frac`` is reported.
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

LINK_GBS = 770.


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--sizes", default="65536,262144,1048576,4194304,16777216,67108864,268435456")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    args = p.parse_args(argv)
    from autodrive_b200.parallel import dist as pdist
    from autodrive_b200.parallel.p2p import FusedAllReduceAdam
    from autodrive_b200.train.optim import FusedAdam
    import torch.distributed as dist
    state = pdist.distributed_state("cuda", timeout_s=300)
    rank, world = state.rank, state.world
    rows = []
    for size in [int(x) for x in args.sizes.split(",")]:
        n = size // 4
        row = {"bytes": size, "world": world}
        for path in ("nccl", "oneshot", "twoshot"):
            if world == 1 and path != "nccl":
                continue
            mod = torch.nn.Module()
            mod.w = torch.nn.Parameter(torch.zeros(n, device="cuda"))
            opt = FusedAdam(mod, lr=1e-4, max_grad_norm=1.)
            peer = None
            if path != "nccl":
                peer = FusedAllReduceAdam(opt, oneshot_bytes=(1 << 62) if path == "oneshot" else 0)
            g = torch.Generator(device="cuda").manual_seed(rank)
            opt.flat.grad.copy_(torch.randn(n, device="cuda", generator=g))

            def step():
                if peer is not None:
                    opt.step_count += 1
                    peer.ext.peer_comm_step(peer.comm, peer.m, peer.v, opt.last_norm, opt.step_count, opt.lr,
                                            opt.betas[0], opt.betas[1], opt.eps, opt.weight_decay,
                                            opt.max_grad_norm, peer.max_wait_iters)
                else:
                    dist.all_reduce(opt.flat.grad)
                    opt.flat.grad.div_(world)
                    opt.step()

            for _ in range(args.warmup):
                step()
            torch.cuda.synchronize()
            ts = []
            for _ in range(args.iters):
                dist.barrier()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                step()
                b.record()
                b.synchronize()
                ts.append(a.elapsed_time(b))
            if peer is not None:
                peer.check()
            t = torch.tensor([statistics.median(ts)], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t)
            moved = (world - 1) * size if path == "oneshot" else 2 * (world - 1) / world * size
            roof_ms = moved / (LINK_GBS * 1e9) * 1e3
            row[path] = {"us": round(ms * 1e3, 2),
                         "busbw_gbs": round(2 * (world - 1) / max(world, 1) * size / (ms * 1e-3) / 1e9, 2),
                         "roofline_us": round(roof_ms * 1e3, 2),
                         "roofline_frac": round(roof_ms / ms, 4) if ms > 0 else None}
            del peer, opt, mod
            torch.cuda.empty_cache()
            dist.barrier()
        rows.append(row)
        if rank == 0:
            print(json.dumps(row), flush=True)
    pdist.teardown(state)
    return rows


if __name__ == "__main__":
    main()
