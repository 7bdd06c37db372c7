"""Fused peer-memory all-reduce + clip + Adam against NCCL/plain references.

One GPU: the kernel with a single rank must equal the two-launch fused Adam.
Two or more GPUs (skipped otherwise): ranks with different gradients must all
end with the parameters of "average the gradients, clip, Adam".
"""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _model(seed=0):
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Linear(37, 64), torch.nn.Tanh(), torch.nn.Linear(64, 9)).cuda()


def test_single_rank_matches_fused_adam():
    from autodrive_b200.parallel.p2p import FusedAllReduceAdam
    from autodrive_b200.train.optim import FusedAdam
    a, b = _model(), _model()
    oa = FusedAdam(a, lr=1e-2, max_grad_norm=.5)
    ob = FusedAdam(b, lr=1e-2, max_grad_norm=.5)
    peer = FusedAllReduceAdam(ob)
    x = torch.randn(128, 37, device="cuda")
    for _ in range(3):
        oa.zero_grad()
        a(x).square().sum().backward()
        oa.step()
        ob.zero_grad()
        b(x).square().sum().backward()
        peer.step()
    torch.cuda.synchronize()
    assert torch.allclose(oa.last_norm, ob.last_norm, rtol=1e-5)
    for pa, pb in zip(a.parameters(), b.parameters()):
        assert torch.allclose(pa, pb, atol=1e-6, rtol=1e-5)


WORKER = r"""
import json, os, sys, torch, torch.distributed as dist
sys.path.insert(0, {root!r})
from autodrive_b200.parallel import dist as pdist
from autodrive_b200.parallel.p2p import FusedAllReduceAdam
from autodrive_b200.train.optim import FusedAdam
state = pdist.distributed_state("cuda", timeout_s=120)
rank, world = state.rank, state.world
def model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(37, 64), torch.nn.Tanh(), torch.nn.Linear(64, 9)).cuda()
a, b = model(), model()
oa = FusedAdam(a, lr=1e-2, max_grad_norm=.5)
ob = FusedAdam(b, lr=1e-2, max_grad_norm=.5)
peer = FusedAllReduceAdam(ob, oneshot_bytes=int(os.environ["AD_ONESHOT_BYTES"]))
torch.manual_seed(100 + rank)
for _ in range(3):
    x = torch.randn(128, 37, device="cuda")
    oa.zero_grad(); a(x).square().sum().backward()
    dist.all_reduce(oa.flat.grad); oa.flat.grad.div_(world); oa.step()
    ob.zero_grad(); b(x).square().sum().backward(); peer.step()
torch.cuda.synchronize()
diff = max(float((pa - pb).abs().max()) for pa, pb in zip(a.parameters(), b.parameters()))
sums = torch.tensor([rank + 1., 2. * (rank + 1)], dtype=torch.float64, device="cuda")
maxes = torch.tensor([float(rank), -float(rank)], dtype=torch.float64, device="cuda")
for _ in range(3):
    s2, m2 = sums.clone(), maxes.clone()
    peer.stats_allreduce(s2, m2)
tri = world * (world + 1) / 2
stats_ok = bool(torch.allclose(s2.cpu(), torch.tensor([tri, 2 * tri], dtype=torch.float64))
                and m2[0].item() == world - 1 and m2[1].item() == 0.)
if rank == 0:
    for p in b.parameters():
        p.data.fill_(.25)
peer.broadcast_parameters(0)
torch.cuda.synchronize()
bcast_ok = all(bool((p == .25).all()) for p in b.parameters())
peer.check()
print(json.dumps({{"rank": rank, "diff": diff, "norm_a": float(oa.last_norm), "norm_b": float(ob.last_norm),
                  "mode": peer.mode, "stats_ok": stats_ok, "bcast_ok": bcast_ok}}))
pdist.teardown(state)
"""


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("oneshot_bytes,mode", [(0, "two-shot"), (1 << 22, "one-shot")])
def test_two_ranks_match_nccl_average(tmp_path, oneshot_bytes, mode):
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT))
    world = min(torch.cuda.device_count(), 8)
    env = {**os.environ, "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()), "WORLD_SIZE": str(world),
           "NCCL_NVLS_ENABLE": "0", "AD_ONESHOT_BYTES": str(oneshot_bytes)}
    procs = [subprocess.Popen([sys.executable, str(script)], stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                              text=True, env={**env, "RANK": str(r), "LOCAL_RANK": str(r)}) for r in range(world)]
    outs = [p.communicate(timeout=300) for p in procs]
    for p, (so, se) in zip(procs, outs):
        assert p.returncode == 0, se[-3000:]
    for so, _ in outs:
        row = json.loads(so.strip().splitlines()[-1])
        assert row["mode"] == mode
        assert row["diff"] < 1e-5, row
        assert row["stats_ok"] and row["bcast_ok"], row
        assert abs(row["norm_a"] - row["norm_b"]) < 1e-4 * max(1., row["norm_a"]), row


TIMEOUT_WORKER = r"""
import json, os, sys, time, torch
sys.path.insert(0, {root!r})
from autodrive_b200.parallel import dist as pdist
from autodrive_b200.parallel.p2p import FusedAllReduceAdam, PeerCommError
from autodrive_b200.train.optim import FusedAdam
state = pdist.distributed_state("cuda", timeout_s=120)
rank = state.rank
torch.manual_seed(0)
model = torch.nn.Sequential(torch.nn.Linear(37, 64), torch.nn.Tanh(), torch.nn.Linear(64, 9)).cuda()
opt = FusedAdam(model, lr=1e-2, max_grad_norm=.5)
peer = FusedAllReduceAdam(opt, max_wait_iters=1 << 12)
result = {{"rank": rank}}
if rank == 0:
    # rank 1 stays alive between steps but never joins this step: every
    # bounded wait of rank 0's kernels must run out and report its phase
    opt.zero_grad()
    model(torch.randn(64, 37, device="cuda")).square().sum().backward()
    t0 = time.perf_counter()
    peer.step()
    try:
        peer.check(block=True)
        result["step_error"] = None
    except PeerCommError as exc:
        result["step_error"] = str(exc)
    result["step_seconds"] = time.perf_counter() - t0
    sums = torch.ones(2, dtype=torch.float64, device="cuda")
    peer.stats_allreduce(sums)
    try:
        peer.check(block=True)
        result["stats_error"] = None
    except PeerCommError as exc:
        result["stats_error"] = str(exc)
    result["status_after"] = int(peer.comm.status.item())
    torch.cuda.synchronize()
pdist.barrier()
print(json.dumps(result))
pdist.teardown(state)
"""


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_wait_expiry_raises(tmp_path):
    """A rank that skips a step makes the other rank's bounded device waits
    run out: the kernel returns, the status word holds the phase and the host
    raises PeerCommError naming it (gradients-ready, then stats exchange)."""
    script = tmp_path / "timeout_worker.py"
    script.write_text(TIMEOUT_WORKER.format(root=ROOT))
    env = {**os.environ, "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()), "WORLD_SIZE": "2",
           "NCCL_NVLS_ENABLE": "0"}
    procs = [subprocess.Popen([sys.executable, str(script)], stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                              text=True, env={**env, "RANK": str(r), "LOCAL_RANK": str(r)}) for r in range(2)]
    outs = [p.communicate(timeout=300) for p in procs]
    for p, (so, se) in zip(procs, outs):
        assert p.returncode == 0, se[-3000:]
    row = json.loads(outs[0][0].strip().splitlines()[-1])
    assert row["step_error"] and "gradients-ready" in row["step_error"], row
    assert row["stats_error"] and "stats exchange" in row["stats_error"], row
    assert row["status_after"] == 0, row
    assert row["step_seconds"] < 30, row
