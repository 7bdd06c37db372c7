"""Failure detection without any GPU fault: corrupt or tampered checkpoints
are refused with a clear error, and a CPU (gloo) rank that raises mid-run
ends its peer with an error within the process-group timeout."""
import os
import socket
import subprocess
import sys

import pytest
import torch

from autodrive_b200.utils.checkpoint import CheckpointError, load_verified
from autodrive_b200.utils.provenance import state_dict_digest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _payload():
    sd = {"trunk.0.weight": torch.randn(8, 4), "trunk.0.bias": torch.zeros(8)}
    return {"model_state_dict": sd, "obs_dim": 4, "action_dim": 2, "weights_sha256": state_dict_digest(sd)}


def test_valid_checkpoint_loads(tmp_path):
    path = tmp_path / "policy.pt"
    torch.save(_payload(), path)
    assert set(load_verified(path)["model_state_dict"]) == {"trunk.0.weight", "trunk.0.bias"}


@pytest.mark.parametrize("damage", ["missing", "empty", "truncated", "garbage", "no_state"])
def test_damaged_checkpoint_is_refused(tmp_path, damage):
    path = tmp_path / "policy.pt"
    torch.save(_payload(), path)
    raw = path.read_bytes()
    if damage == "missing":
        path.unlink()
    elif damage == "empty":
        path.write_bytes(b"")
    elif damage == "truncated":
        path.write_bytes(raw[:len(raw) // 2])
    elif damage == "garbage":
        path.write_bytes(b"\x00not a checkpoint" * 32)
    else:
        torch.save({"obs_dim": 4}, path)
    with pytest.raises(CheckpointError, match="policy.pt"):
        load_verified(path)


def test_tampered_weights_fail_the_digest(tmp_path):
    payload = _payload()
    payload["model_state_dict"]["trunk.0.bias"][3] = 1.0      # changed after the digest was taken
    path = tmp_path / "policy.pt"
    torch.save(payload, path)
    with pytest.raises(CheckpointError, match="SHA-256"):
        load_verified(path)
    payload.pop("weights_sha256")
    torch.save(payload, path)
    with pytest.raises(CheckpointError):
        load_verified(path, require_digest=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


WORKER = r"""
import os, sys, torch
sys.path.insert(0, {root!r})
from autodrive_b200.parallel import dist as pdist
state = pdist.distributed_state("cpu", timeout_s=10)
x = torch.ones(4)
for step in range(50):
    if state.rank == 1 and step == 3:
        raise RuntimeError("injected failure on rank 1")
    pdist.all_reduce_(x)
print("finished", flush=True)
"""


def test_rank_that_raises_mid_run_ends_its_peer(tmp_path):
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT))
    env = {**os.environ, "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()), "WORLD_SIZE": "2"}
    procs = [subprocess.Popen([sys.executable, str(script)], env={**env, "RANK": str(r), "LOCAL_RANK": str(r)},
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True) for r in range(2)]
    outs = [p.communicate(timeout=180) for p in procs]
    assert procs[1].returncode != 0 and "injected failure" in outs[1][1]
    # the survivor gets an error from its next collective instead of hanging
    assert procs[0].returncode != 0
    assert "finished" not in outs[0][0]


def test_trace_stages_are_noops_without_nvtx():
    from autodrive_b200.utils import trace
    trace.set_enabled(True)          # no CUDA here: still a no-op
    with trace.stage("rollout"):
        x = 1
    trace.set_enabled(False)
    assert x == 1 and not trace.enabled()
