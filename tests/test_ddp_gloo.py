"""Data-parallel PPO semantics on two gloo CPU ranks (world_size=2)."""
import json
import math
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


WORKER = r"""
import json, os, sys, torch
sys.path.insert(0, {root!r})
from autodrive_b200.parallel import dist as pdist
from autodrive_b200.train.ppo import train_once
state = pdist.distributed_state("cpu", timeout_s=120)
# CPU plumbing configuration: two-robot defense env, 4 worlds per rank, static
# FUEL (60 spheres at uniform random positions), a 200-tick rollout (16
# strategic decisions held 12/13 ticks) against the deterministic scripted
# offense, the 2 x 256 tanh MLP, PPO with 2 epochs x 4 minibatches, clip 0.2,
# Adam lr 3e-4, seed 0
r = train_once("defense", 4 * 16, {out!r}, seed=0, num_envs=4, device="cpu", opponent="offense",
               rollout_steps=16, epochs=2, minibatch_size=16, horizon=200, fuel_physics=False,
               clip_coef=.2, learning_rate=3e-4, network="mlp256", curriculum=False, dist_state=state,
               env_kwargs={{"fuel_count": 60, "fuel_layout": "uniform"}})
print(json.dumps({{"rank": state.rank, "world": r["world_size"], "transitions": r["transitions"],
                  "ticks": r["physics_world_ticks_per_second"] > 0, "mean_reward": r["mean_reward"],
                  "entropy": r["entropy"], "grad_norm": r["grad_norm"], "params": r["parameters_sha256"]}}))
pdist.teardown(state)
"""


def test_two_rank_ppo(tmp_path):
    out = str(tmp_path / "run")
    script = tmp_path / "worker.py"
    script.write_text(WORKER.format(root=ROOT, out=out))
    env = {**os.environ, "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()), "WORLD_SIZE": "2"}
    procs = []
    for rank in range(2):
        e = {**env, "RANK": str(rank), "LOCAL_RANK": str(rank)}
        procs.append(subprocess.Popen([sys.executable, str(script)], env=e, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=600) for p in procs]
    for p, (so, se) in zip(procs, outs):
        assert p.returncode == 0, se[-3000:]
    rows = [json.loads(so.strip().splitlines()[-1]) for so, _ in outs]
    assert {r["rank"] for r in rows} == {0, 1}
    assert all(r["world"] == 2 for r in rows)
    # counters are all-reduced: both ranks report the global transition count
    assert rows[0]["transitions"] == rows[1]["transitions"] == 2 * 4 * 16
    for r in rows:
        assert all(math.isfinite(r[k]) for k in ("mean_reward", "entropy", "grad_norm")), r
    # identical starting weights + averaged gradients: the replicas end equal
    assert rows[0]["params"] == rows[1]["params"]
    status = json.load(open(os.path.join(out, "status.json")))
    assert status["status"] == "completed" and status["world_size"] == 2
    assert status["network"] == "mlp256"


def test_rank_that_never_joins_times_out(tmp_path):
    """A missing rank must end its peer with an error, not a hang."""
    script = tmp_path / "lonely.py"
    script.write_text(
        "import sys; sys.path.insert(0, %r)\n"
        "from autodrive_b200.parallel import dist as pdist\n"
        "pdist.distributed_state('cpu', timeout_s=5)\n" % ROOT)
    env = {**os.environ, "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(_free_port()), "WORLD_SIZE": "2",
           "RANK": "0", "LOCAL_RANK": "0", "TORCH_DIST_INIT_BARRIER": "1"}
    proc = subprocess.run([sys.executable, str(script)], env=env, capture_output=True, text=True, timeout=120)
    assert proc.returncode != 0
