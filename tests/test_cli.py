"""`python -m frc_defense.tensor_training` end to end on CPU (tiny sizes)."""
import json
import os
import subprocess
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ENV = {**os.environ, "PYTHONPATH": ROOT}


def test_generational_train_then_evaluate(tmp_path):
    out = tmp_path / "run"
    cmd = [sys.executable, "-m", "frc_defense.tensor_training", "train", "--device", "cpu", "--envs", "4",
           "--rollout-steps", "8", "--epochs", "1", "--minibatch-size", "16", "--horizon", "150",
           "--generations", "2", "--evaluation-episodes", "2", "--no-fuel-physics", "--steps", "128",
           "--output", str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, env=ENV, timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    status = json.loads((out / "status.json").read_text())
    assert status["status"] == "completed" and status["generation"] == 2
    history = json.loads((out / "generation-history.json").read_text())
    assert [g["generation"] for g in history["generations"]] == [1, 2]
    members = json.loads((out / "opponent-population" / "population.json").read_text())["members"]
    assert 1 <= len(members) <= 8
    payload = torch.load(out / "policy.pt", weights_only=True)
    for key in ("model_state_dict", "obs_dim", "action_dim", "action_kind", "architecture", "task",
                "observation_normalization", "drivetrain_config"):
        assert key in payload
    assert sorted(payload["model_state_dict"]) == ["actor.bias", "actor.weight", "critic.bias", "critic.weight",
                                                    "trunk.0.bias", "trunk.0.weight", "trunk.2.bias",
                                                    "trunk.2.weight"]
    ev = subprocess.run([sys.executable, "-m", "frc_defense.tensor_training", "evaluate", "--device", "cpu",
                         "--checkpoint", str(out / "policy.pt"), "--episodes", "2", "--envs", "2",
                         "--horizon", "100", "--opponent", "cutoff", "--output", str(tmp_path / "ev.json")],
                        capture_output=True, text=True, env=ENV, timeout=600)
    assert ev.returncode == 0, ev.stderr[-2000:]
    metrics = json.loads((tmp_path / "ev.json").read_text())
    lo, hi = metrics["success_wilson_95"]
    assert 0. <= lo <= metrics["mean_success"] <= hi <= 1.


def test_failed_train_writes_status(tmp_path):
    out = tmp_path / "bad"
    r = subprocess.run([sys.executable, "-m", "frc_defense.tensor_training", "train", "--device", "cpu",
                        "--opponent", "nonsense", "--output", str(out)],
                       capture_output=True, text=True, env=ENV, timeout=300)
    assert r.returncode != 0
    assert json.loads((out / "status.json").read_text())["status"] == "failed"
