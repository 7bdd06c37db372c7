"""Architecture-zoo networks through the product trainer and CLI (CPU, tiny).

The perception networks read dictionaries built from the 3v3 environment's
simulated perception; PPO, generational training, checkpoints and the 3v3
evaluation path must all accept them.
"""
import json

import pytest
import torch

from autodrive_b200.train.cli import main as cli_main
from autodrive_b200.train.evaluation import evaluate_3v3_once
from autodrive_b200.train.ppo import train_once


def _small_3v3():
    return dict(fuel_count=120, perception_interval=2)


@pytest.mark.parametrize("network", ["entity_attention", "full_field_cnn", "deep_sets"])
def test_ppo_trains_a_perception_network_on_3v3(tmp_path, network):
    r = train_once("defense", 2 * 2 * 3, tmp_path / network, seed=0, num_envs=2, device="cpu",
                   opponent="offense", rollout_steps=2, epochs=1, minibatch_size=6, horizon=60,
                   env_kind="3v3", network=network, fuel_physics=False, curriculum=False,
                   env_kwargs=_small_3v3())
    assert r["status"] == "completed" and r["network"] == network
    assert all(map(lambda k: torch.isfinite(torch.tensor(r[k])), ("entropy", "grad_norm", "mean_reward")))
    payload = torch.load(tmp_path / network / "policy.pt", weights_only=False)
    assert payload["env"] == "3v3" and payload["network"] == network
    metrics = evaluate_3v3_once(tmp_path / network / "policy.pt", episodes=2, seed=5, num_envs=2, device="cpu",
                                horizon=40, fuel_physics=False, env_kwargs=_small_3v3())
    assert metrics["episodes"] == 2 and metrics["network"] == network
    assert len(metrics["mean_opponent_acquisitions_by_robot"]) == 3
    for key in ("mean_cycle_time", "mean_passes_attempted", "mean_fuel_transferred", "mean_failed_passes"):
        assert key in metrics


def test_perception_network_needs_the_3v3_env(tmp_path):
    with pytest.raises(ValueError, match="3v3"):
        train_once("defense", 8, tmp_path / "x", seed=0, num_envs=2, device="cpu", opponent="offense",
                   rollout_steps=2, epochs=1, minibatch_size=4, horizon=40, network="entity_attention",
                   fuel_physics=False, curriculum=False)


def test_cli_generational_cnn_on_3v3(tmp_path, capsys, monkeypatch):
    """`train --algorithm generational --network <cnn> --env 3v3` runs two
    generations with an opponent pool and strong-checkpoint elites."""
    import autodrive_b200.train.ppo as ppo
    real = ppo.make_env

    def small(kind, *a, **kw):   # keep the CPU test small: 120 FUEL pieces
        if kind == "3v3":
            kw = {**kw, **_small_3v3()}
        return real(kind, *a, **kw)
    monkeypatch.setattr(ppo, "make_env", small)
    out = tmp_path / "gen"
    cli_main(["train", "--algorithm", "generational", "--network", "full_field_cnn", "--env", "3v3",
              "--no-fuel-physics", "--envs", "2", "--steps", "24", "--rollout-steps", "2", "--epochs", "1",
              "--minibatch-size", "6", "--horizon", "40", "--generations", "2", "--opponent-pool-size", "2",
              "--strong-checkpoints", "1", "--evaluation-episodes", "1", "--device", "cpu",
              "--output", str(out), "--opponent", "offense"])
    history = json.loads((out / "generation-history.json").read_text())
    assert [g["generation"] for g in history["generations"]] == [1, 2]
    record = history["generations"][-1]
    assert "deterministic_offense" in record["opponent_metrics"]
    assert "error" not in record["opponent_metrics"]["deterministic_offense"]
    population = json.loads((out / "opponent-population" / "population.json").read_text())
    assert population["capacity"] == 2 and population["strong_elites"] == 1
    assert len(population["members"]) == 2
    capsys.readouterr()
