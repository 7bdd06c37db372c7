"""Two-robot counter-defense task and options (host twin).

The learner (slot 0) attacks; slot 1 is a scripted defender whose waypoint
comes from its own tracks of the attacker (intercept / lane block / FUEL
denial / shadow / HUB guard) and is reached through the route planner
(frc_defense/tensor_defense_step.py:108-180, tensor_defense_opponent.py:176-214).
"""
import math

import pytest
import torch

from autodrive_b200.sim.env_defense import TensorDefenseEnv


def _env(**kw):
    base = dict(num_envs=3, device="cpu", seed=3, fuel_physics=False, horizon=400)
    base.update(kw)
    return TensorDefenseEnv(**base)


def test_reference_defaults_are_counter_defense_with_a_guard():
    env = _env()
    assert env.task == "counter_defense" and env.defense_mode == "INTERCEPT"
    assert env.attacker == 0
    assert env.ws.params["counter_defense"] == 1 and env.ws.params["role"] == [0, 1]


@pytest.mark.parametrize("opponent,code", [("guard", 5), ("intercept", 5), ("cutoff", 5), ("lane_block", 6),
                                           ("fuel_denial", 7), ("shadow", 8), ("mirror", 8),
                                           ("hub_guard", 9), ("random", 4)])
def test_counter_defense_opponent_names(opponent, code):
    assert _env(opponent=opponent).ws.params["opponent_kind"] == code


def test_defense_mode_selects_the_guard_behaviour():
    env = _env(opponent="guard", defense_mode="hub_guard")
    assert env.ws.params["opponent_kind"] == 9
    with pytest.raises(ValueError, match="defense_mode"):
        _env(defense_mode="zone")
    with pytest.raises(ValueError, match="counter-defense"):
        _env(opponent="offense")


def test_scripted_defender_moves_to_its_waypoint_and_rewards_the_attacker():
    env = _env(opponent="hub_guard", randomize=False)
    env.reset(seed=3)
    # HUB guard: the waypoint sits in front of the attacker's (red) HUB on the lane to the attacker
    for _ in range(150):
        obs, reward, term, trunc, _ = env.step(torch.zeros(env.n, dtype=torch.long))
    hub = env.hub_centers[0]
    tracked = env.ws["o_valid"][:, 1].bool()
    target = env.ws["c_target"][:, 1]
    d_target_hub = (target - hub).norm(dim=-1)
    assert bool(tracked.any())
    assert bool(((d_target_hub[tracked] > .6) & (d_target_hub[tracked] < 2.)).all())
    moved = (env.ws["r_pose"][:, 1, :2] - target).norm(dim=-1)
    assert bool((moved[tracked] < 1.5).all())
    # strategic counter-defense reward: own scores + 0.05 x acquisitions - 0.001
    own = env.ws["g_rcount"][:, 0, 3].float()
    acq = env.ws["g_rcount"][:, 0, 2].float()
    torch.testing.assert_close(reward, own + .05 * acq - .001)


def test_observation_noise_and_dropout_touch_only_the_physical_features():
    clean = _env(observation_noise=0., observation_dropout=0.)
    noisy = _env(observation_noise=.05, observation_dropout=.3)
    a, _ = clean.reset(seed=9)
    b, _ = noisy.reset(seed=9)
    assert not torch.equal(a[:, :18], b[:, :18])
    torch.testing.assert_close(a[:, 18:], b[:, 18:])
    assert bool((b[:, :18] == 0).any())       # dropout zeroes some features


def test_goal_termination_in_direct_mode():
    env = _env(action_mode="direct", randomize=False, goal_radius=50.)
    env.reset(seed=1)
    _, reward, term, _, _ = env.step(torch.zeros((env.n, 3)))
    assert bool(term.all())                        # everything lies within 50 m of the objective
    assert bool((reward > 9.).all())                # counter-defense: +10 on reaching the objective


def test_uniform_fuel_layout_for_small_counts():
    env = _env(task="defense", opponent="offense", fuel_count=60, fuel_layout="uniform")
    env.reset(seed=2)
    pos = env.piece_pos
    assert pos.shape == (3, 60, 2) and bool(env.piece_active.all())
    assert float(pos[..., 0].min()) > 0 and float(pos[..., 0].max()) < 16.54
    assert not torch.equal(pos[0], pos[1])
    with pytest.raises(ValueError):
        _env(task="defense", opponent="offense", fuel_count=60)
    assert math.isfinite(float(env.step(torch.zeros(3, dtype=torch.long))[1].sum()))
