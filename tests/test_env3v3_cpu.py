"""3v3 environment on the host twins: shapes, rules and invariants."""
import math

import torch

from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv, OBS_DIM


def make(n=2, fuel=False, **kw):
    return TensorThreeVsThreeEnv(num_envs=n, device="cpu", seed=3, fuel_physics=fuel, **kw)


def test_reset_shapes_and_layout():
    env = make()
    obs = env.ws["obs"]
    assert obs.shape == (2, 6, OBS_DIM)
    assert torch.isfinite(obs).all()
    # 48 depot + 408 neutral active, 48 reserved slots inactive
    assert int(env.piece_active[0].sum()) == 504 - 48
    assert bool(env.hub_active.all())
    assert float(env.match_remaining[0]) == 160.


def test_step_contract():
    env = make()
    a = torch.full((2, 6), 7, dtype=torch.long)
    obs, rew, done, trunc, info = env.step(a)
    assert obs.shape == (2, 6, OBS_DIM) and rew.shape == (2, 6)
    assert done.shape == (2,) and trunc.shape == (2,) and not bool(trunc.any())
    assert set(info) >= {"fuel_acquired_event", "team_score", "match_elapsed"}
    assert math.isclose(float(env.match_elapsed[0]), .02, rel_tol=1e-5)


def test_zero_sum_rewards_and_progress():
    env = make()
    a = torch.full((2, 6), 7, dtype=torch.long)
    total = torch.zeros(2, 6)
    for _ in range(150):
        _, rew, _, _, _ = env.step(a, capture_observation=False, capture_info=False)
        total += rew
    assert torch.allclose(total[:, :3].sum(-1), -total[:, 3:].sum(-1))
    assert int(env.fuel_acquisition_count.sum()) > 0  # scripted offense collects FUEL


def test_active_mask_freezes_worlds():
    env = make()
    a = torch.full((2, 6), 7, dtype=torch.long)
    before = env.sim.pose[1].clone()
    mask = torch.tensor([True, False])
    for _ in range(5):
        env.step(a, active_mask=mask)
    assert torch.equal(env.sim.pose[1], before)
    assert float(env.match_elapsed[1]) == 0.
    assert float(env.match_elapsed[0]) > 0.


def test_hub_schedule_alternates():
    env = make(n=1)
    el = env.ws["g_time"]
    a = torch.full((1, 6), 7, dtype=torch.long)
    seen = set()
    for t in (29.9, 35., 60., 85., 110., 135.):
        el[:, 0] = t - .02
        env.step(a, capture_observation=False)
        seen.add((t, tuple(env.hub_active[0].tolist())))
    states = dict(seen)
    assert states[29.9] == (True, True)
    assert states[35.] != (True, True)
    assert states[35.] != states[60.]
    assert states[135.] == (True, True)


def test_fuel_physics_keeps_pieces_in_field():
    env = make(fuel=True)
    a = torch.full((2, 6), 7, dtype=torch.long)
    for _ in range(20):
        env.step(a, capture_observation=False, capture_info=False)
    pos = env.fuel_physics.pos
    live = env.piece_active
    assert torch.isfinite(pos).all()
    assert bool((pos[..., 0][live] > -0.01).all() and (pos[..., 0][live] < 16.55).all())
    assert bool((pos[..., 2][live] > 0.).all())


def test_random_gamepiece_placement_and_rejected_obstacles():
    import pytest
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    a = TensorThreeVsThreeEnv(num_envs=2, device="cpu", seed=4, fuel_physics=False, random_gamepiece_placement=True)
    b = TensorThreeVsThreeEnv(num_envs=2, device="cpu", seed=4, fuel_physics=False)
    pa, pb = a.piece_pos, b.piece_pos
    act = a.piece_active
    assert not torch.equal(pa[0][act[0]], pb[0][act[0]])
    assert not torch.equal(pa[0][act[0]], pa[1][act[1]])          # each world draws its own layout
    d = torch.cdist(pa[0][act[0]], pa[0][act[0]]) + torch.eye(int(act[0].sum())) * 10
    assert float(d.min()) >= .159                                  # distinct lattice cells
    with pytest.raises(ValueError, match="obstacles"):
        TensorThreeVsThreeEnv(num_envs=1, device="cpu", fuel_physics=False, obstacles=((8., 4., .3),))
