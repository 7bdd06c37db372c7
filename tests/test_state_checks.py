"""State validation of the simulator kernels (option `state_checks`): a
corrupted world state is reported in a per-environment status word and made
harmless instead of being indexed with or propagated (host twin here; the GPU
test runs a clean batch with the checks on)."""
import pytest
import torch

from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
from autodrive_b200.sim.world import SimulationStateError


def test_corrupted_state_is_reported_and_sanitised():
    env = TensorThreeVsThreeEnv(num_envs=3, device="cpu", seed=1, fuel_physics=True, state_checks=True)
    ws = env.ws
    active = ws["f_active"][0].nonzero().reshape(-1)
    ws["f_owner"][0, active[0]] = 17                      # an owner index past the robots
    ws["f_vel"][1, 0, active[1]] = float("nan")           # a NaN FUEL velocity
    ws["r_vel"][2, 4, 1] = float("inf")                   # a non-finite robot velocity
    ws["f_pos"][2, 0, active[2]] = 40.                    # a piece far outside the field
    env.step(None)
    with pytest.raises(SimulationStateError, match="3 environment"):
        env.check_state()
    assert env.check_state()["environments"] == []       # cleared by the read
    assert int(ws["f_owner"][0, active[0]]) == -1
    assert not bool(ws["f_active"][1, active[1]]) and not bool(ws["f_active"][2, active[2]])
    for name in ("f_pos", "f_vel", "r_pose", "r_vel"):
        t = ws[name]
        assert torch.isfinite(t[ws["f_active"].bool().unsqueeze(1).expand_as(t)] if name.startswith("f")
                              else t).all(), name


def test_clean_batch_reports_nothing():
    env = TensorThreeVsThreeEnv(num_envs=2, device="cpu", seed=2, fuel_physics=True, state_checks=True)
    env.step_held(None, 5)
    assert env.check_state()["environments"] == []


@pytest.mark.gpu
def test_state_checks_on_the_gpu_kernels():
    """The validation pass inside the GPU tick kernel: a clean batch reports
    nothing, and a piece moved 40 m outside the field (finite values, so every
    index computed from it stays clamped) is reported and deactivated."""
    env = TensorThreeVsThreeEnv(num_envs=64, device="cuda", seed=3, fuel_physics=True, state_checks=True)
    env.step_held(None, 10)
    assert env.check_state()["environments"] == []
    piece = int(env.ws["f_active"][5].nonzero()[0])
    env.ws["f_pos"][5, 0, piece] = 40.
    env.step_held(None, 2)
    report = env.check_state(raise_error=False)
    assert report["environments"] == [5] and "outside the field" in report["problems"][5][0]
    assert not bool(env.ws["f_active"][5, piece])
