"""sm_100a simulator kernels against their host twins (same routines, serial).

The GPU path runs with fast-math transcendentals and a different summation
order in the FUEL grid, so states are compared with tolerances after one tick;
discrete game state must match exactly.
"""
import pytest
import torch

from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv

pytestmark = pytest.mark.gpu


def _pair(n, fuel, seed=11):
    cpu = TensorThreeVsThreeEnv(num_envs=n, device="cpu", seed=seed, fuel_physics=fuel)
    gpu = TensorThreeVsThreeEnv(num_envs=n, device="cuda:0", seed=seed, fuel_physics=fuel)
    gpu.ws.load_state_dict({k: v.to("cuda:0") for k, v in cpu.ws.state_dict().items()})
    return cpu, gpu


@pytest.mark.parametrize("fuel", [False, True])
def test_one_tick_matches_host(fuel):
    cpu, gpu = _pair(4, fuel)
    a = torch.full((4, 6), 7, dtype=torch.long)
    cpu.step(a)
    gpu.step(a.cuda())
    torch.cuda.synchronize()
    for name, atol in (("r_pose", 2e-4), ("r_vel", 2e-3), ("f_pos", 2e-4), ("f_vel", 5e-3), ("obs", 2e-3)):
        c, g = cpu.ws[name], gpu.ws[name].cpu()
        assert torch.allclose(c, g, atol=atol, rtol=1e-3), (name, (c - g).abs().max())
    for name in ("f_owner", "g_rcount", "g_action", "g_scores", "p_len"):
        assert torch.equal(cpu.ws[name], gpu.ws[name].cpu()), name


def test_graph_replay_matches_eager():
    eager = TensorThreeVsThreeEnv(num_envs=8, device="cuda:0", seed=5, fuel_physics=True)
    graph = TensorThreeVsThreeEnv(num_envs=8, device="cuda:0", seed=5, fuel_physics=True)
    a = torch.full((8, 6), 7, dtype=torch.int32, device="cuda:0")
    for _ in range(3):
        o1, r1, _ = eager.step_held(a, 12, use_graph=False)
        o2, r2, _ = graph.step_held(a, 12, use_graph=True)
    torch.cuda.synchronize()
    assert torch.equal(eager.ws["g_steps"], graph.ws["g_steps"])
    assert torch.allclose(o1, o2, atol=1e-5)
    assert torch.allclose(r1, r2)


def test_full_batch_runs_and_scores():
    env = TensorThreeVsThreeEnv(num_envs=64, device="cuda:0", seed=2, fuel_physics=True)
    a = torch.full((64, 6), 7, dtype=torch.int32, device="cuda:0")
    for _ in range(40):
        obs, rew, _ = env.step_held(a, 20)
    torch.cuda.synchronize()
    assert torch.isfinite(obs).all()
    assert int(env.fuel_acquisition_count.sum()) > 0
    assert float(env.match_elapsed[0]) == pytest.approx(16.0, abs=1e-3)
