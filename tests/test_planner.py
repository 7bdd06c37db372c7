"""Grid route planner on the host twin: PathPlanner-style line-of-sight
simplification and Bezier corner smoothing (frc_defense/tensor_adstar.py:772-1037)."""
import math

import pytest
import torch

from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv


def _route(start, goal, heading=0., resolution=.3, device="cpu"):
    env = TensorThreeVsThreeEnv(num_envs=1, device=device, seed=2, fuel_physics=False,
                                planner_resolution=resolution)
    ws = env.ws
    for k in range(6):      # park everyone else far away
        ws["policy_pose"][0, k] = torch.tensor((15.8, .6 + 1.35 * k, math.pi), device=ws.device)
    ws["policy_pose"][0, 0] = torch.tensor((start[0], start[1], heading), device=ws.device)
    ws["r_pose"].copy_(ws["policy_pose"])
    ws["o_valid"].zero_()
    ws["g_rlatch"].zero_()
    ws["c_target"][0, 0] = torch.tensor(goal, device=ws.device)
    ws.sim.plan(1)
    n = int(ws["p_len"][0, 0])
    env.sweeps = int(ws["p_sweeps"][0, 0])
    return env, ws["p_path"][0, 0][:n].clone(), ws["p_profile"][0, 0][:n].clone()


def test_route_around_the_hub_is_smooth_and_free():
    env, path, profile = _route((3.0, 2.2), (6.6, 5.8))
    assert path.shape[0] == 72
    assert float((path[0] - torch.tensor((3.0, 2.2))).norm()) < .3
    assert float((path[-1] - torch.tensor((6.6, 5.8))).norm()) < .3
    hub = next(b for b in env.field_boxes if b.name == "red_hub")
    inside = ((path[:, 0] - hub.x).abs() <= hub.length / 2) & ((path[:, 1] - hub.y).abs() <= hub.width / 2)
    assert not bool(inside.any())
    seg = path[1:] - path[:-1]
    keep = seg.norm(dim=-1) > 1e-4
    ang = torch.atan2(seg[keep, 1], seg[keep, 0])
    turn = torch.atan2(torch.sin(ang[1:] - ang[:-1]), torch.cos(ang[1:] - ang[:-1])).abs()
    # the smoothed corners bend gradually (a raw lattice corner turns 45 degrees in one step)
    assert float(turn.max()) < math.radians(30)
    step = seg.norm(dim=-1)
    assert float(step.max() - step.min()) < .02        # equal arc-length samples
    assert float(profile[-1]) == 0.0 and bool((profile >= 0).all())


def test_open_field_route_is_straight():
    _, path, _ = _route((7.0, 1.5), (9.5, 1.5))
    assert path.shape[0] == 72
    assert float((path[:, 1] - 1.5).abs().max()) < .2


def _inside_solid(env, pts):
    hit = torch.zeros(pts.shape[0], dtype=torch.bool)
    for b in env.field_boxes:
        if b.kind in ("hub", "tower", "upright", "support"):
            hit |= ((pts[:, 0] - b.x).abs() <= b.length / 2) & ((pts[:, 1] - b.y).abs() <= b.width / 2)
    return hit


def test_fine_grid_route_across_the_field_converges():
    """0.1 m grid (166 x 81 cells): a route from the red alliance zone around
    both hubs to the far blue side reaches its goal on free cells (the value
    iteration converges over the full field diameter)."""
    env, path, profile = _route((1.8, 6.5), (15.0, 1.7), resolution=.1)
    assert (env.ws.params["plan_nx"], env.ws.params["plan_ny"]) == (166, 81)
    assert 0 < env.sweeps < 60             # converged: a whole sweep changed no cell
    assert path.shape[0] == 72
    assert float((path[0] - torch.tensor((1.8, 6.5))).norm()) < .2
    assert float((path[-1] - torch.tensor((15.0, 1.7))).norm()) < .2
    assert not bool(_inside_solid(env, path).any())
    length = float((path[1:] - path[:-1]).norm(dim=-1).sum())
    assert 13.3 < length < 20.


@pytest.mark.gpu
@pytest.mark.parametrize("resolution", [.3, .1])
def test_gpu_routes_equal_host_twin(resolution):
    """The GPU planner (racing line sweeps, one CTA per route) converges like
    the serial host twin and returns the same route up to a few grid cells:
    the device build contracts multiply-adds into FMAs, so a cell exactly on
    an obstacle's inflated boundary (or a sample of a sight line or Bezier
    corner) can be classified differently, which moves a corner of the route
    by a cell or two or makes one side keep a less smoothed corner."""
    pairs = [((1.8, 6.5), (15.0, 1.7)), ((3.0, 2.2), (6.6, 5.8)), ((8.2, .6), (8.3, 7.4)),
             ((12.9, 4.0), (2.1, 4.0))]
    for start, goal in pairs:
        he, host, hp = _route(start, goal, resolution=resolution)
        de, dev, dp = _route(start, goal, resolution=resolution, device="cuda")
        assert he.sweeps > 0 and de.sweeps > 0, (he.sweeps, de.sweeps)
        assert dev.shape == host.shape
        dev = dev.cpu()
        assert float((dev[-1] - host[-1]).norm()) <= resolution * 1.01, (start, goal)
        assert float((dev - host).norm(dim=-1).max()) <= resolution * 3.01, (start, goal, he.sweeps, de.sweeps)
        lh = float((host[1:] - host[:-1]).norm(dim=-1).sum())
        ld = float((dev[1:] - dev[:-1]).norm(dim=-1).sum())
        assert abs(lh - ld) <= .15 * lh, (start, goal, lh, ld)
