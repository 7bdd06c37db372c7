"""Grid route planner on the host twin: PathPlanner-style line-of-sight
simplification and Bezier corner smoothing (frc_defense/tensor_adstar.py:772-1037)."""
import math

import torch

from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv


def _route(start, goal, heading=0.):
    env = TensorThreeVsThreeEnv(num_envs=1, device="cpu", seed=2, fuel_physics=False)
    ws = env.ws
    for k in range(6):      # park everyone else far away
        ws["policy_pose"][0, k] = torch.tensor((15.8, .6 + 1.35 * k, math.pi))
    ws["policy_pose"][0, 0] = torch.tensor((start[0], start[1], heading))
    ws["r_pose"].copy_(ws["policy_pose"])
    ws["o_valid"].zero_()
    ws["g_rlatch"].zero_()
    ws["c_target"][0, 0] = torch.tensor(goal)
    ws.sim.plan(1)
    n = int(ws["p_len"][0, 0])
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
