"""Scripted offense collection on the host twins: raster route, sweeping,
cluster collection with contour tracing, and the no-track search target
(frc_defense/_tensor_3v3_actions.py:677-890, _tensor_3v3_navigation.py)."""
import math

import torch

from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv

RL_TARGET_COLLECTING = 5


def make(**kw):
    return TensorThreeVsThreeEnv(num_envs=1, device="cpu", seed=4, fuel_physics=False, **kw)


def test_raster_routes_are_closed_even_loops_in_each_alliance_half():
    env = make()
    pts = env.ws["raster_pts"]
    assert pts.shape == (6, 256, 2)
    step = (pts.roll(-1, dims=1) - pts).norm(dim=-1)
    assert float(step.max()) < 1.5 * float(step.mean())       # even arc-length spacing, closed
    assert float(pts[..., 1].min()) >= .5 and float(pts[..., 1].max()) <= env.field_width - .5  # U-turn overshoot
    mid = env.field_length / 2
    assert bool((pts[:3, :, 0] < mid).all()) and bool((pts[3:, :, 0] > mid).all())
    assert bool((pts[:3, :, 0] > env.alliance_zone_depth).all())


def test_sweeping_offense_follows_its_raster_route():
    env = make(sweeping_enabled=True)
    a = torch.full((1, 6), 7, dtype=torch.long)
    for _ in range(30):
        env.step(a, capture_observation=False, capture_info=False)
    ws = env.ws
    cursor = ws["c_raster"][0, :3]
    assert bool((cursor > 0).all())                  # scripted offense robots track their cursor
    target = ws["c_target"][0, 0]
    route = ws["raster_pts"][0]
    assert float((route - target).norm(dim=-1).min()) < 1e-5   # the target is a route sample
    assert int(ws["c_raster"][0, 3:].abs().sum()) == 0          # defenders never use the route


def _clear_tracks(env):
    ws = env.ws
    for name in ("t_pos", "t_vel", "t_conf", "t_mask"):
        ws[name].zero_()
    ws["t_age"].fill_(float("inf"))


def test_no_track_search_heads_for_the_raster_route():
    env = make()
    ws = env.ws
    ws["f_active"].zero_()          # nothing to see: every robot empty-handed, no tracks
    ws["f_owner"].fill_(-1)
    _clear_tracks(env)
    ws.sim.control(env._actions_buf)
    route = ws["raster_pts"][0]
    target = ws["c_target"][0, 0]
    assert float((route - target).norm(dim=-1).min()) < 1e-5
    assert int(ws["g_rlatch"][0, 0, 6]) == 1        # no-track search


def test_cluster_collection_traces_the_contour():
    env = make()
    ws = env.ws
    _clear_tracks(env)
    pose = ws["policy_pose"][0, 0]
    x, y, th = float(pose[0]), float(pose[1]), float(pose[2])
    fx, fy = math.cos(th), math.sin(th)
    # a tight cluster just ahead of robot 0's intake, seen by robot 0
    for k in range(6):
        ws["t_pos"][0, 0, 0, k] = x + fx * (1.0 + .12 * (k % 3)) - fy * (.12 * (k // 3))
        ws["t_pos"][0, 0, 1, k] = y + fy * (1.0 + .12 * (k % 3)) + fx * (.12 * (k // 3))
        ws["t_mask"][0, 0, k] = 1
        ws["t_age"][0, 0, k] = 0.
        ws["t_conf"][0, 0, k] = .9
    ws["g_rlatch"][0, 0].zero_()
    ws.sim.control(env._actions_buf)
    assert int(ws["g_action"][0, 0]) < 4                       # collecting a candidate
    assert int(ws["g_rlatch"][0, 0, RL_TARGET_COLLECTING]) == 1  # entered the cluster
    target = ws["c_target"][0, 0]
    p = ws["policy_pose"][0, 0, :2]
    heading = float(ws["c_collect_heading"][0, 0])
    along = torch.tensor((math.cos(heading), math.sin(heading)))
    # contour tracing: 3 m ahead along the (turn-limited) collect heading
    assert abs(float((target - p).norm()) - 3.) < 1e-3
    assert float(((target - p) / 3. - along).norm()) < 1e-3
