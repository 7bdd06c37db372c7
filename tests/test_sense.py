"""Anonymous stereo FUEL perception (host twin of the sense kernel).

Scenes are staged by hand in one 3v3 world: robot 0 looks along +x from the
neutral zone, the other robots are parked out of the way, and only the listed
FUEL pieces are active. Repeated sensor updates (each with a fresh tick key)
let the per-detection quality state ramp up until the tracks are written.
"""
import math

import pytest
import torch

from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv

_INF = float("inf")


def _stage(pieces, device="cpu", robot0=(7.0, 2.0, 0.0)):
    env = TensorThreeVsThreeEnv(num_envs=1, device=device, seed=5, fuel_physics=False)
    ws = env.ws
    pose = ws["r_pose"]
    pose[0, 0] = torch.tensor(robot0)
    for k in range(1, 6):
        pose[0, k] = torch.tensor((15.5, .8 + 1.2 * k, math.pi))
    ws["r_vel"].zero_()
    ws["f_active"].zero_()
    ws["f_owner"].fill_(-1)
    ws["f_vel"].zero_()
    for idx, (x, y) in pieces.items():
        ws["f_active"][0, idx] = 1
        ws["f_pos"][0, 0, idx] = x
        ws["f_pos"][0, 1, idx] = y
        ws["f_pos"][0, 2, idx] = .075
    for name in ("t_pos", "t_vel", "t_conf", "t_quality", "t_mask", "t_spatial", "t_angular", "t_merged",
                 "t_visible"):
        ws[name].zero_()
    ws["t_age"].fill_(_INF)
    return env


def _sense(env, updates=40):
    ws = env.ws
    for _ in range(updates):
        ws["e_episode"].add_(1)          # fresh counter key for every sensor update
        ws.sim.perceive()


def _tracks(env, robot=0):
    ws = env.ws
    live = ws["t_mask"][0, robot].bool().cpu()
    slots = live.nonzero().flatten().tolist()
    pos = ws["t_pos"][0, robot].cpu().T[live]
    return slots, pos


def test_separate_pieces_become_anonymous_tracks():
    pieces = {100: (8.6, 2.0), 200: (8.8, 2.9), 300: (9.4, 1.1)}
    env = _stage(pieces)
    _sense(env)
    slots, pos = _tracks(env)
    # three tracks in the first free slots: the tracker never sees piece indices
    assert slots == [0, 1, 2]
    truth = torch.tensor(list(pieces.values()))
    d = torch.cdist(pos, truth)
    assert (d.min(1).values < .15).all()   # measurement noise and the velocity estimate
    assert sorted(d.argmin(1).tolist()) == [0, 1, 2]
    ws = env.ws
    assert (ws["t_conf"][0, 0, :3] > 0).all()
    ext = ws["t_spatial"][0, 0, :, :3]
    assert (ext > .1).all() and (ext < .25).all()   # one FUEL diameter (+ lens spread)


def test_touching_pieces_merge_into_one_object():
    pieces = {7: (8.6, 2.0), 8: (8.6, 2.14)}
    env = _stage(pieces)
    _sense(env)
    slots, pos = _tracks(env)
    assert len(slots) == 1
    # both lenses' objects fused (the flag also marks a piece seen by both lenses)
    assert bool(env.ws["t_merged"][0, 0, slots[0]])
    # the object spans both pieces across the bearing
    assert float(env.ws["t_spatial"][0, 0, 1, slots[0]]) > .25
    assert abs(float(pos[0, 1]) - 2.07) < .15


def test_piece_hidden_behind_a_nearer_piece_is_not_reported():
    pieces = {3: (8.6, 2.0), 4: (9.4, 2.0)}
    env = _stage(pieces)
    _sense(env)
    slots, pos = _tracks(env)
    assert len(slots) == 1
    assert abs(float(pos[0, 0]) - 8.6) < .15


def test_rear_pair_sees_behind_and_range_limits():
    pieces = {10: (6.0, 2.0), 11: (7.0 - 7.0, 2.0)}   # one behind, one beyond 6 m
    env = _stage(pieces)
    _sense(env)
    slots, pos = _tracks(env)
    assert len(slots) == 1 and abs(float(pos[0, 0]) - 6.0) < .15


def test_tracks_keep_their_slot_while_observed():
    pieces = {100: (8.6, 2.0), 200: (8.8, 2.9)}
    env = _stage(pieces)
    _sense(env)
    before, _ = _tracks(env)
    _sense(env, updates=10)
    after, _ = _tracks(env)
    assert before == after == [0, 1]


def test_scripted_match_builds_bounded_track_sets():
    env = TensorThreeVsThreeEnv(num_envs=2, device="cpu", seed=9, fuel_physics=False)
    a = torch.full((2, 6), 7, dtype=torch.long)
    for _ in range(40):
        env.step(a, capture_observation=False, capture_info=False)
    live = env.ws["t_mask"].bool()
    assert int(live.sum()) > 0
    # anonymous detections fill slots from 0: no gaps larger than the live count
    for e in range(2):
        for r in range(6):
            n = int(live[e, r].sum())
            if n:
                assert int(live[e, r].nonzero().max()) < max(2 * n, 8)
    conf = env.ws["t_conf"][live]
    assert bool(((conf >= 0) & (conf <= 1)).all())


@pytest.mark.gpu
def test_sense_kernel_matches_host_twin():
    pieces = {100: (8.6, 2.0), 200: (8.8, 2.9), 300: (9.4, 1.1), 7: (8.2, 2.6), 8: (8.2, 2.74),
              9: (6.1, 1.7)}
    cpu = _stage(pieces)
    gpu = _stage(pieces, device="cuda:0")
    gpu.ws.load_state_dict({k: v.to("cuda:0") for k, v in cpu.ws.state_dict().items()})
    _sense(cpu, 25)
    _sense(gpu, 25)
    torch.cuda.synchronize()
    assert torch.equal(cpu.ws["t_mask"], gpu.ws["t_mask"].cpu())
    assert torch.equal(cpu.ws["t_merged"], gpu.ws["t_merged"].cpu())
    for name in ("t_pos", "t_spatial", "t_conf", "t_quality"):
        assert torch.allclose(cpu.ws[name], gpu.ws[name].cpu(), atol=2e-3, rtol=1e-3), name


@pytest.mark.parametrize("n", [1, 37, 256, 257, 600, 1280])
def test_bearing_rank_sort_is_a_stable_sort(n):
    from autodrive_b200.ops import require_extension
    g = torch.Generator().manual_seed(n)
    keys = (torch.rand(n, generator=g) * 2 - 1) * math.pi
    keys[::7] = keys[0]                      # ties resolve by index
    keys[1::11] = math.pi                    # the last bucket's edge
    order = require_extension().sense_rank_sort_host(keys)
    assert torch.equal(order, torch.sort(keys, stable=True).indices)
