"""Physical invariants of the FUEL contact model on the simulator core.

The cases follow the reference's property tests (tests/test_fuel_physics.py:
43-300 in the reference: rolling loss on carpet, airborne fall and damped
rebound, ball-ball energy dissipation, wall reversal, horizontal momentum
conservation, robot push with momentum transfer and yaw, a sleeping pile that
wakes on impact, masked worlds, no tunnelling, no frictional energy creation)
and run the host twin of the tick kernel (the same `csrc` routines the GPU
runs), one world of the REBUILT field with the test spheres on open carpet in
the red alliance zone and the six robots parked in the neutral zone.
"""
import math

import pytest
import torch

from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
from autodrive_b200.sim.world import FuelPhysicsConfig

R = .075
PARK_X = (5.9, 6.9, 7.9, 8.9, 9.9, 10.7)


class World:
    def __init__(self, pieces=2, worlds=1, modes=("none",) * 6, **options):
        self.cfg = FuelPhysicsConfig(**options)
        # robots without a controller are parked (pose restored, velocity zeroed) after every tick
        self.env = TensorThreeVsThreeEnv(num_envs=worlds, device="cpu", seed=0, control_modes=modes,
                                         fuel_count=96, fuel_physics=self.cfg, randomize=False, allow_nn_offense=True)
        ws = self.ws = self.env.ws
        self.pieces = pieces
        ws["f_active"].zero_()
        ws["f_active"][:, :pieces] = 1
        ws["f_owner"].fill_(-1)
        for name in ("f_vel", "f_ang", "f_sleep", "f_clock"):
            ws[name].zero_()
        ws["f_pos"][:, 0, :pieces] = 2.4 + .4 * torch.arange(pieces, dtype=torch.float32)
        ws["f_pos"][:, 1, :pieces] = 2.8
        ws["f_pos"][:, 2, :pieces] = R
        ws["f_pos"][:, :, pieces:] = torch.tensor([8.27, 4.035, R])[:, None]
        pose = ws["r_pose"]
        pose.zero_()
        pose[..., 0] = torch.tensor(PARK_X)
        pose[..., 1] = 4.04
        ws["r_vel"].zero_()
        ws["c_command"].zero_()

    # [worlds, pieces, 3] views like the reference's FuelPhysics attributes
    pos = property(lambda self: self.ws["f_pos"][:, :, :self.pieces].transpose(1, 2))
    vel = property(lambda self: self.ws["f_vel"][:, :, :self.pieces].transpose(1, 2))
    angular = property(lambda self: self.ws["f_ang"][:, :, :self.pieces].transpose(1, 2))
    sleeping = property(lambda self: self.ws["f_sleep"][:, :self.pieces].bool())

    def set(self, name, piece, xyz, world=0):
        self.ws[name][world, :, piece] = torch.as_tensor(xyz, dtype=torch.float32)

    def advance(self, ticks=1):
        self.ws.sim.physics(ticks)


def test_fuel_rolls_and_loses_speed_on_carpet():
    w = World(pieces=1)
    w.set("f_vel", 0, (1., 0., 0.))
    x0 = w.pos[0, 0, 0].item()
    w.advance()
    assert w.angular[0, 0].norm().item() > 0
    w.advance(24)
    assert w.pos[0, 0, 0].item() > x0
    assert 0 <= w.vel[0, 0, 0].item() < 1.
    assert w.pos[0, 0, 2].item() >= R * .5


def test_carpet_rolling_resistance_settles_released_fuel():
    w = World(pieces=1)
    w.set("f_vel", 0, (.5, 0., 0.))
    w.advance(40)
    assert w.vel[0, 0, :2].norm().item() < .04


def test_airborne_fuel_falls_and_rebounds_with_damping():
    w = World(pieces=1)
    w.ws["f_pos"][0, 2, 0] = .5
    rebounds = []
    for _ in range(60):
        w.advance()
        if w.vel[0, 0, 2].item() > .05:
            rebounds.append(w.vel[0, 0, 2].item())
        assert torch.isfinite(w.ws["f_pos"]).all()
        assert w.pos[0, 0, 2].item() >= R * .5
    assert rebounds, "floor contact must produce a damped rebound"
    assert max(rebounds) < 1., "foam-ball impacts dissipate most of the impact energy"


def test_ball_ball_impact_dissipates_kinetic_energy():
    w = World(pieces=2, gravity=0., friction=0., rolling_friction=0., sleep=False)
    w.set("f_pos", 0, (3., 3., R))
    w.set("f_pos", 1, (3.14, 3., R))
    w.set("f_vel", 0, (1., 0., 0.))
    w.set("f_vel", 1, (-1., 0., 0.))
    before = w.vel.square().sum().item()
    w.advance()
    assert w.vel.square().sum().item() < before * .5


def test_wall_collision_reverses_approach_velocity():
    w = World(pieces=1)
    w.set("f_pos", 0, (R + .01, 3., R))
    w.set("f_vel", 0, (-2., 0., 0.))
    w.advance(3)
    assert w.vel[0, 0, 0].item() > 0
    assert w.pos[0, 0, 0].item() >= R - 1e-5


def test_contact_conserves_horizontal_momentum_without_external_friction():
    w = World(pieces=2, gravity=0., friction=0., rolling_friction=0., sleep=False)
    w.set("f_pos", 0, (3., 3., R))
    w.set("f_pos", 1, (3.15, 3., R))
    w.set("f_vel", 0, (1., 0., 0.))
    p0 = w.vel[..., :2].sum(1).clone()
    e0 = w.vel.square().sum().item()
    w.advance(10)
    torch.testing.assert_close(w.vel[..., :2].sum(1), p0, rtol=1e-5, atol=1e-5)
    assert w.vel[0, 1, 0].item() > .1
    assert w.vel.square().sum().item() <= e0 + 1e-4
    assert w.pos[0, 1, 0] > w.pos[0, 0, 0]


def _push(with_ball: bool, pieces=1, offset=.2):
    w = World(pieces=pieces, modes=("nn",) + ("none",) * 5, gravity=0., friction=0., rolling_friction=0.,
              sleep=False)
    ws = w.ws
    ws["r_pose"][0, 0] = torch.tensor([2.6, 2.8, 0.])
    ws["r_vel"][0, 0] = torch.tensor([3., 0., 0.])
    ws["c_command"][0, 0] = torch.tensor([3., 0., 0.])
    if with_ball:
        ys = torch.linspace(2.8 - .35, 2.8 + .35, pieces) if pieces > 1 else torch.tensor([2.8 + offset])
        for k in range(pieces):
            w.set("f_pos", k, (3.1, float(ys[k]), R))
    else:
        ws["f_active"].zero_()
    w.advance()
    return w


def test_robot_push_transfers_momentum_and_generates_yaw():
    free = _push(False)
    hit = _push(True)
    ball_v = hit.vel[0, 0, :2]
    assert ball_v[0].item() > 0
    robot_free, robot_hit = free.ws["r_vel"][0, 0], hit.ws["r_vel"][0, 0]
    assert robot_hit[0].item() < robot_free[0].item()
    # contact ahead-left turns the chassis positively (the drive's heading hold
    # then damps the yaw rate within the tick, so the heading records the turn)
    assert hit.ws["r_pose"][0, 0, 2].item() > free.ws["r_pose"][0, 0, 2].item() + 1e-7
    # the momentum the ball gained is the robot's deficit against the same tick
    # without contact (the drive keeps pushing toward 3 m/s, so within 25 %)
    mass = hit.ws["r_param"][0, 0, 2].item()
    deficit = mass * (robot_free[:2] - robot_hit[:2])
    gained = hit.cfg.mass * ball_v
    assert deficit[0].item() == pytest.approx(gained[0].item(), rel=.25)


def test_a_row_of_fuel_resists_a_robot_more_than_one_ball():
    free, single, row = _push(False), _push(True, offset=0.), _push(True, pieces=6)
    v0 = free.ws["r_vel"][0, 0, 0].item()
    single_loss = v0 - single.ws["r_vel"][0, 0, 0].item()
    row_loss = v0 - row.ws["r_vel"][0, 0, 0].item()
    assert single_loss > 0
    assert row_loss > single_loss * 2


@pytest.mark.parametrize("islands", [False, True])
def test_sleeping_pile_wakes_and_transmits_an_impact(islands):
    w = World(pieces=4, sleep=True, sleep_time=.04, sleep_islands=islands)
    for k, x in enumerate((3., 3.15, 3.30, 3.45)):
        w.set("f_pos", k, (x, 3., R))
    w.advance(50)
    assert w.sleeping.all()
    w.set("f_vel", 0, (2., 0., 0.))
    w.advance(4)
    assert not w.sleeping[0, 0]
    assert w.vel[0, 1:, 0].max().item() > .02
    assert torch.isfinite(w.ws["f_pos"]).all()


def test_island_sleep_keeps_a_touching_group_awake_together():
    """A resting sphere that touches a spinning one (spin about the vertical
    axis, which the floor does not brake) sleeps on its own in per-sphere
    mode but stays awake in island mode, where its island is never quiet."""
    def run(islands):
        w = World(pieces=2, sleep=True, sleep_time=.04, sleep_islands=islands, rolling_friction=0.)
        w.set("f_pos", 0, (3., 3., R))
        w.set("f_pos", 1, (3. + 2 * R - 1e-5, 3., R))
        w.set("f_ang", 1, (0., 0., 5.))
        w.advance(5)
        return w.sleeping[0].tolist()
    assert run(False) == [True, False]
    assert run(True) == [False, False]


def test_inactive_worlds_and_held_or_inactive_fuel_do_not_move():
    w = World(pieces=3, worlds=2)
    ws = w.ws
    ws["f_owner"][0, 1] = 0
    ws["f_active"][0, 2] = 0
    ws["f_vel"][:, 0, :3] = 1.
    before = {k: ws[k].clone() for k in ("f_pos", "f_vel", "f_ang")}
    robots = ws["r_vel"].clone()
    ws["active"][1] = 0
    w.advance(4)
    for k, b in before.items():
        torch.testing.assert_close(ws[k][1], b[1], rtol=0, atol=0)
        torch.testing.assert_close(ws[k][0, :, 1:3], b[0, :, 1:3], rtol=0, atol=0)
    torch.testing.assert_close(ws["r_vel"][1], robots[1], rtol=0, atol=0)
    assert ws["f_pos"][0, 0, 0] > before["f_pos"][0, 0, 0]


def test_grid_resolution_does_not_change_contacts():
    """The broadphase is exact: a 0.2 m and a 0.6 m grid give identical
    trajectories for a moving cluster (the reference compares its grid and
    all-pairs broadphases)."""
    g = torch.Generator().manual_seed(907)
    pos = torch.rand((12, 3), generator=g)
    pos[:, :2] = pos[:, :2] * .5 + 2.6
    pos[:, 2] = R
    vel = torch.randn((12, 3), generator=g) * .4
    vel[:, 2] = 0.
    out = []
    for cell in (.2, .6):
        w = World(pieces=12, sleep=False, grid_cell=cell)
        w.ws["f_pos"][0, :, :12] = pos.T
        w.ws["f_vel"][0, :, :12] = vel.T
        w.advance(8)
        out.append({k: w.ws[k].clone() for k in ("f_pos", "f_vel", "f_ang")})
    for k in out[0]:
        torch.testing.assert_close(out[0][k], out[1][k], rtol=2e-4, atol=2e-4)


def test_fast_fuel_does_not_tunnel_through_another_ball():
    w = World(pieces=2, gravity=0., friction=0., rolling_friction=0., sleep=False)
    w.set("f_pos", 0, (3., 3., R))
    w.set("f_pos", 1, (3.16, 3., R))
    w.set("f_vel", 0, (25., 0., 0.))
    w.set("f_vel", 1, (-25., 0., 0.))
    w.advance()
    assert w.pos[0, 0, 0].item() < w.pos[0, 1, 0].item(), "fast spheres must not pass through each other"
    assert w.vel[0, 0, 0].item() < 25.
    torch.testing.assert_close(w.vel[..., :2].sum(1), torch.zeros((1, 2)), atol=1e-4, rtol=0)


def test_frictional_collision_creates_no_translational_or_spin_energy():
    w = World(pieces=2, gravity=0., friction=10., rolling_friction=0., sleep=False)
    w.set("f_pos", 0, (3., 3., R))
    w.set("f_pos", 1, (3.15, 3., R))
    w.set("f_vel", 0, (1., 1., 0.))
    w.ws["f_ang"][0, 2, :2] = 10.
    inertia = .4 * w.cfg.mass * R * R

    def energy():
        return (.5 * w.cfg.mass * w.vel.square().sum() + .5 * inertia * w.angular.square().sum()).item()
    e0 = energy()
    for _ in range(6):
        w.advance()
        assert energy() <= e0 + 1e-5
    assert energy() < e0
    assert w.vel[0, 1, :2].norm().item() > 0


def test_colored_solver_is_rejected():
    with pytest.raises(ValueError, match="colored"):
        FuelPhysicsConfig(solver="colored")


def test_gravity_option_reaches_the_kernel():
    w = World(pieces=1, gravity=0., sleep=False)
    w.ws["f_pos"][0, 2, 0] = .5
    w.advance(5)
    assert w.pos[0, 0, 2].item() == pytest.approx(.5, abs=1e-6)
    g = World(pieces=1, sleep=False)
    g.ws["f_pos"][0, 2, 0] = .5
    g.advance(5)
    assert g.pos[0, 0, 2].item() < .5 - .5 * 9.81 * (.1 ** 2) * .8
    assert math.isfinite(g.pos[0, 0, 2].item())
