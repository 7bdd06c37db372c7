"""Parity against the reference implementation as an independent oracle.

The reference package (installed unmodified in ``baseline/_ref``; these tests
skip when it is absent) is imported read-only and run on its own CPU PyTorch
path. Identical states are loaded into both simulators and advanced with the
same inputs; the simulator core here runs its host twin (the same routines
the sm_100a kernels run). Compared:

* swerve drivetrain trajectories of a driven robot (pose and velocity, 10
  and 25 ticks), a head-on robot-robot contact and a robot driving into the
  field wall (frc_defense/tensor_physics.py:347-514);
* FUEL contacts after whole ticks of 64 substeps: a head-on pair, an oblique
  pair with spin and friction, an airborne sphere, and a six-sphere pile
  (frc_defense/fuel_physics.py:384-664);
* the REBUILT HUB schedule over the whole match for every AUTO outcome
  (frc_defense/_tensor_3v3_gamepieces.py:148-179).
"""
import os
import subprocess
import sys
import tempfile
import textwrap

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "frc_defense")),
                                reason="the reference is not installed in baseline/_ref")

PARK = [(15.8, .6 + 1.35 * k, 0.) for k in range(6)]
R = .075


def _run_reference(body: str, **inputs):
    """Run `body` in a fresh interpreter that imports only the reference
    package (this repository's ``frc_defense`` compatibility package shares
    its name); `inputs` arrive as variables and the snippet's `out` dict is
    returned."""
    with tempfile.TemporaryDirectory() as tmp:
        src, dst = os.path.join(tmp, "in.pt"), os.path.join(tmp, "out.pt")
        torch.save(inputs, src)
        script = ("import sys, torch\nsys.path.insert(0, %r)\n" % REF +
                  "globals().update(torch.load(%r, weights_only=False))\n" % src +
                  textwrap.dedent(body) + "\ntorch.save(out, %r)\n" % dst)
        proc = subprocess.run([sys.executable, "-c", script], cwd=tmp, capture_output=True, text=True,
                              timeout=600, env={**os.environ, "PYTHONPATH": REF})
        assert proc.returncode == 0, proc.stderr[-3000:]
        return torch.load(dst, weights_only=False)


def _robot_pair(starts, commands, ticks):
    """Advance both simulators `ticks` ticks from the same six robot poses at
    rest under constant chassis commands; returns (ours, reference) as
    [6, 6] tensors of pose + velocity."""
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    ours = TensorThreeVsThreeEnv(num_envs=1, device="cpu", seed=0, control_modes=("nn",) * 6, fuel_physics=False,
                                 randomize=False, allow_nn_offense=True, fuel_count=96)
    ws = ours.ws
    ws["f_active"].zero_()
    cmd = torch.tensor(commands, dtype=torch.float32)[None]
    for k in range(6):
        ws["r_pose"][0, k] = torch.tensor(starts[k])
    ws["r_vel"].zero_()
    for _ in range(ticks):
        ws["c_command"].copy_(cmd)
        ws.sim.physics(1)
    ref = _run_reference("""
        from frc_defense.tensor_physics import TensorVectorizedSimulator
        sim = TensorVectorizedSimulator(
            num_envs=1, device="cpu", dt=.02, field_length=16.54, field_width=8.07, robot_length=p[0],
            robot_width=p[1], mass=p[2], max_speed=p[3], max_acceleration=p[4], max_omega=p[5], max_alpha=p[6],
            lateral_friction=p[12], yaw_inertia_multiplier=p[13], num_robots=6, randomize=False,
            bumper_friction=mu[0], field_friction=mu[1])
        sim.pose[0] = starts
        sim.velocity.zero_()
        for _ in range(ticks):
            sim.step(cmd.clone())
        out = {"state": torch.cat((sim.pose[0], sim.velocity[0]), -1)}
    """, p=ws["r_param"][0, 0].tolist(), mu=ws["e_mu"][0].tolist(), starts=torch.tensor(starts),
        cmd=cmd, ticks=ticks)
    return torch.cat((ws["r_pose"][0], ws["r_vel"][0]), -1), ref["state"]


def test_swerve_trajectory_matches_reference():
    starts = list(PARK)
    starts[0] = (3.0, 2.5, .3)
    cmds = [[0., 0., 0.]] * 6
    cmds[0] = [2.0, 1.0, .8]
    ours, ref = _robot_pair(starts, cmds, 10)
    torch.testing.assert_close(ours[0], ref[0], rtol=0, atol=1e-3)
    ours, ref = _robot_pair(starts, cmds, 25)
    torch.testing.assert_close(ours[0, :3], ref[0, :3], rtol=0, atol=5e-3)
    torch.testing.assert_close(ours[0, 3:], ref[0, 3:], rtol=0, atol=3e-2)


def test_head_on_robot_contact_matches_reference():
    starts = list(PARK)
    starts[0], starts[1] = (7.0, 4.0, 0.), (8.2, 4.05, 0.)
    cmds = [[0., 0., 0.]] * 6
    cmds[0], cmds[1] = [2., 0., 0.], [-2., 0., 0.]
    ours, ref = _robot_pair(starts, cmds, 30)
    torch.testing.assert_close(ours[:2], ref[:2], rtol=0, atol=1e-3)


def test_wall_contact_matches_reference():
    starts = list(PARK)
    starts[0] = (1.0, 6.8, .2)
    cmds = [[0., 0., 0.]] * 6
    cmds[0] = [0., 2.5, 0.]
    ours, ref = _robot_pair(starts, cmds, 30)
    torch.testing.assert_close(ours[0], ref[0], rtol=0, atol=1e-3)


def _fuel_pair(setup, ticks, **options):
    """Advance both FUEL models from the same sphere states (robots parked in
    the neutral zone, no field boxes near the spheres)."""
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    from test_fuel_physics import World
    n = len(setup)
    ours = World(pieces=n, **options)
    for k, (pos, vel, ang) in enumerate(setup):
        ours.set("f_pos", k, pos)
        ours.set("f_vel", k, vel)
        ours.set("f_ang", k, ang)
    ours.advance(ticks)
    ref = _run_reference("""
        from types import SimpleNamespace
        from frc_defense.fuel_physics import FuelPhysics, FuelPhysicsConfig
        sim = SimpleNamespace(dt=.02, field_length=16.54, field_width=8.07, pose=torch.zeros((1, 6, 3)),
                              velocity=torch.zeros((1, 6, 3)), length=torch.full((1, 6), .9),
                              width=torch.full((1, 6), .9), mass=torch.full((1, 6), 55.),
                              yaw_inertia_multiplier=torch.full((1, 6), 1.5),
                              field_colliders=torch.empty((0, 4)), bump_regions=torch.empty((0, 4)))
        sim.pose[0, :, 0] = torch.tensor((5.9, 6.9, 7.9, 8.9, 9.9, 10.7))
        sim.pose[0, :, 1] = 4.04
        n = len(setup)
        ph = FuelPhysics(sim, torch.zeros((1, n, 2)), torch.zeros((1, n, 2)),
                         config=FuelPhysicsConfig(backend="torch", **options))
        for k, (pos, vel, ang) in enumerate(setup):
            ph.pos[0, k] = torch.tensor(pos)
            ph.vel[0, k] = torch.tensor(vel)
            ph.angular[0, k] = torch.tensor(ang)
        for _ in range(ticks):
            ph.step(torch.ones(1, dtype=torch.bool), torch.ones((1, n), dtype=torch.bool), torch.full((1, n), -1))
        out = {"pos": ph.pos.clone(), "vel": ph.vel.clone(), "angular": ph.angular.clone(),
               "substeps": ph.required_substeps()}
    """, setup=setup, ticks=ticks, options=options)
    assert ref["substeps"] == ours.ws.params["substeps"] == 64
    return ours, ref


def _assert_same_fuel(ours, ref, atol):
    for name in ("pos", "vel", "angular"):
        torch.testing.assert_close(getattr(ours, name), ref[name], rtol=0, atol=atol)


def test_fuel_head_on_pair_matches_reference():
    ours, ref = _fuel_pair([((3., 3., R), (1., 0., 0.), (0., 0., 0.)), ((3.15, 3., R), (0., 0., 0.), (0., 0., 0.))],
                           1, gravity=0., friction=0., rolling_friction=0., sleep=False)
    _assert_same_fuel(ours, ref, 1e-4)


def test_fuel_oblique_pair_with_spin_and_friction_matches_reference():
    ours, ref = _fuel_pair([((3., 3., R), (1., .3, 0.), (0., 0., 4.)),
                            ((3.14, 3.02, R), (-.5, 0., 0.), (0., 0., 0.))], 3)
    _assert_same_fuel(ours, ref, 2e-4)


def test_airborne_fuel_matches_reference():
    ours, ref = _fuel_pair([((3., 3., .4), (.5, 0., 0.), (0., 0., 0.))], 10)
    _assert_same_fuel(ours, ref, 2e-4)


def test_fuel_pile_matches_reference():
    offsets = ((0., 0.), (.13, 0.), (0., .13), (.13, .13), (.065, .065), (.26, .065))
    setup = [((3. + dx, 3. + dy, R), (.4 if k == 0 else 0., 0., 0.), (0., 0., 0.))
             for k, (dx, dy) in enumerate(offsets)]
    ours, ref = _fuel_pair(setup, 2, sleep=False)
    _assert_same_fuel(ours, ref, 5e-4)


def test_hub_schedule_matches_reference_for_every_auto_outcome():
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    n = 4
    ours = TensorThreeVsThreeEnv(num_envs=n, device="cpu", seed=0, control_modes=("none",) * 6,
                                 fuel_physics=False, randomize=False)
    auto = torch.tensor([[3, 1], [1, 3], [2, 2], [0, 0]])
    times = [k * .5 + .013 for k in range(322)]
    ref = _run_reference("""
        from frc_defense.tensor_3v3 import TensorThreeVsThreeEnv
        env = TensorThreeVsThreeEnv(num_envs=4, device="cpu", seed=0, control_modes=("none",) * 6,
                                    fuel_physics=False, randomize=False)
        active = torch.ones(4, dtype=torch.bool)
        rows = []
        for t in times:
            env.match_elapsed.fill_(t)
            env.auto_fuel_scores.copy_(auto)
            env._update_match(active)
            rows.append(env.hub_active.clone())
        out = {"hub": torch.stack(rows)}
    """, times=times, auto=auto)
    for k, t in enumerate(times):
        ours.ws["g_time"][:, 0] = t
        ours.ws["g_scores"][:, :2] = auto.int()
        ours.step(None, capture_observation=False, capture_info=False)
        assert torch.equal(ref["hub"][k], ours.hub_active), t
