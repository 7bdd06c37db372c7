"""Deployment boundary: SafePolicyRunner fallbacks and limits (CPU)."""
import json
import math
import subprocess
from pathlib import Path

import pytest

from autodrive_b200.deploy import (ChassisCommand, Objective, Obstacle, RobotParameters, RobotState,
                                   SafePolicyRunner, WorldState)

ROOT = Path(__file__).resolve().parents[1]


class Const:
    def __init__(self, cmd):
        self.cmd = cmd
        self.calls = 0

    def predict(self, state, params, goal):
        self.calls += 1
        if isinstance(self.cmd, Exception):
            raise self.cmd
        return self.cmd


def _state(t=100., x=8., y=4., theta=0., obstacles=()):
    return WorldState(RobotState(x, y, theta), RobotState(3., 3., 0.), t, 16.54, 8.07, obstacles)


def _runner(cmd, now=100., **kw):
    return SafePolicyRunner(Const(cmd), RobotParameters(), clock=lambda: now, **kw)


def test_policy_command_is_rate_limited():
    r = _runner(ChassisCommand(4., 0., 8.))
    out = r.predict(_state(), Objective(1., 1.))
    assert out.reason == "policy"
    assert out.constrained.vx == pytest.approx(8. * .02)        # max_acceleration * dt
    assert out.constrained.omega == pytest.approx(18. * .02)    # max_alpha * dt
    for _ in range(200):
        out = r.predict(_state(), Objective(1., 1.))
    assert out.constrained.vx == pytest.approx(4.)
    assert out.constrained.omega == pytest.approx(8.)


def test_planar_speed_is_capped():
    r = _runner(ChassisCommand(10., 10., 0.))
    for _ in range(500):
        out = r.predict(_state(), Objective(1., 1.))
    assert math.hypot(out.constrained.vx, out.constrained.vy) == pytest.approx(4.8, rel=1e-6)


@pytest.mark.parametrize("ts,reason", [(99.8, "stale-state"), (100.2, "stale-state"),
                                        (float("nan"), "stale-state")])
def test_stale_state_falls_back(ts, reason):
    pol = Const(ChassisCommand(1., 0., 0.))
    r = SafePolicyRunner(pol, RobotParameters(), clock=lambda: 100.)
    out = r.predict(_state(t=ts), Objective(1., 1.), manual=ChassisCommand(0., .5, 0.))
    assert out.reason == reason and pol.calls == 0
    assert out.raw == ChassisCommand(0., .5, 0.)


def test_invalid_state_and_output_and_errors():
    bad = _state(obstacles=(Obstacle(1., 1., -1.),))
    assert _runner(ChassisCommand(1., 0., 0.)).predict(bad, Objective(1., 1.)).reason == "invalid-output"
    out = _runner(ChassisCommand(float("inf"), 0., 0.)).predict(_state(), Objective(1., 1.))
    assert out.reason == "invalid-output" and out.constrained == ChassisCommand()
    out = _runner(RuntimeError("boom")).predict(_state(), Objective(1., 1.),
                                                manual=ChassisCommand(float("nan"), 0., 0.))
    assert out.reason == "policy-error" and out.raw == ChassisCommand()


def test_wall_guard_keeps_tangential_motion():
    r = _runner(ChassisCommand(-1., 1., 0.))
    for _ in range(50):
        out = r.predict(_state(x=.4), Objective(1., 1.))
    assert out.constrained.vx == 0. and out.constrained.vy == pytest.approx(1.)


def test_logger_and_validation():
    logs = []
    r = _runner(ChassisCommand(1., 0., 0.), logger=logs.append)
    r.predict(_state(), Objective(1., 1.))
    assert logs and logs[0]["reason"] == "policy"
    with pytest.raises(ValueError):
        RobotParameters(max_speed=0.)
    with pytest.raises(ValueError):
        Objective(0., 0., radius=0.)
    with pytest.raises(ValueError):
        SafePolicyRunner(Const(ChassisCommand()), RobotParameters(), dt=0.)


def test_compat_import_paths():
    from frc_defense.runtime import SafePolicyRunner as S2
    from frc_defense.types import ChassisCommand as C2
    assert S2 is SafePolicyRunner and C2 is ChassisCommand


def test_ops_files(tmp_path):
    cfg = json.loads((ROOT / "config" / "drivetrain.generic.example.json").read_text())
    from autodrive_b200.sim.world import SwerveParameters
    SwerveParameters(**cfg["swerve"])
    assert cfg["robot_length"] > 0 and "randomize" in cfg
    unit = (ROOT / "ops" / "frc-defense-training.service").read_text()
    assert "Restart=on-failure" in unit and "run_training.sh" in unit
    script = ROOT / "ops" / "run_training.sh"
    assert subprocess.run(["bash", "-n", str(script)]).returncode == 0
    usage = subprocess.run(["bash", str(script)], capture_output=True, text=True)
    assert usage.returncode == 2 and "usage" in usage.stderr
