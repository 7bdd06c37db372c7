"""Device-resident environment state and the parameter block shared by kernels.

`WorldState` allocates one torch tensor per entry of the extension's schema
(``csrc/world.h``) and binds them to a native ``Sim`` handle. Every public
environment attribute (``piece_pos``, ``sim.pose`` ...) is a view into these
tensors, so Python, checkpoints and the dashboard see exactly what the kernels
see.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, asdict

import torch

from .. import field as fieldmod
from ..ops import require_extension

_DTYPES = {0: torch.float32, 1: torch.int32, 2: torch.uint8, 3: torch.int8, 4: torch.float64}

ROBOT_PARAMS = ("length", "width", "mass", "speed", "accel", "omega_limit", "alpha",
                "drive_ratio", "drive_current_limit", "drive_supply_limit",
                "robot_supply_limit", "battery_resistance", "lateral_mu",
                "yaw_inertia_multiplier")
# Multiplicative domain-randomisation ranges per robot parameter
# (frc_defense/tensor_physics.py:312-345); the same ranges keep training
# distributions comparable between simulators.
RANDOM_RANGES = {
    "length": (.82, 1.2), "width": (.82, 1.2), "mass": (.65, 1.45), "speed": (.75, 1.3),
    "accel": (.65, 1.4), "omega_limit": (.7, 1.3), "alpha": (.65, 1.4),
    "drive_ratio": (.9, 1.1), "drive_current_limit": (.75, 1.25),
    "drive_supply_limit": (.75, 1.25), "robot_supply_limit": (.8, 1.2),
    "battery_resistance": (.7, 1.6), "lateral_mu": (.8, 1.25),
    "yaw_inertia_multiplier": (.8, 1.2),
}
ENV_MU_RANGES = ((.25, 1.1), (.35, 1.2), (.25, 1.1))  # bumper, ground, wall


@dataclass(frozen=True)
class SwerveParameters:
    """Drivetrain constants (defaults: Kraken X60, 6.75:1, 4 in wheel)."""
    wheel_radius: float = .0508
    drive_ratio: float = 6.75
    drive_current_limit: float = 60.
    drive_supply_current_limit: float = 80.
    robot_supply_current_limit: float = 180.
    steer_current_limit: float = 20.
    steer_rate_limit: float = 12.
    steer_acceleration: float = 80.
    motor_efficiency: float = .9
    battery_voltage: float = 12.6
    battery_internal_resistance: float = .018
    stall_torque_nm: float = 7.09
    stall_current_a: float = 366.
    free_speed_rpm: float = 6000.
    free_current_a: float = 2.
    nominal_voltage: float = 12.
    module_x_offset: float = .36
    module_y_offset: float = .36


TensorSwerveParameters = SwerveParameters


@dataclass
class FuelPhysicsConfig:
    """FUEL contact model options (frc_defense/fuel_physics.py:22-81).

    ``backend`` selects ``"cuda"`` (the fused sm_100a tick kernel; default on
    CUDA devices), ``"host"`` (the same routines on CPU threads) or ``"auto"``.
    Options that only tune the reference's pair-list caching (``cache``,
    ``skin``, ``max_neighbors``, ``contact_mode``, ``compact_capacity``,
    ``broadphase``, ``robot_broadphase``) are accepted for compatibility: the
    kernel rebuilds an exact uniform grid every substep, so they do not change
    results. ``sleep_islands`` sleeps and wakes whole contact islands.
    ``solver="colored"`` is rejected (the kernel's solver is Jacobi).
    """
    radius: float = .075
    mass: float = .215
    substeps: int = 10
    gravity: float = 9.81
    stiffness: float = 2000.
    damping: float = 40.
    friction: float = .45
    rolling_friction: float = .20
    robot_height: float = .5
    broadphase: str = "grid"
    robot_broadphase: str = "all_pairs"
    cache: bool = True
    skin: float = .075
    max_neighbors: int = 64
    contact_mode: str = "fused"
    compact_capacity: str = "bounded"
    solver: str = "jacobi"
    backend: str = "auto"
    sleep: bool = True
    sleep_islands: bool = False
    sleep_time: float = .5
    sleep_speed: float = .025
    sleep_angular_speed: float = .5
    adaptive_substeps: bool = True
    max_adaptive_substeps: int = 64
    gpu_qualifying: bool = False
    max_compression_fraction: float = .5
    max_translation_per_substep: float | None = None
    grid_cell: float = .2

    def __post_init__(self):
        for name, choices in (("broadphase", ("grid", "all_pairs")),
                              ("robot_broadphase", ("grid", "all_pairs")),
                              ("contact_mode", ("compact", "fused")),
                              ("compact_capacity", ("bounded", "full")),
                              ("solver", ("jacobi", "colored")),
                              ("backend", ("auto", "torch", "hip", "cuda", "host"))):
            if getattr(self, name) not in choices:
                raise ValueError(f"{name} must be one of {choices}")
        if (not isinstance(self.substeps, int) or isinstance(self.substeps, bool)
                or not isinstance(self.max_neighbors, int)):
            raise ValueError("substeps and max_neighbors must be integers")
        if (not isinstance(self.max_adaptive_substeps, int) or isinstance(self.max_adaptive_substeps, bool)
                or self.max_adaptive_substeps < 1):
            raise ValueError("max_adaptive_substeps must be a positive integer")
        numeric = (self.radius, self.mass, self.gravity, self.stiffness, self.damping, self.friction,
                   self.rolling_friction, self.robot_height, self.skin, self.sleep_time,
                   self.sleep_speed, self.sleep_angular_speed, self.max_compression_fraction)
        if not all(math.isfinite(float(v)) for v in numeric):
            raise ValueError("fuel coefficients must be finite")
        if not 0 < self.max_compression_fraction <= 1:
            raise ValueError("max_compression_fraction must be in (0,1]")
        if self.radius <= 0 or self.mass <= 0 or self.substeps < 1 or self.max_neighbors < 1:
            raise ValueError("positive radius, mass, substeps and max_neighbors required")
        if min(self.skin, self.stiffness, self.damping, self.friction, self.rolling_friction,
               self.sleep_time, self.sleep_speed, self.sleep_angular_speed) < 0:
            raise ValueError("contact and sleep coefficients must be nonnegative")
        if self.grid_cell < 2 * self.radius:
            raise ValueError("grid_cell must be at least the sphere diameter")
        if self.solver == "colored":
            raise ValueError("solver='colored' (sequential colour passes) is not available: the FUEL kernel "
                             "solves contacts with owner-computes Jacobi; use solver='jacobi'")

    @property
    def effective_substeps(self) -> int:
        """Substeps per controller tick (adaptive mode runs its fixed upper bound)."""
        return self.max_adaptive_substeps if self.adaptive_substeps else self.substeps


def fuel_config(value) -> FuelPhysicsConfig | None:
    if value is False or value is None:
        return None
    if value is True:
        return FuelPhysicsConfig()
    if isinstance(value, FuelPhysicsConfig):
        return value
    if isinstance(value, dict):
        return FuelPhysicsConfig(**value)
    raise ValueError("fuel_physics must be True, False, a dict or FuelPhysicsConfig")


def build_params(*, n: int, robots: int, pieces: int, dt: float, field_length: float,
                 field_width: float, boxes, bumps, hubs, team, mode, role, kind, capacity,
                 score_interval, fuel: FuelPhysicsConfig | None, swerve: SwerveParameters,
                 contact_iterations: int = 3, field_sweep_spacing: float = .02,
                 base_speed: float = 4.8, base_omega: float = 8., base_length: float = .9,
                 base_width: float = .9, seed: int = 0, **extra) -> dict:
    """Assemble the SimParams dictionary consumed by the extension."""
    fuel_on = fuel is not None
    fc = fuel or FuelPhysicsConfig()
    # swept field contacts: increments per substep from the worst-case motion
    substeps = fc.effective_substeps if fuel_on else 1
    h = dt / substeps
    radius = .5 * math.hypot(base_length * 1.2, base_width * 1.2)
    motion = (base_speed * 1.3 + base_omega * 1.3 * radius) * h
    sweep = max(1, math.ceil(motion / field_sweep_spacing))
    cell = fc.grid_cell
    seed = int(seed) & 0xFFFFFFFFFFFF
    p = dict(
        n=n, R=robots, P=pieces, substeps=substeps, contact_iterations=contact_iterations,
        sweep_steps=sweep, dt=dt, field_length=field_length, field_width=field_width,
        alliance_depth=fieldmod.ALLIANCE_ZONE_DEPTH,
        boxes=[list(b) for b in boxes], bumps=[list(b) for b in bumps],
        hub_x=[hubs[0][0], hubs[1][0]], hub_y=[hubs[0][1], hubs[1][1]],
        team=list(team), mode=list(mode), role=list(role), kind=list(kind),
        capacity=list(capacity), score_interval=list(score_interval),
        wheel_radius=swerve.wheel_radius, steer_current_limit=swerve.steer_current_limit,
        steer_rate_limit=swerve.steer_rate_limit, steer_acceleration=swerve.steer_acceleration,
        motor_efficiency=swerve.motor_efficiency, battery_voltage=swerve.battery_voltage,
        stall_torque=swerve.stall_torque_nm, stall_current=swerve.stall_current_a,
        free_speed_rpm=swerve.free_speed_rpm, free_current=swerve.free_current_a,
        nominal_voltage=swerve.nominal_voltage, module_x=swerve.module_x_offset,
        module_y=swerve.module_y_offset,
        fuel_physics=1 if fuel_on else 0, fr=fc.radius, fm=fc.mass, fk=fc.stiffness, fg=fc.gravity,
        fc=fc.damping, fmu=fc.friction, froll=fc.rolling_friction, robot_height=fc.robot_height,
        max_comp=fc.max_compression_fraction, sleep=1 if fc.sleep else 0,
        sleep_islands=1 if (fc.sleep and fc.sleep_islands) else 0,
        sleep_time=fc.sleep_time, sleep_speed=fc.sleep_speed, sleep_ang=fc.sleep_angular_speed,
        grid_cell=cell, grid_nx=math.ceil(field_length / cell), grid_ny=math.ceil(field_width / cell),
        colored_solver=1 if fc.solver == "colored" else 0,
        seed0=seed & 0xFFFFFFFF, seed1=(seed >> 32) & 0xFFFF | 0x5EED0000,
    )
    p.update(extra)
    return p


STATUS_BITS = {1: "FUEL owner outside [-1, robots) cleared", 2: "non-finite FUEL state (piece deactivated)",
               4: "FUEL outside the field (piece deactivated)",
               8: "non-finite robot pose / velocity / command (zeroed)"}


class SimulationStateError(RuntimeError):
    """The state validation of the simulator kernels found invalid entries."""


def state_checks_default() -> bool:
    import os
    return os.environ.get("AUTODRIVE_STATE_CHECKS", "0") == "1"


def check_state(ws: "WorldState", clear: bool = True, raise_error: bool = True) -> dict:
    """Read the per-environment status words of the state validation (the
    `state_checks` environment option), decode them and clear them; raises
    SimulationStateError when any environment reported a problem."""
    words = ws["e_status"].reshape(-1)
    hit = (words != 0).nonzero().reshape(-1).tolist()
    report = {"environments": hit, "problems": {}}
    for e in hit:
        w = int(words[e])
        report["problems"][e] = [msg for bit, msg in STATUS_BITS.items() if w & bit]
    if clear:
        words.zero_()
    if hit and raise_error:
        raise SimulationStateError(f"invalid simulator state in {len(hit)} environment(s): "
                                   f"{dict(list(report['problems'].items())[:4])}")
    return report


class WorldState:
    """All state tensors of a batch of environments plus the native handle."""

    def __init__(self, params: dict, device: torch.device):
        ext = require_extension()
        self.params = params
        self.device = torch.device(device)
        if self.device.type == "cuda" and not torch.cuda.is_available():
            raise RuntimeError(f"Requested accelerator {device!r} is unavailable; refusing CPU simulation")
        self.schema = ext.schema(params["n"], params["R"], params["P"])
        self.t: dict[str, torch.Tensor] = {}
        tensors = []
        for name, code, shape in self.schema:
            tensor = torch.zeros(tuple(shape), dtype=_DTYPES[code], device=self.device)
            self.t[name] = tensor
            tensors.append(tensor)
        self.sim = ext.Sim(tensors, params)
        self.t["active"].fill_(1)

    def __getitem__(self, name: str) -> torch.Tensor:
        return self.t[name]

    def state_dict(self) -> dict:
        return {name: tensor.detach().clone() for name, tensor in self.t.items()}

    def load_state_dict(self, state: dict) -> None:
        for name, tensor in state.items():
            self.t[name].copy_(tensor)
