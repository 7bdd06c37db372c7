"""Robot-side views and resets over the device-resident world state.

``RobotView`` exposes the attribute surface of the reference's
``TensorVectorizedSimulator`` (``pose``, ``velocity``, ``length`` ...,
frc_defense/tensor_physics.py:76-236) as views into the kernel state, so code
written against the reference reads the same names here.
"""
from __future__ import annotations

import math

import torch

from .world import ENV_MU_RANGES, RANDOM_RANGES, ROBOT_PARAMS, SwerveParameters, WorldState


class RobotView:
    def __init__(self, ws: WorldState, *, dt: float, field_length: float, field_width: float,
                 team_ids, boxes, bumps, swerve: SwerveParameters, base: dict, seed: int,
                 randomize: bool, obstacles=()):
        self.ws = ws
        self.n = ws.params["n"]
        self.num_robots = ws.params["R"]
        self.device = ws.device
        self.dt = float(dt)
        self.field_length, self.field_width = float(field_length), float(field_width)
        self.swerve = swerve
        self.randomize = bool(randomize)
        self._base = dict(base)
        self._team_ids_host = tuple(int(t) for t in team_ids)
        self.team_ids = torch.tensor(self._team_ids_host, device=self.device, dtype=torch.long)
        pairs = torch.triu_indices(self.num_robots, self.num_robots, offset=1, device=self.device)
        self._collision_pair_i, self._collision_pair_j = pairs[0], pairs[1]
        self.field_colliders = torch.tensor(boxes, dtype=torch.float32, device=self.device).reshape(-1, 4)
        self.bump_regions = torch.tensor(bumps, dtype=torch.float32, device=self.device).reshape(-1, 4)
        self.obstacles = torch.tensor(obstacles, dtype=torch.float32, device=self.device).reshape(-1, 3)
        self.generator = torch.Generator(device="cpu").manual_seed(int(seed or 0))
        self.contact_iterations = int(ws.params["contact_iterations"])

    # --- state views -------------------------------------------------------
    @property
    def pose(self) -> torch.Tensor:
        return self.ws["r_pose"]

    @property
    def velocity(self) -> torch.Tensor:
        return self.ws["r_vel"]

    def _param(self, name: str) -> torch.Tensor:
        return self.ws["r_param"][..., ROBOT_PARAMS.index(name)]

    length = property(lambda self: self._param("length"))
    width = property(lambda self: self._param("width"))
    mass = property(lambda self: self._param("mass"))
    speed = property(lambda self: self._param("speed"))
    accel = property(lambda self: self._param("accel"))
    omega_limit = property(lambda self: self._param("omega_limit"))
    alpha = property(lambda self: self._param("alpha"))
    drive_ratio = property(lambda self: self._param("drive_ratio"))
    drive_current_limit = property(lambda self: self._param("drive_current_limit"))
    lateral_mu = property(lambda self: self._param("lateral_mu"))
    yaw_inertia_multiplier = property(lambda self: self._param("yaw_inertia_multiplier"))
    mu = property(lambda self: self.ws["e_mu"][:, 0])
    ground_mu = property(lambda self: self.ws["e_mu"][:, 1])
    wall_mu = property(lambda self: self.ws["e_mu"][:, 2])
    module_angle = property(lambda self: self.ws["m_state"][:, :, 0])
    module_steer_rate = property(lambda self: self.ws["m_state"][:, :, 1])
    module_drive_speed = property(lambda self: self.ws["m_state"][:, :, 2])
    module_current = property(lambda self: self.ws["m_state"][:, :, 3])
    module_supply_current = property(lambda self: self.ws["m_state"][:, :, 4])
    robot_current = property(lambda self: self.ws["r_current"])
    robot_contact = property(lambda self: self.ws["e_flags"][:, 0].bool())
    opponent_contact = property(lambda self: self.ws["e_flags"][:, 1].bool())
    robot_contact_by_robot = property(lambda self: self.ws["r_flags"][:, :, 0].bool())
    field_contact = property(lambda self: self.ws["r_flags"][:, :, 1].bool())
    wall_contact = property(lambda self: self.ws["r_flags"][:, :, 2:4].bool())
    safety_active_physics_ticks = property(lambda self: self.ws["r_safety"][:, :, 0])
    safety_robot_contact_ticks = property(lambda self: self.ws["r_safety"][:, :, 1])
    safety_field_contact_ticks = property(lambda self: self.ws["r_safety"][:, :, 2])
    safety_wall_contact_ticks = property(lambda self: self.ws["r_safety"][:, :, 3])
    pair_contact_event_count = property(lambda self: self.ws["pair_count"][:, :, 0])
    pair_contact_solver_report_count = property(lambda self: self.ws["pair_count"][:, :, 1])
    pair_contact_first_substep = property(lambda self: self.ws["pair_substep"][:, :, 0])
    pair_contact_last_substep = property(lambda self: self.ws["pair_substep"][:, :, 1])
    pair_contact_impulse_sum = property(lambda self: self.ws["pair_impulse"])
    physics_substep_index = property(lambda self: self.ws["e_substep"])
    physics_time_s = property(lambda self: self.ws["e_phys_time"])

    # --- resets ------------------------------------------------------------
    def _rand(self, shape) -> torch.Tensor:
        return torch.rand(shape, generator=self.generator).to(self.device)

    def randomize_parameters(self, mask: torch.Tensor, nominal: bool = False) -> None:
        """Sample (or restore nominal) physical parameters for masked worlds."""
        mask = mask.to(self.device).bool().reshape(self.n)
        R = self.num_robots
        params = self.ws["r_param"]
        base = {
            "length": self._base["length"], "width": self._base["width"], "mass": self._base["mass"],
            "speed": self._base["speed"], "accel": self._base["accel"], "omega_limit": self._base["omega"],
            "alpha": self._base["alpha"], "drive_ratio": self.swerve.drive_ratio,
            "drive_current_limit": self.swerve.drive_current_limit,
            "drive_supply_limit": self.swerve.drive_supply_current_limit,
            "robot_supply_limit": self.swerve.robot_supply_current_limit,
            "battery_resistance": self.swerve.battery_internal_resistance,
            "lateral_mu": self._base["lateral_friction"],
            "yaw_inertia_multiplier": self._base["yaw_inertia_multiplier"],
        }
        for k, name in enumerate(ROBOT_PARAMS):
            if nominal or not self.randomize:
                value = torch.full((self.n, R), float(base[name]), device=self.device)
            else:
                lo, hi = RANDOM_RANGES[name]
                value = float(base[name]) * (lo + self._rand((self.n, R)) * (hi - lo))
            params[..., k] = torch.where(mask[:, None], value, params[..., k])
        mu_base = (self._base["bumper_friction"], self._base["field_friction"], self._base["field_friction"])
        for k in range(3):
            if nominal or not self.randomize:
                value = torch.full((self.n,), float(mu_base[k]), device=self.device)
            else:
                lo, hi = ENV_MU_RANGES[k]
                value = float(mu_base[k]) * (lo + self._rand((self.n,)) * (hi - lo))
            self.ws["e_mu"][:, k] = torch.where(mask, value, self.ws["e_mu"][:, k])
        # motor- and tire-limited acceleration cap
        sw = self.swerve
        torque_per_amp = sw.stall_torque_nm / sw.stall_current_a
        motor = (4 * torque_per_amp * self.drive_current_limit * self.drive_ratio * sw.motor_efficiency /
                 (sw.wheel_radius * self.mass).clamp_min(1e-6))
        tire = self.ground_mu[:, None] * 9.81
        accel = torch.minimum(self.accel, torch.minimum(motor, tire))
        params[..., ROBOT_PARAMS.index("accel")] = torch.where(mask[:, None], accel, self.accel)

    def clear_dynamics(self, mask: torch.Tensor) -> None:
        m = mask.to(self.device).bool()
        for name in ("r_vel", "m_state", "r_current", "r_flags", "r_safety", "pair_count",
                     "pair_time", "pair_impulse"):
            t = self.ws[name]
            t.masked_fill_(m.reshape((-1,) + (1,) * (t.ndim - 1)), 0)
        self.ws["pair_substep"].masked_fill_(m[:, None, None], -1)
        self.ws["e_flags"].masked_fill_(m[:, None], 0)
        self.ws["e_substep"].masked_fill_(m, 0)
        self.ws["e_phys_time"].masked_fill_(m, 0.)

    def nominal_reset(self) -> None:
        self.randomize_parameters(torch.ones(self.n, dtype=torch.bool), nominal=not self.randomize)


def hub_line_spawn_poses(view: RobotView, team_ids, alliance_depth: float, randomize: bool) -> torch.Tensor:
    """Six robots against their alliance's HUB-side zone line
    (frc_defense/tensor_3v3.py:428-451)."""
    n, R = view.n, view.num_robots
    dev = view.device
    pose = torch.zeros((n, R, 3), device=dev)
    offsets = torch.tensor((-2.685, 0., 2.665, -2.685, 0., 2.665), device=dev)[:R]
    team = torch.as_tensor(team_ids, device=dev)
    pose[:, :, 1] = view.field_width * .5 + offsets[None]
    pose[:, :, 2] = torch.where(team[None] == 0, 0., math.pi)
    if randomize:
        pose[:, :, 1] += (view._rand((n, R)) - .5) * .3
        pose[:, :, 2] += (view._rand((n, R)) - .5) * .2
    heading = pose[:, :, 2]
    support = .5 * view.length * heading.cos().abs() + .5 * view.width * heading.sin().abs()
    red = torch.full_like(support, alliance_depth)
    blue = torch.full_like(support, view.field_length - alliance_depth)
    face = torch.where(team[None] == 0, red, blue)
    pose[:, :, 0] = torch.where(team[None] == 0, face - support, face + support)
    return pose
