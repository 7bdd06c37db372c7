"""Six-robot REBUILT match environment (`TensorThreeVsThreeEnv`).

Public surface mirrors frc_defense/tensor_3v3.py:33-1486: the constructor
keywords, ``reset(seed, defer_perception)``, ``reset_done(mask)``,
``step(actions, active_mask, capture_observation, capture_info)`` returning
``(obs[N,6,137], rewards[N,6], done[N], truncated[N], info)`` and
``observe(active_mask)``.

Execution: every tick is three native stages on the world's device — control
(targets), plan (routes on replanning ticks), tick (commands, all physics
substeps, game rules, perception, rewards) — plus observe when requested. On
CUDA each stage is one sm_100a kernel over the whole batch; a held decision
interval can be captured as one CUDA graph (``step_held``).
"""
from __future__ import annotations

import math

import torch

from .. import field as fieldmod
from ..utils import trace
from .robots import RobotView, hub_line_spawn_poses
from .world import (FuelPhysicsConfig, SwerveParameters, WorldState, build_params, check_state,
                    fuel_config, state_checks_default)

NUM_ROBOTS = 6
OBS_DIM = 137
ACTION_DIM = 8
TEAM_IDS = (0, 0, 0, 1, 1, 1)
CONTROL_MODES = ("none", "nn", "deterministic")
_MODE_CODE = {"none": 0, "nn": 1, "deterministic": 2}
_INF = 1e30


class FuelView:
    """Reference-compatible handle on the FUEL state (``env.fuel_physics``)."""

    def __init__(self, ws: WorldState, config: FuelPhysicsConfig):
        self.ws = ws
        self.config = config
        self.n, self.p = ws.params["n"], ws.params["P"]
        backend = "cuda" if ws.device.type == "cuda" else "host"
        self.stats = dict(backend=backend, substeps=ws.params["substeps"], rebuilds=0, overflows=0)

    pos = property(lambda self: self.ws["f_pos"].transpose(1, 2))
    vel = property(lambda self: self.ws["f_vel"].transpose(1, 2))
    angular = property(lambda self: self.ws["f_ang"].transpose(1, 2))
    sleeping = property(lambda self: self.ws["f_sleep"].bool())
    sleep_clock = property(lambda self: self.ws["f_clock"])

    def required_substeps(self, *_, **__):
        return self.ws.params["substeps"]

    def refresh_stats(self):
        return self.stats


class TensorThreeVsThreeEnv:
    """A batched 3v3 environment with per-robot controller assignments."""

    def __init__(self, num_envs=1, device="cuda", seed=0, *, control_modes=None,
                 robot_roles=None, robot_types=None, allow_nn_offense=False,
                 dt=.02, horizon=8000, randomize=True, fuel_count=504,
                 preloaded_per_robot=0, max_fuel_capacity=60,
                 max_scoring_bps=25.0, turret_fuel_capacity=40,
                 turret_scoring_bps=15.0, perception_interval=2, contact_iterations=3,
                 teammate_intent_knowledge=False, teammate_coordination_enabled=None,
                 sweeping_enabled=False, perception_range=6., perception_fov=120.,
                 stereo_baseline=.0635, fuel_ball_diameter=.15,
                 perception_dropout=.02, position_noise=.015,
                 velocity_noise=.05, replan_interval=20,
                 normalize_observations=True, fused_sensor_rng=False,
                 field_sweep_spacing=.02, behavior_probe=None, behavior_probe_robot=0,
                 behavior_probe_hub_active=True, random_gamepiece_placement=False,
                 field_length=16.54, field_width=8.07, obstacles=(), fuel_physics=True,
                 field_layout="2026_rebuilt", defer_initial_perception=False,
                 planner_resolution=.3, planner_sweeps=None, swerve=None, state_checks=None):
        self.n = int(num_envs)
        if self.n < 1:
            raise ValueError("num_envs must be positive")
        if horizon < 1 or dt <= 0:
            raise ValueError("horizon and dt must be positive")
        if not 96 + NUM_ROBOTS * preloaded_per_robot <= fuel_count <= 600:
            raise ValueError("fuel_count must include staging and six robot preloads")
        if not 0 <= preloaded_per_robot <= 8:
            raise ValueError("preloaded_per_robot must be between 0 and 8")
        if not 1 <= max_fuel_capacity <= fuel_count:
            raise ValueError("max_fuel_capacity must be between 1 and fuel_count")
        if not math.isfinite(max_scoring_bps) or max_scoring_bps <= 0:
            raise ValueError("max_scoring_bps must be finite and positive")
        if not 1 <= turret_fuel_capacity <= fuel_count:
            raise ValueError("turret_fuel_capacity must be between 1 and fuel_count")
        if not math.isfinite(turret_scoring_bps) or turret_scoring_bps <= 0:
            raise ValueError("turret_scoring_bps must be finite and positive")
        if behavior_probe is not None:
            raise ValueError("behavior probes are not supported by this simulator")
        if len(tuple(obstacles)):
            raise ValueError("static circular obstacles are not modelled by the 3v3 kernels; the field's "
                             "structures are the REBUILT layout's boxes")
        # the sensor noise/dropout draws always come from the in-kernel
        # counter-based generator (the reference's fused_sensor_rng=True path)
        self.fused_sensor_rng = True
        self.random_gamepiece_placement = bool(random_gamepiece_placement)
        self._placement_generator = torch.Generator(device="cpu").manual_seed(int(seed or 0) ^ 0x5A17)
        self.device = torch.device(device)
        self.dt, self.horizon = float(dt), int(horizon)
        self.field_length = float(field_length)
        self.field_width = float(field_width)
        self.alliance_zone_depth = float(fieldmod.ALLIANCE_ZONE_DEPTH)
        self.obs_dim, self.action_dim, self.action_kind = OBS_DIM, ACTION_DIM, "categorical"
        self.fuel_count = int(fuel_count)
        self.preloaded_per_robot = int(preloaded_per_robot)
        modes = list(control_modes or ("deterministic",) * NUM_ROBOTS)
        if len(modes) != NUM_ROBOTS or any(m not in CONTROL_MODES for m in modes):
            raise ValueError("control_modes must assign none, nn, or deterministic to six robots")
        roles = list(robot_roles or ("offense",) * 3 + ("defense",) * 3)
        if len(roles) != NUM_ROBOTS or any(r not in ("offense", "defense") for r in roles):
            raise ValueError("robot_roles must assign offense or defense to six robots")
        if not allow_nn_offense and any(m == "nn" and r != "defense" for m, r in zip(modes, roles)):
            raise ValueError("neural control is available only for defense-role robots")
        types = list(robot_types or ("dumper",) * NUM_ROBOTS)
        if len(types) != NUM_ROBOTS or any(t not in ("dumper", "turret") for t in types):
            raise ValueError("robot_types must assign dumper or turret to six robots")
        self.control_modes, self.robot_roles, self.robot_types = tuple(modes), tuple(roles), tuple(types)
        if teammate_coordination_enabled is None:
            teammate_coordination_enabled = teammate_intent_knowledge
        self.teammate_coordination_enabled = bool(teammate_coordination_enabled)
        self.sweeping_enabled = bool(sweeping_enabled)
        self.robot_fuel_capacity_values = tuple(
            int(turret_fuel_capacity if k == "turret" else max_fuel_capacity) for k in types)
        self.fuel_capacity = max(self.robot_fuel_capacity_values)
        self.robot_score_interval_values = tuple(
            1. / float(turret_scoring_bps if k == "turret" else max_scoring_bps) for k in types)
        self.perception_interval = max(1, int(perception_interval))
        self.replan_interval = max(1, int(replan_interval))
        self.perception_range = float(perception_range)
        self.perception_fov_degrees = float(perception_fov)
        self.perception_fov = math.radians(self.perception_fov_degrees) * .5
        self.perception_track_timeout = 2.0
        self.perception_dropout = float(perception_dropout)
        self.position_noise, self.velocity_noise = float(position_noise), float(velocity_noise)
        self.normalize_observations = bool(normalize_observations)
        self.randomize = bool(randomize)
        self.seed = int(seed or 0)
        self.field_layout_id = str(field_layout)
        self.field_boxes = fieldmod.qualification_field(self.field_layout_id, field_length, field_width)
        solids = fieldmod.static_collision_boxes(self.field_boxes)
        bumps = fieldmod.bump_boxes(self.field_boxes)
        self.field_feature_boxes = solids + bumps
        by_name = {b.name: b for b in self.field_boxes}
        hubs = [(by_name["red_hub"].x, by_name["red_hub"].y), (by_name["blue_hub"].x, by_name["blue_hub"].y)]
        self.fuel_config = fuel_config(fuel_physics)
        self.swerve = swerve or SwerveParameters()
        base = dict(length=.9, width=.9, mass=55., speed=9.6, accel=8., omega=16., alpha=18.,
                    bumper_friction=.65, field_friction=.7, lateral_friction=1.2,
                    yaw_inertia_multiplier=1.5)
        plan_nx = math.ceil(field_length / planner_resolution)
        plan_ny = math.ceil(field_width / planner_resolution)
        params = build_params(
            n=self.n, robots=NUM_ROBOTS, pieces=self.fuel_count, dt=self.dt,
            field_length=field_length, field_width=field_width,
            boxes=[b.as_tensor() for b in solids], bumps=[b.as_tensor() for b in bumps], hubs=hubs,
            team=TEAM_IDS, mode=[_MODE_CODE[m] for m in modes],
            role=[0 if r == "offense" else 1 for r in roles],
            kind=[0 if k == "dumper" else 1 for k in types],
            capacity=self.robot_fuel_capacity_values, score_interval=self.robot_score_interval_values,
            fuel=self.fuel_config, swerve=self.swerve, contact_iterations=contact_iterations,
            field_sweep_spacing=field_sweep_spacing, base_speed=base["speed"], base_omega=base["omega"],
            seed=self.seed,
            perception_interval=self.perception_interval, perception_range=self.perception_range,
            perception_fov=self.perception_fov, perception_dropout=self.perception_dropout,
            position_noise=self.position_noise, velocity_noise=self.velocity_noise,
            track_timeout=self.perception_track_timeout, ball_diameter=float(fuel_ball_diameter),
            stereo_baseline=float(stereo_baseline), replan_interval=self.replan_interval,
            teammate_coordination=int(self.teammate_coordination_enabled),
            normalize_obs=int(self.normalize_observations), horizon=self.horizon,
            plan_res=float(planner_resolution), plan_nx=plan_nx, plan_ny=plan_ny,
            checks=int(state_checks_default() if state_checks is None else bool(state_checks)),
            # directional line sweeps; the iteration stops at the first sweep
            # that changes no cell, so the budget only bounds pathological grids
            plan_sweeps=int(planner_sweeps if planner_sweeps is not None else 4 * (plan_nx + plan_ny)),
            fuel_radius_rules=.0825, stereo_tracks=1,
            sweeping=int(self.sweeping_enabled), raster_lookahead=20,
            depots=[d.as_tensor() for d in sorted(fieldmod.depot_boxes(self.field_boxes),
                                                   key=lambda b: b.alliance != "red")],
        )
        self.ws = WorldState(params, self.device)
        self.raster_sweep_points = torch.tensor(self._raster_route_points(), device=self.device,
                                                dtype=torch.float32)
        self.ws["raster_pts"].copy_(self.raster_sweep_points)
        self.sim = RobotView(self.ws, dt=self.dt, field_length=field_length, field_width=field_width,
                             team_ids=TEAM_IDS, boxes=[b.as_tensor() for b in solids],
                             bumps=[b.as_tensor() for b in bumps], swerve=self.swerve, base=base,
                             seed=self.seed, randomize=self.randomize, obstacles=obstacles)
        self.fuel_physics = FuelView(self.ws, self.fuel_config) if self.fuel_config else None
        self.team_ids = self.sim.team_ids
        self.hub_centers = torch.tensor(hubs, device=self.device, dtype=torch.float32)
        self._controlled_mode_mask = torch.tensor([m != "none" for m in modes], device=self.device)
        self.agent_train_mask = torch.tensor([m == "nn" for m in modes], device=self.device)
        self.robot_fuel_capacities = torch.tensor(self.robot_fuel_capacity_values, device=self.device)
        self.drivetrain_config = {"name": "built-in illustrative defaults", "randomize": self.randomize,
                                  "mass": 55.0, "robot_length": .9, "robot_width": .9,
                                  "max_speed": 9.6, "max_acceleration": 8.0, "max_omega": 16.0,
                                  "max_alpha": 18.0, "swerve": self.swerve.__dict__.copy()}
        self._initial_fuel = self._initial_fuel_layout()
        self._episode = 0
        self._graphs: dict = {}
        self._actions_buf = torch.full((self.n, NUM_ROBOTS), 7, device=self.device, dtype=torch.int32)
        self._last_obs = None
        self.reset(seed=seed, defer_perception=defer_initial_perception)

    # ------------------------------------------------------------------ views
    piece_pos = property(lambda self: self.ws["f_pos"][:, :2].transpose(1, 2))
    piece_vel = property(lambda self: self.ws["f_vel"][:, :2].transpose(1, 2))
    piece_active = property(lambda self: self.ws["f_active"].bool())
    piece_owner = property(lambda self: self.ws["f_owner"].long())
    piece_zone = property(lambda self: self.ws["f_zone"].long())
    match_elapsed = property(lambda self: self.ws["g_time"][:, 0])
    match_remaining = property(lambda self: self.ws["g_time"][:, 1])
    steps = property(lambda self: self.ws["g_steps"][:, 0].long())
    planner_ticks = property(lambda self: self.ws["g_steps"][:, 1].long())
    hub_active = property(lambda self: self.ws["g_hub"].bool())
    auto_fuel_scores = property(lambda self: self.ws["g_scores"][:, :2].long())
    fuel_score_count = property(lambda self: self.ws["g_scores"][:, 2:4].long())
    fuel_acquisition_count = property(lambda self: self.ws["g_rcount"][:, :, 0].long())
    fuel_denied_count = property(lambda self: self.ws["g_rcount"][:, :, 1].long())
    fuel_acquired_event = property(lambda self: self.ws["g_rcount"][:, :, 2].long())
    fuel_scored_event = property(lambda self: self.ws["g_rcount"][:, :, 3].long())
    fuel_passed_event = property(lambda self: self.ws["g_rcount"][:, :, 4].long())
    fuel_denied_event = property(lambda self: self.ws["g_rcount"][:, :, 5].long())
    last_actions = property(lambda self: self.ws["g_action"].long())
    policy_pose = property(lambda self: self.ws["policy_pose"])
    estimated_pose = property(lambda self: self.ws["est_pose"])
    track_pos = property(lambda self: self.ws["t_pos"].transpose(2, 3))
    track_vel = property(lambda self: self.ws["t_vel"].transpose(2, 3))
    track_mask = property(lambda self: self.ws["t_mask"].bool())
    track_age = property(lambda self: self.ws["t_age"])
    track_confidence = property(lambda self: self.ws["t_conf"])
    track_spatial_extent = property(lambda self: self.ws["t_spatial"].transpose(2, 3))
    track_angular_extent = property(lambda self: self.ws["t_angular"])
    track_merged = property(lambda self: self.ws["t_merged"].bool())
    perception_quality_state = property(lambda self: self.ws["t_quality"])
    _current_fuel_visibility = property(lambda self: self.ws["t_visible"].bool())
    opponent_pose = property(lambda self: self.ws["o_pose"])
    opponent_velocity = property(lambda self: self.ws["o_vel"])
    opponent_size = property(lambda self: self.ws["o_size"])
    opponent_valid = property(lambda self: self.ws["o_valid"].bool())
    opponent_age = property(lambda self: self.ws["o_age"])
    num_agents = property(lambda self: self.n * NUM_ROBOTS)

    @property
    def planner(self):
        return PlannerView(self.ws)

    # ------------------------------------------------------------ raster route
    def _raster_route_points(self, samples: int = 256):
        """Closed raster route of every robot, `samples` points evenly spaced by
        arc length (frc_defense/_tensor_3v3_navigation.py:13-82).

        Each alliance sweeps its own half of the neutral zone: two passes that
        span almost the whole field height (0.65 m from the walls) joined by
        cubic Bezier U-turns of radius 0.32 m whose control points overshoot
        the turn line by 0.55 radius, densified at 0.10 m on the passes and
        0.04 m on the turns before resampling.
        """
        width, length = self.field_width, self.field_length
        y_lo, y_hi, turn = .65, width - .65, .32
        x_near = self.alliance_zone_depth + .55
        x_far = length * .5 - .35
        routes = []
        for team in TEAM_IDS:
            if team == 0:
                xa, xb = x_near + turn, x_far - turn
            else:
                xa, xb = length - x_near - turn, length - x_far + turn
            pts = []

            def segment(a, b):
                n = max(2, math.ceil(math.dist(a, b) / .10))
                pts.extend((a[0] + (b[0] - a[0]) * k / n, a[1] + (b[1] - a[1]) * k / n) for k in range(n))

            def u_turn(a, c1, c2, b):
                n = max(8, math.ceil(math.dist(a, b) / .04))
                for k in range(n):
                    t = k / n
                    u = 1. - t
                    w = (u * u * u, 3. * u * u * t, 3. * u * t * t, t * t * t)
                    pts.append(tuple(w[0] * a[i] + w[1] * c1[i] + w[2] * c2[i] + w[3] * b[i] for i in (0, 1)))

            top_a, top_b = (xa, y_hi - turn), (xb, y_hi - turn)
            bot_a, bot_b = (xb, y_lo + turn), (xa, y_lo + turn)
            segment((xa, y_lo + turn), top_a)
            u_turn(top_a, (xa, y_hi + .55 * turn), (xb, y_hi + .55 * turn), top_b)
            segment(top_b, bot_a)
            u_turn(bot_a, (xb, y_lo - .55 * turn), (xa, y_lo - .55 * turn), bot_b)
            pts.append(pts[0])
            arc = [0.]
            for a, b in zip(pts, pts[1:]):
                arc.append(arc[-1] + math.dist(a, b))
            route, seg = [], 0
            for k in range(samples):
                s = arc[-1] * k / samples
                while seg + 1 < len(arc) - 1 and arc[seg + 1] < s:
                    seg += 1
                f = (s - arc[seg]) / max(arc[seg + 1] - arc[seg], 1e-9)
                a, b = pts[seg], pts[seg + 1]
                route.append((a[0] + (b[0] - a[0]) * f, a[1] + (b[1] - a[1]) * f))
            routes.append(route)
        return routes

    # ------------------------------------------------------------ fuel layout
    def _initial_fuel_layout(self):
        """Depot arrays, neutral midfield array and robot preloads
        (frc_defense/_tensor_3v3_gamepieces.py:80-138)."""
        P = self.fuel_count
        pos = torch.zeros((P, 2))
        active = torch.zeros(P, dtype=torch.bool)
        zone = torch.full((P,), -1, dtype=torch.int8)
        owner = torch.full((P,), -1, dtype=torch.int8)
        depots = {b.name: b for b in self.field_boxes if b.kind == "depot"}
        half = .075
        fw = self.sim.field_width
        for begin, name in ((0, "red_depot"), (24, "blue_depot")):
            d = depots[name]
            pts = fieldmod.grid_array_points(
                24, max(half, d.x - d.length / 2), min(self.field_length - half, d.x + d.length / 2),
                max(half, d.y - d.width / 2), min(fw - half, d.y + d.width / 2))
            pos[begin:begin + 24] = torch.tensor(pts)
        active[:48] = True
        zone[:24] = 1
        zone[24:48] = 2
        neutral = P - 96 - 6 * self.preloaded_per_robot
        if neutral:
            pts = fieldmod.grid_array_points(neutral, 8.27 - .915, 8.27 + .915, 4.035 - 2.615, 4.035 + 2.615)
            pos[96:96 + neutral] = torch.tensor(pts)
            active[96:96 + neutral] = True
            zone[96:96 + neutral] = 0
        preload_slots = []
        if self.preloaded_per_robot:
            for r in range(NUM_ROBOTS):
                b = P - 6 * self.preloaded_per_robot + r * self.preloaded_per_robot
                active[b:b + self.preloaded_per_robot] = True
                owner[b:b + self.preloaded_per_robot] = r
                zone[b:b + self.preloaded_per_robot] = 5
                preload_slots.append((r, b, b + self.preloaded_per_robot))
        return pos, active, zone, owner, preload_slots

    def _spawn_height(self, xy: torch.Tensor) -> torch.Tensor:
        r = self.fuel_config.radius if self.fuel_config else .075
        h = torch.full(xy.shape[:-1], r, device=xy.device)
        panel = fieldmod.BUMP_PANEL_THICKNESS
        rise = fieldmod.BUMP_RAMP_RISE
        for b in self.sim.bump_regions.tolist():
            dx = xy[..., 0] - b[0]
            within = (dx.abs() <= b[2]) & ((xy[..., 1] - b[1]).abs() <= b[3])
            terrain = panel + rise * (1 - dx.abs() / b[2])
            slope = -dx.sign() * rise / b[2]
            h = torch.where(within, h.maximum(terrain + r * (1 + slope.square()).sqrt()), h)
        return h

    # --------------------------------------------------------------- resets
    def _reset_worlds(self, mask: torch.Tensor) -> None:
        ws = self.ws
        m = mask.to(self.device).bool()
        self.sim.randomize_parameters(m)
        self.sim.clear_dynamics(m)
        pose = hub_line_spawn_poses(self.sim, TEAM_IDS, self.alliance_zone_depth, self.randomize)
        ws["r_pose"].copy_(torch.where(m[:, None, None], pose, ws["r_pose"]))
        ws["est_pose"].copy_(torch.where(m[:, None, None], ws["r_pose"], ws["est_pose"]))
        ws["policy_pose"].copy_(torch.where(m[:, None, None], ws["r_pose"], ws["policy_pose"]))
        pos, active, zone, owner, preload = self._initial_fuel
        P = self.fuel_count
        fpos = torch.zeros((self.n, 3, P), device=self.device)
        xy = pos.to(self.device)[None].expand(self.n, -1, -1).clone()
        if self.random_gamepiece_placement:
            # every staged piece on a random distinct cell of a whole-field
            # lattice spaced one diameter + 1 cm (frc_defense/tensor_defense_gamepieces.py:175-193)
            half = .075
            spacing = 2 * half + .01
            nx = int((self.field_length - 2 * half) // spacing) + 1
            ny = int((self.field_width - 2 * half) // spacing) + 1
            gx, gy = torch.meshgrid(half + torch.arange(nx) * spacing, half + torch.arange(ny) * spacing,
                                    indexing="ij")
            cells = torch.stack((gx.reshape(-1), gy.reshape(-1)), -1)
            staged = active & (owner < 0)
            count = int(staged.sum())
            order = torch.rand((self.n, cells.shape[0]), generator=self._placement_generator).argsort(-1)[:, :count]
            idx = staged.nonzero().squeeze(-1)
            xy[:, idx] = cells[order].to(self.device)
        for r, b, e in preload:
            xy[:, b:e] = ws["r_pose"][:, r, None, :2]
        fpos[:, 0] = xy[..., 0]
        fpos[:, 1] = xy[..., 1]
        fpos[:, 2] = self._spawn_height(xy)
        mm = m[:, None, None]
        ws["f_pos"].copy_(torch.where(mm, fpos, ws["f_pos"]))
        for name in ("f_vel", "f_ang"):
            ws[name].masked_fill_(mm, 0.)
        ws["f_clock"].masked_fill_(m[:, None], 0.)
        ws["f_sleep"].masked_fill_(m[:, None], 0)
        ws["f_active"].copy_(torch.where(m[:, None], active.to(self.device).to(torch.uint8)[None],
                                         ws["f_active"]))
        ws["f_owner"].copy_(torch.where(m[:, None], owner.to(self.device)[None], ws["f_owner"]))
        ws["f_zone"].copy_(torch.where(m[:, None], zone.to(self.device)[None], ws["f_zone"]))
        # game
        ws["g_time"][:, 0].masked_fill_(m, 0.)
        ws["g_time"][:, 1].masked_fill_(m, 160.)
        ws["g_steps"][:, 0].masked_fill_(m, 0)
        ws["g_steps"][:, 1].masked_fill_(m, self.replan_interval - 1)
        ws["g_hub"].masked_fill_(m[:, None], 1)
        for name in ("g_scores", "g_rcount", "g_rtime", "g_rlatch", "g_reward", "c_target",
                     "c_fuel_target", "c_fuel_delta", "c_command", "c_empty_ticks", "c_raster", "t_pos", "t_vel",
                     "t_conf", "t_quality", "t_mask", "t_spatial", "t_angular", "t_merged", "t_visible",
                     "o_pose", "o_vel", "o_size", "o_valid", "p_path", "p_profile", "p_len", "p_goal", "p_start", "p_progress", "p_trench"):
            t = ws[name]
            t.masked_fill_(m.reshape((-1,) + (1,) * (t.ndim - 1)), 0)
        ws["g_action"].masked_fill_(m[:, None], 7)
        ws["c_target_index"].masked_fill_(m[:, None], -1)
        ws["c_avoid"].masked_fill_(m[:, None], -1)
        ws["c_collect_heading"].copy_(torch.where(m[:, None], ws["r_pose"][..., 2], ws["c_collect_heading"]))
        ws["p_heading"].copy_(torch.where(m[:, None], ws["r_pose"][..., 2], ws["p_heading"]))
        ws["t_age"].masked_fill_(m[:, None, None], _INF)
        ws["o_age"].masked_fill_(m[:, None], _INF)
        self._episode += 1
        ws["e_episode"].copy_(torch.where(m, torch.full_like(ws["e_episode"], self._episode),
                                          ws["e_episode"]))

    def _perceive_and_observe(self, mask: torch.Tensor) -> None:
        ws = self.ws
        saved = ws["active"].clone()
        ws["active"].copy_(mask.to(torch.uint8))
        ws.sim.perceive()
        ws.sim.observe()
        ws["active"].copy_(saved)

    def reset(self, seed=None, *, defer_perception=False):
        if type(defer_perception) is not bool:
            raise ValueError("defer_perception must be boolean")
        if seed is not None:
            self.seed = int(seed)
            self.sim.generator.manual_seed(self.seed)
            p = self.ws.params
            s = self.seed & 0xFFFFFFFFFFFF
            self.ws.sim.set_seed(s & 0xFFFFFFFF, (s >> 32) & 0xFFFF | 0x5EED0000)
        self._graphs.clear()
        allm = torch.ones(self.n, dtype=torch.bool, device=self.device)
        self.ws["active"].fill_(1)
        self._reset_worlds(allm)
        if defer_perception:
            self._last_obs = None
            return None
        self._perceive_and_observe(allm)
        self._last_obs = self.ws["obs"]
        return self._last_obs, {"field_layout": self.field_layout_id, "robots": NUM_ROBOTS}

    def reset_done(self, mask):
        if self.device.type != "cpu" and (not isinstance(mask, torch.Tensor) or mask.device != self.device):
            raise ValueError("GPU reset mask must already reside on the environment device")
        m = torch.as_tensor(mask, device=self.device, dtype=torch.bool).reshape(self.n)
        self._reset_worlds(m)
        self._perceive_and_observe(m)
        self.ws["active"].fill_(1)
        return self.ws["obs"]

    # ----------------------------------------------------------------- steps
    def _set_actions(self, actions) -> None:
        if actions is None:
            return
        a = torch.as_tensor(actions, device=self.device).reshape(self.n, NUM_ROBOTS)
        self._actions_buf.copy_(a.to(torch.int32))

    def _launch_tick(self) -> None:
        sim = self.ws.sim
        sim.control(self._actions_buf)
        sim.plan(0)
        sim.tick(0, 1)

    def step(self, actions, active_mask=None, *, capture_observation=True, capture_info=True,
             _active_count=None, _return_info=None, **unsupported):
        if unsupported:
            raise ValueError(f"unsupported step options: {sorted(unsupported)}")
        if _return_info is not None:
            capture_info = bool(_return_info)
        full = active_mask is None
        if not full:
            if self.device.type != "cpu" and (not isinstance(active_mask, torch.Tensor)
                                              or active_mask.device != self.device):
                raise ValueError("GPU active mask must already reside on the environment device")
            act = torch.as_tensor(active_mask, device=self.device, dtype=torch.bool).reshape(self.n)
            self.ws["active"].copy_(act.to(torch.uint8))
        self._set_actions(actions)
        self._launch_tick()
        if capture_observation:
            self.ws.sim.observe()
        active = self.ws["active"].bool()
        rewards = self.ws["g_reward"] * active[:, None]
        truncated = active & (self.steps >= self.horizon)
        done = torch.zeros_like(active)
        info = {}
        if capture_info:
            info = {"fuel_acquired_event": self.fuel_acquired_event.clone(),
                    "fuel_scored_event": self.fuel_scored_event.clone(),
                    "fuel_passed_event": self.fuel_passed_event.clone(),
                    "fuel_denied_event": self.fuel_denied_event.clone(),
                    "team_score": self.fuel_score_count.clone(),
                    "match_elapsed": self.match_elapsed.clone()}
        if not full:
            self.ws["active"].fill_(1)
        self._last_obs = self.ws["obs"]
        return self._last_obs, rewards, done, truncated, info

    def step_held(self, actions, ticks: int, *, use_graph: bool = True, observe_every_tick: bool = False):
        """Advance every world `ticks` ticks under one held action and build
        the final observation; returns (obs, summed rewards, truncated).

        `observe_every_tick` builds the strategic observation after every
        tick instead of only after the last one (the intermediate ones are
        overwritten; this is the cost of a rollout that records observations
        at the physics rate).

        On CUDA the interval is captured once as a CUDA graph (control, plan
        and tick kernels per tick plus observe) and replayed afterwards.
        """
        self._set_actions(actions)
        ticks = int(ticks)
        observe_every_tick = bool(observe_every_tick)

        def interval(reward_buf):
            for k in range(ticks):
                self._launch_tick()
                reward_buf.add_(self.ws["g_reward"])
                if observe_every_tick and k < ticks - 1:
                    self.ws.sim.observe()
            self.ws.sim.observe()

        if self.device.type == "cuda" and use_graph:
            key = ("held", ticks, observe_every_tick)
            entry = self._graphs.get(key)
            if entry is None:
                reward_buf = torch.zeros((self.n, NUM_ROBOTS), device=self.device)
                stream = torch.cuda.Stream(device=self.device)
                stream.wait_stream(torch.cuda.current_stream(self.device))
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    reward_buf.zero_()
                    interval(reward_buf)
                entry = (graph, reward_buf)
                self._graphs[key] = entry
            graph, reward_buf = entry
            with trace.stage("sim_interval"):
                graph.replay()
            rewards = reward_buf
        else:
            rewards = torch.zeros((self.n, NUM_ROBOTS), device=self.device)
            interval(rewards)
        truncated = self.steps >= self.horizon
        self._last_obs = self.ws["obs"]
        return self._last_obs, rewards, truncated

    def observe(self, active_mask=None):
        if active_mask is None:
            self.ws.sim.observe()
        else:
            act = torch.as_tensor(active_mask, device=self.device, dtype=torch.bool).reshape(self.n)
            saved = self.ws["active"].clone()
            self.ws["active"].copy_(act.to(torch.uint8))
            self.ws.sim.observe()
            self.ws["active"].copy_(saved)
        return self.ws["obs"]

    def check_state(self, raise_error: bool = True) -> dict:
        """Status words of the per-tick state validation (constructor option
        `state_checks`, or AUTODRIVE_STATE_CHECKS=1): decoded, cleared, and
        raised as SimulationStateError when an environment reported one."""
        return check_state(self.ws, raise_error=raise_error)

    def action_mask(self) -> torch.Tensor:
        """Legal strategic actions per robot (last 8 observation features)."""
        return self.ws["obs"][..., -8:] > .5


class PlannerView:
    """Cached route state with the reference planner attribute names."""

    def __init__(self, ws: WorldState):
        self.ws = ws

    last_path = property(lambda self: self.ws["p_path"].reshape(-1, self.ws["p_path"].shape[2], 2))
    last_lengths = property(lambda self: self.ws["p_len"].reshape(-1).long())
    last_goal = property(lambda self: self.ws["p_goal"].reshape(-1, 2))
    last_start = property(lambda self: self.ws["p_start"].reshape(-1, 2))
    last_heading = property(lambda self: self.ws["p_heading"].reshape(-1))
    last_progress = property(lambda self: self.ws["p_progress"].reshape(-1))
    last_trench_alignment = property(lambda self: self.ws["p_trench"].reshape(-1).bool())
    # value-iteration sweeps of each row's last plan (negative: budget ran out first)
    last_sweeps = property(lambda self: self.ws["p_sweeps"].reshape(-1))
    last_speed_profile = property(lambda self: self.ws["p_profile"].reshape(-1, self.ws["p_profile"].shape[2]))
