"""Two-robot REBUILT environment (`TensorDefenseEnv`).

Slot 0 is the learner and slot 1 the scripted opponent
(frc_defense/tensor_sim.py:82-398). Tasks:

* ``counter_defense`` (default): the learner attacks (collects and scores
  FUEL) against a scripted defender; reward = own scores + 0.05 per
  acquisition - 0.001 per tick. Defenders (``opponent=``): ``guard`` (the
  default, alias ``adstar_defender``) runs ``defense_mode`` (``INTERCEPT``
  default, ``LANE_BLOCK``, ``FUEL_DENIAL``, ``SHADOW``, ``HUB_GUARD``), or
  one of those modes by name (``intercept``, ``lane_block``, ``fuel_denial``,
  ``shadow``, ``hub_guard``); ``cutoff`` / ``velocity_intercept`` alias
  ``intercept``, ``mirror`` / ``pursuit`` alias ``shadow``, and ``random``
  drives random velocity commands. A defender builds its waypoint from its
  own tracks of the attacker and reaches it through the route planner
  (frc_defense/tensor_defense_opponent.py:176-214).
* ``defense``: the learner defends against a scripted attacker; reward =
  -attacker scores - 0.02 per attacker acquisition - 0.001 per tick + a
  lane-position bonus.

Action modes:

* ``strategic`` (default, 8 categorical actions, 137 observations):
  collect x4 / shoot / defend / ferry / hold, executed by the native
  controller and route planner.
* ``direct`` (3 continuous actions in [-1, 1], 35 observations): normalised
  chassis velocity and yaw-rate command.
* ``tactical`` (2 continuous actions, 38 observations): a normalised field
  waypoint offset followed through the route planner.

Defense-task attackers (``opponent=``): ``offense`` (full scripted game
strategy with route planning; ``adstar``, ``guard`` and ``pursuit`` alias it),
``mirror``, ``cutoff``, ``velocity_intercept``, ``random``.
``static_opponent_fraction`` parks the opponent in a random share of worlds.
Control and observation latency rings (``max_control_latency_steps`` /
``max_observation_latency_steps``) delay the learner's actions and
observations by a per-episode number of ticks. With ``randomize``, the
first 18 observation features get Gaussian noise (``observation_noise``,
default 0.01) and then dropout (``observation_dropout``, default 0.02), as
in frc_defense/tensor_defense_observation.py:507-515. In the direct and
tactical modes an episode terminates when the attacker comes within
``goal_radius`` (0.5 m; randomised to 0.3-0.8 m per episode with
``randomize``) of its objective, with a 10-point penalty (defense) or bonus
(counter-defense). ``adstar_spawn_hint`` (default on) places the defender on
the attacker's line to its HUB at reset; off, both robots spawn uniformly.
"""
from __future__ import annotations

import json
import math
import os
from dataclasses import asdict
from pathlib import Path

import torch

from .. import field as fieldmod
from .env3v3 import FuelView, PlannerView, _INF
from .robots import RobotView
from .world import SwerveParameters, WorldState, build_params, check_state, fuel_config, state_checks_default

OPPONENT_KINDS = {"offense": 0, "adstar": 0, "guard": 0, "pursuit": 0, "mirror": 1, "cutoff": 2,
                  "velocity_intercept": 3, "random": 4}
DEFENSE_MODES = {"INTERCEPT": 5, "LANE_BLOCK": 6, "FUEL_DENIAL": 7, "SHADOW": 8, "HUB_GUARD": 9}
# counter-defense opponent names -> scripted defender (frc_defense/tensor_defense_step.py:110-119)
COUNTER_DEFENSE_ALIASES = {"cutoff": "intercept", "mirror": "shadow", "velocity_intercept": "intercept",
                           "pursuit": "shadow", "guard": "adstar_defender"}
COUNTER_DEFENSE_KINDS = ("adstar_defender", "intercept", "lane_block", "fuel_denial", "shadow", "hub_guard",
                         "random")
ACTION_MODES = {"direct": (3, 35), "tactical": (2, 38), "strategic": (8, 137)}


class TensorDefenseEnv:
    def __init__(self, num_envs=1, task="counter_defense", device="cuda", seed=0, opponent="guard", **kwargs):
        if task not in ("defense", "counter_defense"):
            raise ValueError("task must be counter_defense or defense")
        kind = opponent.get("value", opponent.get("mode", "guard")) if isinstance(opponent, dict) else opponent
        kind = str(kind or "guard").lower()
        if kind == "learned":
            raise ValueError("learned opponents are no longer supported; use a deterministic opponent")
        default_mode = (opponent.get("mode", "INTERCEPT") if isinstance(opponent, dict) else "INTERCEPT")
        selected = kwargs.pop("defense_mode", default_mode if task == "counter_defense" else None)
        self.defense_mode = None if selected is None else str(selected).upper()
        if self.defense_mode is not None and self.defense_mode not in DEFENSE_MODES:
            raise ValueError("defense_mode must be INTERCEPT, LANE_BLOCK, FUEL_DENIAL, SHADOW, or HUB_GUARD")
        if task == "counter_defense":
            kind = COUNTER_DEFENSE_ALIASES.get(kind, kind)
            if kind not in COUNTER_DEFENSE_KINDS:
                raise ValueError(f"opponent {kind!r} is not a scripted defender of the counter-defense task")
            if kind == "random":
                opponent_code = OPPONENT_KINDS["random"]
            else:
                opponent_code = DEFENSE_MODES[self.defense_mode if kind == "adstar_defender" else kind.upper()]
        else:
            if kind not in OPPONENT_KINDS:
                raise ValueError(f"unknown opponent {kind!r} for the defense task")
            opponent_code = OPPONENT_KINDS[kind]
        self.opponent_code = opponent_code
        config_path = os.environ.get("FRC_DRIVETRAIN_CONFIG")
        drivetrain = None
        if config_path:
            drivetrain = json.loads(Path(config_path).read_text())
            kwargs.setdefault("randomize", drivetrain.get("randomize", False))
            for name in ("robot_length", "robot_width", "mass", "max_speed", "max_acceleration",
                         "max_omega", "max_alpha", "field_friction", "lateral_friction"):
                if name in drivetrain:
                    kwargs.setdefault(name, drivetrain[name])
            kwargs.setdefault("swerve", SwerveParameters(**drivetrain.get("swerve", {})))
            if "gamepieces" in drivetrain:
                kwargs.setdefault("gamepiece_config", drivetrain["gamepieces"])
        self.n, self.device, self.task = int(num_envs), torch.device(device), task
        self.opponent = kind
        self.action_mode = str(kwargs.pop("action_mode", "strategic")).lower()
        if self.action_mode not in ACTION_MODES:
            raise ValueError("action_mode must be direct, tactical, or strategic")
        self.action_dim, self.obs_dim = ACTION_MODES[self.action_mode]
        self.action_kind = "categorical" if self.action_mode == "strategic" else "continuous"
        gp = kwargs.pop("gamepiece_config", {}) or {}
        fuel_physics = kwargs.pop("fuel_physics", gp.get("physics", True))
        self.fuel_capacity = max(1, int(kwargs.pop("max_fuel_capacity", gp.get("max_capacity", 8))))
        self.intake_interval = float(kwargs.pop("intake_interval", gp.get("intake_interval_s", .20)))
        self.score_interval = float(kwargs.pop("score_interval", gp.get("score_interval_s", .10)))
        self.fuel_count = int(kwargs.pop("fuel_count", 504))
        preload = kwargs.pop("preloaded_per_robot", None)
        self.preloaded_per_robot = int(preload or 0)
        # "staged": depot arrays + neutral-zone array (the match layout);
        # "uniform": every piece at a uniformly random floor position each reset
        self.fuel_layout = str(kwargs.pop("fuel_layout", "staged"))
        if self.fuel_layout not in ("staged", "uniform"):
            raise ValueError("fuel_layout must be 'staged' or 'uniform'")
        if self.fuel_layout == "uniform":
            if not 1 <= self.fuel_count <= 600:
                raise ValueError("fuel_count must be 1 through 600")
        elif not 96 + 6 * self.preloaded_per_robot <= self.fuel_count <= 600:
            raise ValueError("fuel_count must be 96 + 6*preloaded_per_robot through 600")
        self.dt = float(kwargs.pop("dt", .02))
        self.horizon = int(kwargs.pop("horizon", 8000))
        # The horizon is honoured as given (the reference raises strategic
        # horizons to a full 160 s match; pass horizon=8000 for that).
        self.randomize = bool(kwargs.pop("randomize", True))
        self.static_opponent_fraction = float(kwargs.pop("static_opponent_fraction", 0.))
        if not 0. <= self.static_opponent_fraction <= 1.:
            raise ValueError("static_opponent_fraction must be between 0 and 1")
        self.normalize_observations = bool(kwargs.pop("normalize_observations", True))
        self.max_control_latency_steps = max(0, int(kwargs.pop("max_control_latency_steps", 6)))
        self.max_observation_latency_steps = max(0, int(kwargs.pop("max_observation_latency_steps", 8)))
        perception = kwargs.pop("perception_config", {}) or {}
        field_length = float(kwargs.pop("field_length", 16.54))
        field_width = float(kwargs.pop("field_width", 8.07))
        self.perception_range = float(perception.get("range_m", math.hypot(field_length, field_width)))
        fov = float(perception.get("fov_degrees", 360.))
        self.perception_track_timeout = float(perception.get("track_timeout_s", 1.0))
        replan = max(1, int(kwargs.pop("adstar_replan_interval", 20)))
        swerve = kwargs.pop("swerve", None) or SwerveParameters()
        base = dict(length=float(kwargs.pop("robot_length", .9)), width=float(kwargs.pop("robot_width", .9)),
                    mass=float(kwargs.pop("mass", 55.)), speed=float(kwargs.pop("max_speed", 4.8)),
                    accel=float(kwargs.pop("max_acceleration", 8.)), omega=float(kwargs.pop("max_omega", 8.)),
                    alpha=float(kwargs.pop("max_alpha", 18.)),
                    bumper_friction=float(kwargs.pop("bumper_friction", .65)),
                    field_friction=float(kwargs.pop("field_friction", .7)),
                    lateral_friction=float(kwargs.pop("lateral_friction", 1.2)),
                    yaw_inertia_multiplier=float(kwargs.pop("yaw_inertia_multiplier", 1.5)))
        layout = kwargs.pop("field_layout", "2026_rebuilt")
        self.observation_noise = float(kwargs.pop("observation_noise", .01))
        self.observation_dropout = float(kwargs.pop("observation_dropout", .02))
        if not (self.observation_noise >= 0 and 0 <= self.observation_dropout < 1):
            raise ValueError("observation_noise must be >= 0 and observation_dropout in [0, 1)")
        self.adstar_spawn_hint = bool(kwargs.pop("adstar_spawn_hint", True))
        self.base_goal_radius = float(kwargs.pop("goal_radius", .5))
        state_checks = kwargs.pop("state_checks", None)
        # reference options that only select among equivalent implementations
        # of the same computation (candidate reuse, squared distances, skipping
        # a metric-only objective) change nothing here
        for equivalent in ("reuse_strategic_own_candidates", "squared_fuel_candidate_distance",
                           "skip_strategic_offense_metric_objective"):
            kwargs.pop(equivalent, None)
        if kwargs:
            raise TypeError(f"unexpected TensorDefenseEnv options: {sorted(kwargs)}")
        self.field_boxes = fieldmod.qualification_field(layout, field_length, field_width)
        solids = fieldmod.static_collision_boxes(self.field_boxes)
        bumps = fieldmod.bump_boxes(self.field_boxes)
        self.field_feature_boxes = solids + bumps
        by_name = {b.name: b for b in self.field_boxes}
        hubs = [(by_name["red_hub"].x, by_name["red_hub"].y), (by_name["blue_hub"].x, by_name["blue_hub"].y)]
        self.fuel_config = fuel_config(fuel_physics)
        self.swerve = swerve
        learner_mode = 1 if self.action_mode == "strategic" else 3
        params = build_params(
            n=self.n, robots=2, pieces=self.fuel_count, dt=self.dt, field_length=field_length,
            field_width=field_width, boxes=[b.as_tensor() for b in solids],
            bumps=[b.as_tensor() for b in bumps], hubs=hubs, team=(0, 1), mode=(learner_mode, 2),
            role=(0, 1) if task == "counter_defense" else (1, 0), kind=(0, 0),
            counter_defense=1 if task == "counter_defense" else 0,
            checks=int(state_checks_default() if state_checks is None else bool(state_checks)), capacity=(self.fuel_capacity, self.fuel_capacity),
            score_interval=(self.score_interval, self.score_interval), fuel=self.fuel_config,
            swerve=swerve, base_speed=base["speed"], base_omega=base["omega"], seed=int(seed or 0),
            two_robot_schedule=1, opponent_kind=opponent_code, perception_range=self.perception_range,
            perception_fov=math.radians(fov) * .5, track_timeout=self.perception_track_timeout,
            replan_interval=replan, normalize_obs=int(self.normalize_observations), horizon=self.horizon,
            plan_res=.3, plan_nx=math.ceil(field_length / .3), plan_ny=math.ceil(field_width / .3),
            plan_sweeps=4 * (math.ceil(field_length / .3) + math.ceil(field_width / .3)), fuel_radius_rules=.0825,
            perception_interval=1)
        self.ws = WorldState(params, self.device)
        self.sim = RobotView(self.ws, dt=self.dt, field_length=field_length, field_width=field_width,
                             team_ids=(0, 1), boxes=[b.as_tensor() for b in solids],
                             bumps=[b.as_tensor() for b in bumps], swerve=swerve, base=base,
                             seed=int(seed or 0), randomize=self.randomize)
        self.fuel_physics = FuelView(self.ws, self.fuel_config) if self.fuel_config else None
        self.team_ids = self.sim.team_ids
        self.hub_centers = torch.tensor(hubs, device=self.device, dtype=torch.float32)
        self.alliance_zone_depth = fieldmod.ALLIANCE_ZONE_DEPTH
        self.field_length = field_length
        self.replan_interval = replan
        self.drivetrain_config = drivetrain or {
            "name": "built-in illustrative defaults", "randomize": self.randomize, "mass": base["mass"],
            "robot_length": base["length"], "robot_width": base["width"], "max_speed": base["speed"],
            "max_acceleration": base["accel"], "max_omega": base["omega"], "max_alpha": base["alpha"],
            "swerve": asdict(swerve)}
        self.generator = torch.Generator(device="cpu").manual_seed(int(seed or 0))
        self.obs_generator = torch.Generator(device=self.device).manual_seed(int(seed or 0) + 0x0B5)
        self.attacker = 0 if task == "counter_defense" else 1
        self.goal_radius = torch.full((self.n,), self.base_goal_radius, device=self.device)
        self._episode = 0
        L = self.max_control_latency_steps + 1
        self.action_history = torch.zeros((self.n, L, 3), device=self.device)
        self.control_delay = torch.zeros(self.n, dtype=torch.long, device=self.device)
        self.observation_delay = torch.zeros(self.n, dtype=torch.long, device=self.device)
        self.observation_history = torch.zeros((self.n, self.max_observation_latency_steps + 1, self.obs_dim),
                                               device=self.device)
        self._actions = torch.full((self.n, 2), 7, dtype=torch.int32, device=self.device)
        self._graphs: dict = {}
        self.reset(seed=seed)

    # ------------------------------------------------------------------ views
    piece_pos = property(lambda self: self.ws["f_pos"][:, :2].transpose(1, 2))
    piece_vel = property(lambda self: self.ws["f_vel"][:, :2].transpose(1, 2))
    piece_active = property(lambda self: self.ws["f_active"].bool())
    piece_owner = property(lambda self: self.ws["f_owner"].long())
    match_elapsed = property(lambda self: self.ws["g_time"][:, 0])
    match_remaining = property(lambda self: self.ws["g_time"][:, 1])
    steps = property(lambda self: self.ws["g_steps"][:, 0].long())
    hub_active = property(lambda self: self.ws["g_hub"].bool())
    fuel_score_count = property(lambda self: self.ws["g_scores"][:, 2:4].long())
    fuel_acquisition_count = property(lambda self: self.ws["g_rcount"][:, :, 0].long())
    fuel_denied_count = property(lambda self: self.ws["g_rcount"][:, :, 1].long())
    fuel_acquired_event = property(lambda self: self.ws["g_rcount"][:, :, 2].long())
    fuel_scored_event = property(lambda self: self.ws["g_rcount"][:, :, 3].long())
    track_pos = property(lambda self: self.ws["t_pos"].transpose(2, 3))
    track_mask = property(lambda self: self.ws["t_mask"].bool())
    planner = property(lambda self: PlannerView(self.ws))
    static_opponent_mask = property(lambda self: self.ws["g_rlatch"][:, 1, 7].bool())

    # ----------------------------------------------------------------- resets
    def _rand(self, shape):
        return torch.rand(shape, generator=self.generator).to(self.device)

    def _reset_worlds(self, m: torch.Tensor) -> None:
        ws = self.ws
        self.sim.randomize_parameters(m)
        self.sim.clear_dynamics(m)
        margin = .9
        L, W = self.sim.field_length, self.sim.field_width
        pose = torch.zeros((self.n, 2, 3), device=self.device)
        pose[..., 0] = margin + self._rand((self.n, 2)) * (L - 2 * margin)
        pose[..., 1] = margin + self._rand((self.n, 2)) * (W - 2 * margin)
        pose[..., 2] = (2 * self._rand((self.n, 2)) - 1) * math.pi
        atk, dfd = self.attacker, 1 - self.attacker
        if self.adstar_spawn_hint:
            # place the defender on the attacker's line to its HUB, 1.25-2.75 m ahead
            hub = self.hub_centers[atk]
            d = hub[None] - pose[:, atk, :2]
            dn = d.norm(dim=-1, keepdim=True).clamp_min(1e-6)
            along = 1.25 + 1.5 * self._rand((self.n, 1))
            place = pose[:, atk, :2] + d / dn * along.minimum(dn * .8) + (self._rand((self.n, 2)) - .5) * .18
            pose[:, dfd, 0] = place[:, 0].clamp(margin, L - margin)
            pose[:, dfd, 1] = place[:, 1].clamp(margin, W - margin)
        radius = (.3 + self._rand(self.n) * .5) if self.randomize else torch.full(
            (self.n,), self.base_goal_radius, device=self.device)
        self.goal_radius = torch.where(m, radius, self.goal_radius)
        ws["r_pose"].copy_(torch.where(m[:, None, None], pose, ws["r_pose"]))
        if self.randomize:
            vel = torch.zeros((self.n, 2, 3), device=self.device)
            vel[..., :2] = (self._rand((self.n, 2, 2)) * 2 - 1) * .25 * self.sim.speed[..., None]
            vel[..., 2] = (self._rand((self.n, 2)) * 2 - 1) * .2 * self.sim.omega_limit
            ws["r_vel"].copy_(torch.where(m[:, None, None], vel, ws["r_vel"]))
        ws["est_pose"].copy_(torch.where(m[:, None, None], ws["r_pose"], ws["est_pose"]))
        ws["policy_pose"].copy_(torch.where(m[:, None, None], ws["r_pose"], ws["policy_pose"]))
        # FUEL: depots + neutral array, or a uniform scatter over the floor
        P = self.fuel_count
        r = self.fuel_config.radius if self.fuel_config else .075
        if self.fuel_layout == "uniform":
            active = torch.ones(P, dtype=torch.uint8)
            u = self._rand((self.n, P, 2))
            xyd = torch.stack((r + u[..., 0] * (L - 2 * r), r + u[..., 1] * (W - 2 * r)), -1)
        else:
            xy = torch.zeros((P, 2))
            active = torch.zeros(P, dtype=torch.uint8)
            depots = {b.name: b for b in self.field_boxes if b.kind == "depot"}
            for begin, name in ((0, "red_depot"), (24, "blue_depot")):
                dd = depots[name]
                pts = fieldmod.grid_array_points(24, dd.x - dd.length / 2, dd.x + dd.length / 2,
                                                 dd.y - dd.width / 2, dd.y + dd.width / 2)
                xy[begin:begin + 24] = torch.tensor(pts)
            active[:48] = 1
            neutral = P - 96
            pts = fieldmod.grid_array_points(neutral, 8.27 - .915, 8.27 + .915, 4.035 - 2.615, 4.035 + 2.615)
            xy[96:] = torch.tensor(pts)
            active[96:] = 1
            xyd = xy.to(self.device)[None].expand(self.n, -1, -1)
        fpos = torch.zeros((self.n, 3, P), device=self.device)
        fpos[:, 0], fpos[:, 1] = xyd[..., 0], xyd[..., 1]
        fpos[:, 2] = r
        ws["f_pos"].copy_(torch.where(m[:, None, None], fpos, ws["f_pos"]))
        for name in ("f_vel", "f_ang"):
            ws[name].masked_fill_(m[:, None, None], 0.)
        ws["f_clock"].masked_fill_(m[:, None], 0.)
        ws["f_sleep"].masked_fill_(m[:, None], 0)
        ws["f_active"].copy_(torch.where(m[:, None], active.to(self.device)[None], ws["f_active"]))
        ws["f_owner"].masked_fill_(m[:, None], -1)
        ws["f_zone"].masked_fill_(m[:, None], 0)
        ws["g_time"][:, 0].masked_fill_(m, 0.)
        ws["g_time"][:, 1].masked_fill_(m, 160.)
        ws["g_steps"][:, 0].masked_fill_(m, 0)
        ws["g_steps"][:, 1].masked_fill_(m, self.replan_interval - 1)
        ws["g_hub"].masked_fill_(m[:, None], 1)
        first = (self._rand(self.n) < .5).to(torch.int32)
        ws["g_first_inactive"].copy_(torch.where(m, first, ws["g_first_inactive"]))
        for name in ("g_scores", "g_rcount", "g_rtime", "g_rlatch", "g_reward", "c_target", "c_fuel_target",
                     "c_fuel_delta", "c_command", "c_empty_ticks", "t_pos", "t_vel", "t_conf", "t_quality",
                     "t_mask", "o_pose", "o_vel", "o_size", "o_valid", "p_path", "p_profile", "p_len",
                     "p_goal", "p_start", "p_progress", "p_trench"):
            t = ws[name]
            t.masked_fill_(m.reshape((-1,) + (1,) * (t.ndim - 1)), 0)
        static = self._rand(self.n) < self.static_opponent_fraction
        ws["g_rlatch"][:, 1, 7] = torch.where(m, static.to(torch.uint8), ws["g_rlatch"][:, 1, 7])
        ws["g_action"].masked_fill_(m[:, None], 7)
        ws["c_target_index"].masked_fill_(m[:, None], -1)
        ws["c_avoid"].masked_fill_(m[:, None], -1)
        ws["t_age"].masked_fill_(m[:, None, None], _INF)
        ws["o_age"].masked_fill_(m[:, None], _INF)
        ws["p_heading"].copy_(torch.where(m[:, None], ws["r_pose"][..., 2], ws["p_heading"]))
        self._episode += 1
        ws["e_episode"].copy_(torch.where(m, torch.full_like(ws["e_episode"], self._episode), ws["e_episode"]))
        self.action_history.masked_fill_(m[:, None, None], 0.)
        self.observation_history.masked_fill_(m[:, None, None], 0.)
        if self.randomize and self.max_control_latency_steps:
            delay = torch.randint(self.max_control_latency_steps + 1, (self.n,), generator=self.generator)
            self.control_delay.copy_(torch.where(m, delay.to(self.device), self.control_delay))
        if self.randomize and self.max_observation_latency_steps:
            delay = torch.randint(self.max_observation_latency_steps + 1, (self.n,), generator=self.generator)
            self.observation_delay.copy_(torch.where(m, delay.to(self.device), self.observation_delay))

    def _observe_learner(self) -> torch.Tensor:
        self.ws.sim.observe()
        raw = self.ws["obs"][:, 0, :self.obs_dim]
        shifted = torch.cat((raw[:, None], self.observation_history[:, :-1]), 1)
        active = self.ws["active"].bool()
        self.observation_history.copy_(torch.where(active[:, None, None], shifted, self.observation_history))
        obs = self.observation_history.gather(
            1, self.observation_delay[:, None, None].expand(-1, 1, self.obs_dim)).squeeze(1)
        if self.randomize and self.observation_noise > 0:
            obs[:, :18].add_(torch.randn((self.n, 18), device=self.device, generator=self.obs_generator)
                             * self.observation_noise)
        if self.randomize and self.observation_dropout > 0:
            keep = torch.rand((self.n, 18), device=self.device, generator=self.obs_generator) >= self.observation_dropout
            obs[:, :18].mul_(keep)
        return obs

    def _attacker_goal(self) -> torch.Tensor:
        """The attacker's objective (frc_defense/tensor_sim.py:354-370): its HUB
        approach ring when carrying FUEL to an active HUB, else its nearest
        perceived FUEL track, else the approach ring."""
        ws, a = self.ws, self.attacker
        pos = ws["r_pose"][:, a, :2]
        hub = self.hub_centers[a][None]
        d = pos - hub
        d = d / d.norm(dim=-1, keepdim=True).clamp_min(1e-6)
        size = ws["r_param"][:, a, :2]
        approach = hub + d * (.595 + .5 * size.square().sum(-1).sqrt() + .02)[:, None]
        tracks = ws["t_pos"][:, a].transpose(1, 2)
        dist = (tracks - pos[:, None]).norm(dim=-1).masked_fill(~ws["t_mask"][:, a].bool(), float("inf"))
        nearest, idx = dist.min(-1)
        piece = tracks[torch.arange(self.n, device=self.device), idx]
        carrying = ((ws["f_owner"] == a) & ws["f_active"].bool()).any(-1)
        score = carrying & ws["g_hub"][:, a].bool()
        return torch.where(score[:, None], approach, torch.where(torch.isfinite(nearest)[:, None], piece, approach))

    def reset(self, seed=None, options=None):
        if seed is not None:
            self.generator.manual_seed(int(seed))
            self.sim.generator.manual_seed(int(seed))
            self.obs_generator.manual_seed(int(seed) + 0x0B5)
        self._graphs.clear()
        allm = torch.ones(self.n, dtype=torch.bool, device=self.device)
        self.ws["active"].fill_(1)
        self._reset_worlds(allm)
        self.ws.sim.perceive()
        obs = self._observe_learner()
        self.observation_history.copy_(obs[:, None].expand_as(self.observation_history))
        self._last_observation = obs
        radius = torch.full((self.n,), .595, device=self.device) if self.action_mode == "strategic" else self.goal_radius
        return obs, {"field_layout": "2026_rebuilt", "goal_radius": radius}

    def reset_done(self, mask):
        if self.device.type != "cpu" and (not isinstance(mask, torch.Tensor) or mask.device != self.device):
            raise ValueError("GPU reset mask must already reside on the environment device")
        m = torch.as_tensor(mask, device=self.device, dtype=torch.bool).reshape(self.n)
        self._reset_worlds(m)
        saved = self.ws["active"].clone()
        self.ws["active"].copy_(m.to(torch.uint8))
        self.ws.sim.perceive()
        fresh = self._observe_learner()
        self.observation_history.copy_(torch.where(m[:, None, None], fresh[:, None].expand_as(
            self.observation_history), self.observation_history))
        self.ws["active"].copy_(saved)
        self._last_observation = torch.where(m[:, None], fresh, self._last_observation)
        return self._last_observation

    # ------------------------------------------------------------------ steps
    def _apply_action(self, action, active: torch.Tensor) -> None:
        a = torch.as_tensor(action, device=self.device)
        stored = torch.zeros((self.n, 3), device=self.device)
        if self.action_mode == "strategic":
            stored[:, 0] = a.reshape(self.n).clamp(0, 7).to(torch.float32)
        else:
            a = torch.nan_to_num(a.to(torch.float32)).clamp(-1, 1).reshape(self.n, self.action_dim)
            stored[:, :self.action_dim] = a
        shifted = torch.cat((stored[:, None], self.action_history[:, :-1]), 1)
        self.action_history.copy_(torch.where(active[:, None, None], shifted, self.action_history))
        applied = self.action_history.gather(1, self.control_delay[:, None, None].expand(-1, 1, 3)).squeeze(1)
        if self.action_mode == "strategic":
            self._actions[:, 0] = applied[:, 0].to(torch.int32)
        elif self.action_mode == "direct":
            cmd = self.ws["c_command"]
            cmd[:, 0, 0] = applied[:, 0] * self.sim.speed[:, 0]
            cmd[:, 0, 1] = applied[:, 1] * self.sim.speed[:, 0]
            cmd[:, 0, 2] = applied[:, 2] * self.sim.omega_limit[:, 0]
        else:  # tactical: waypoint offset, straight-line tracking
            p = self.ws["policy_pose"][:, 0]
            target = p[:, :2] + applied[:, :2] * 2.
            d = target - p[:, :2]
            v = d / d.norm(dim=-1, keepdim=True).clamp_min(1e-6) * self.sim.speed[:, 0, None] * (
                d.norm(dim=-1, keepdim=True) / .5).clamp(max=1.)
            cmd = self.ws["c_command"]
            cmd[:, 0, 0], cmd[:, 0, 1], cmd[:, 0, 2] = v[:, 0], v[:, 1], 0.

    def step(self, action, active_mask=None, *, _active_count=None, _return_info=True,
             _capture_observation=True):
        full = active_mask is None
        if not full:
            if self.device.type != "cpu" and (not isinstance(active_mask, torch.Tensor)
                                              or active_mask.device != self.device):
                raise ValueError("GPU active mask must already reside on the environment device")
            active = torch.as_tensor(active_mask, device=self.device, dtype=torch.bool).reshape(self.n)
            self.ws["active"].copy_(active.to(torch.uint8))
        else:
            active = torch.ones(self.n, dtype=torch.bool, device=self.device)
        self._apply_action(action, active)
        sim = self.ws.sim
        sim.control(self._actions)
        sim.plan(0)
        sim.tick(0, 1)
        reward = self.ws["g_reward"][:, 0] * active
        truncated = active & (self.steps >= self.horizon)
        terminated = torch.zeros_like(active)
        if self.action_mode != "strategic":
            # direct / tactical episodes end when the attacker reaches its objective
            goal = self._attacker_goal()
            reached = (goal - self.ws["r_pose"][:, self.attacker, :2]).norm(dim=-1) < self.goal_radius
            terminated = active & reached
            reward = reward + terminated * (10. if self.task == "counter_defense" else -10.)
        if _capture_observation:
            obs = self._observe_learner()
            self._last_observation = torch.where(active[:, None], obs, self._last_observation)
        info = {}
        if _return_info:
            info = {"fuel_acquired_event": self.fuel_acquired_event.clone(),
                    "fuel_scored_event": self.fuel_scored_event.clone(),
                    "team_score": self.fuel_score_count.clone(),
                    "match_elapsed": self.match_elapsed.clone(),
                    "robot_contact": self.sim.robot_contact.clone()}
        if not full:
            self.ws["active"].fill_(1)
        return self._last_observation, reward, terminated, truncated, info

    def check_state(self, raise_error: bool = True) -> dict:
        """Decoded status words of the per-tick state validation (option `state_checks`)."""
        return check_state(self.ws, raise_error=raise_error)

    def strategic_action_mask(self) -> torch.Tensor:
        return self._last_observation[:, -8:] > .5 if self.action_mode == "strategic" else None
