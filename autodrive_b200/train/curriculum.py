"""Outcome-gated offense curriculum on the 3v3 simulator.

Parity with frc_defense/training_curriculum.py (scenario table, gates,
seed partitions, promotion and task mixture), frc_defense/curriculum_scenarios.py
(CurriculumEnv: staged scenario resets), frc_defense/curriculum_metrics.py
(physical outcome counters) and frc_defense/curriculum_training.py (scripted
teachers, PPO / SAC training with periodic validation, strict resume):

* ``SCENARIOS``            12 staged scenarios with prerequisites, category
                           lists, time budgets and promotion gates;
* ``seed_partition``       stable 63-bit seeds, disjoint across the
                           train / validation / test / calibration pools;
* ``evaluate_promotion``   consumes one validation round: gate checks
                           (episodes, success rate, throughput vs the scripted
                           reference, retention of every prerequisite at >= 90 %
                           of its qualified throughput), consecutive-pass streaks,
                           duplicate-round rejection;
* ``task_mixture``         70 % current, 20 % earlier-qualified, 10 % next;
* ``CurriculumEnv``        one neural offense robot (slot 0) on the batched 3v3
                           simulator, scenario placements written straight into
                           the device state tensors;
* ``D1HandWeightedPolicy`` / ``D2PredictivePolicy``  scripted teachers;
* ``train_curriculum`` / ``evaluate_curriculum`` / ``main``.

Success is judged only from physical outcomes (acquired, scored, staged
FUEL within the time budget), never from reward.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path

import torch

CURRICULUM_VERSION = "2"
SPLITS = {"train": 0, "validation": 1, "test": 2, "calibration": 3}


@dataclass(frozen=True)
class GateDefinition:
    min_episodes: int = 100
    consecutive_evaluations: int = 3
    success_rate: float = .9
    throughput_ratio: float = 0.
    min_useful_throughput: float = 0.


@dataclass(frozen=True)
class ScenarioDefinition:
    scenario_id: str
    stage: str
    prerequisites: tuple[str, ...]
    required_categories: tuple[str, ...]
    time_budget_s: float
    gate: GateDefinition
    success_criterion: str
    version: str = "1"


_PRIM = GateDefinition()
_CYCLE = GateDefinition(throughput_ratio=.8)
_PRESS = GateDefinition(throughput_ratio=.8, min_useful_throughput=.01)
_ROUTES = ("open", "trench", "bump")
_BOTH_ROUTES = tuple(f"{phase}/{route}" for phase in ("active", "inactive") for route in _ROUTES)
# HUB-switch categories: direction / load / time left before the switch / situation
_TRANSITIONS = tuple(
    f"{direction}/{load}/{timing}/{situation}"
    for direction, situations in (("active_to_inactive", ("collecting", "carrying_home", "approaching_shot")),
                                  ("inactive_to_active", ("before_release", "after_release", "staged_at_home")))
    for load in ("empty", "partial", "full")
    for timing in ("enough_time", "too_little_time")
    for situation in situations) + ("empty_collection", "hold_useful_load")
# blocker levels: none, a parked robot on the route, a patrolling defender, a
# blocker in the trench / on the bump / at a seeded choice of route, two
# reactive defenders, and a per-world mixture
_BLOCKERS = ("level_0", "level_1_stationary", "level_2_patrol", "level_3_trench", "level_3_bump",
             "level_3_seeded_choice", "level_4_reactive", "level_5_mixed")
_PRESSURE = tuple(f"{ph}/{route}/{lvl}" for ph in ("active", "inactive") for route in _ROUTES
                  for lvl in _BLOCKERS
                  if (lvl != "level_3_trench" or route == "trench") and (lvl != "level_3_bump" or route == "bump")
                  and (lvl != "level_3_seeded_choice" or route != "open"))


def _sc(name, stage, prereq, cats, budget, gate, success):
    return ScenarioDefinition(name, stage, tuple(prereq), tuple(cats), float(budget), gate, success)


SCENARIOS = {s.scenario_id: s for s in (
    _sc("pickup_simple", "1", (), ("single", "cluster"), 20., _PRIM, "acquire and retain the required distinct FUEL"),
    _sc("pickup_scattered", "2", ("pickup_simple",), ("sparse", "dense", "initially_hidden"), 40., _PRIM,
        "retain the required fraction of the available FUEL"),
    _sc("pickup_multi_zone", "3", ("pickup_scattered",), ("productive", "empty", "depleted"), 60., _PRIM,
        "leave empty or depleted zones and collect from productive ones"),
    _sc("active_carry_to_zone", "4A", ("pickup_multi_zone",), ("active/trench", "active/bump"), 35., _PRIM,
        "reach the scoring area with the load while the HUB is active"),
    _sc("active_shoot_preloaded", "4B", ("pickup_simple",),
        ("active/preloaded", "active/approach", "active/heading_error"), 25., _PRIM,
        "score the preloaded FUEL while the friendly HUB is active"),
    _sc("inactive_ferry_preloaded", "4C", ("pickup_simple",),
        ("inactive/preloaded", "inactive/approach", "inactive/alignment", "inactive/partial_load",
         "inactive/full_load", "inactive/landing"), 30.,
        _PRIM, "deliver preloaded FUEL into the friendly staging zone"),
    _sc("active_collect_carry_score", "5A", ("pickup_multi_zone", "active_carry_to_zone", "active_shoot_preloaded"),
        tuple(f"active/{r}" for r in _ROUTES), 90., _CYCLE, "repeat collect-and-score cycles"),
    _sc("inactive_collect_ferry", "5B", ("pickup_multi_zone", "inactive_ferry_preloaded"),
        tuple(f"inactive/{r}" for r in _ROUTES), 90., _CYCLE, "repeat collect-and-ferry deliveries"),
    _sc("hub_transition_cycles", "6", ("active_collect_carry_score", "inactive_collect_ferry"),
        _TRANSITIONS, 120., _CYCLE, "keep useful objectives across HUB switches"),
    _sc("offense_vs_scripted_pressure", "7", ("hub_transition_cycles",), _PRESSURE, 120., _PRESS,
        "deliver useful FUEL under scripted defensive pressure"),
    _sc("team_delivery_cycles", "8", ("offense_vs_scripted_pressure",),
        tuple(f"{c}/{t}" for c in _BOTH_ROUTES for t in ("receiver", "multiple_teammates", "opponents")), 150.,
        _CYCLE, "convert deliveries into team scoring"),
    _sc("full_match_offense", "9", ("team_delivery_cycles", "offense_vs_scripted_pressure", "hub_transition_cycles"),
        _PRESSURE, 160., _PRESS, "contribute across the full match schedule"),
)}


def get_scenario(scenario_id: str) -> ScenarioDefinition:
    if scenario_id not in SCENARIOS:
        raise ValueError(f"unknown scenario {scenario_id!r}")
    return SCENARIOS[scenario_id]


def ancestors(scenario_id: str) -> set[str]:
    out: set[str] = set()
    for p in get_scenario(scenario_id).prerequisites:
        out |= {p} | ancestors(p)
    return out


def seed_partition(scenario_id: str, split: str, count: int, *, master_seed: int = 0) -> tuple[int, ...]:
    """63-bit seeds: a 40-bit scenario/master-seed namespace, a 21-bit counter and
    the 2-bit split id in the low bits, so pools never overlap."""
    get_scenario(scenario_id)
    if split not in SPLITS:
        raise ValueError("split must be train, validation, test or calibration")
    if type(count) is not int or not 0 <= count < 2 ** 21:
        raise ValueError("count must be an integer in [0, 2**21)")
    if type(master_seed) is not int or master_seed < 0:
        raise ValueError("master_seed must be a nonnegative integer")
    ns = int.from_bytes(hashlib.sha256(f"{CURRICULUM_VERSION}/{scenario_id}/{master_seed}".encode()).digest()[:5], "big")
    return tuple((ns << 23) | (i << 2) | SPLITS[split] for i in range(count))


def wilson_interval(successes: int, n: int, z: float = 1.959963984540054) -> tuple[float, float]:
    if n <= 0:
        return 0., 1.
    p = successes / n
    den = 1 + z * z / n
    mid = (p + z * z / (2 * n)) / den
    half = z * math.sqrt(p * (1 - p) / n + z * z / (4 * n * n)) / den
    return max(0., mid - half), min(1., mid + half)


@dataclass(frozen=True)
class CategoryResult:
    category: str
    episodes: int
    successes: int
    useful_throughput: float = 0.
    reference_throughput: float = 0.


@dataclass(frozen=True)
class EvaluationResult:
    evaluation_id: str
    scenario_id: str
    split: str
    categories: tuple[CategoryResult, ...]
    checkpoint_id: str = ""
    protocol_id: str = ""

    @property
    def episodes(self) -> int:
        return sum(c.episodes for c in self.categories)

    @property
    def successes(self) -> int:
        return sum(c.successes for c in self.categories)


@dataclass
class CurriculumState:
    qualified: set = field(default_factory=set)
    consecutive_passes: dict = field(default_factory=dict)
    qualified_throughput: dict = field(default_factory=dict)
    qualified_checkpoint: dict = field(default_factory=dict)
    seen_evaluation_ids: set = field(default_factory=set)

    def to_dict(self) -> dict:
        return {"curriculum_version": CURRICULUM_VERSION, "qualified": sorted(self.qualified),
                "consecutive_passes": dict(self.consecutive_passes),
                "qualified_throughput": {k: dict(v) for k, v in self.qualified_throughput.items()},
                "qualified_checkpoint": dict(self.qualified_checkpoint),
                "seen_evaluation_ids": sorted(self.seen_evaluation_ids)}

    @classmethod
    def from_dict(cls, data: dict) -> "CurriculumState":
        if not isinstance(data, dict) or data.get("curriculum_version") != CURRICULUM_VERSION:
            raise ValueError("invalid curriculum state or version")
        q = set(data["qualified"])
        if not q <= SCENARIOS.keys() or any(not ancestors(s) <= q for s in q):
            raise ValueError("qualified scenarios must be known and have qualified prerequisites")
        if set(data["qualified_throughput"]) != q or set(data["qualified_checkpoint"]) != q:
            raise ValueError("qualified scenarios need throughput baselines and checkpoints")
        passes = data["consecutive_passes"]
        if any(s not in SCENARIOS or type(n) is not int or n < 0 for s, n in passes.items()):
            raise ValueError("invalid pass counts")
        return cls(q, dict(passes), {k: dict(v) for k, v in data["qualified_throughput"].items()},
                   dict(data["qualified_checkpoint"]), set(data["seen_evaluation_ids"]))


@dataclass(frozen=True)
class PromotionDecision:
    promoted: bool
    passed: bool
    failures: tuple[str, ...]


def gate_failures(result: EvaluationResult) -> list[str]:
    sc = get_scenario(result.scenario_id)
    g = sc.gate
    out = []
    cats = {c.category for c in result.categories}
    if cats != set(sc.required_categories):
        out.append("evaluation must cover exactly the scenario's categories")
    for c in result.categories:
        if c.episodes < max(1, g.min_episodes // max(1, len(sc.required_categories))):
            out.append(f"{c.category}: too few episodes")
        elif c.successes / c.episodes < g.success_rate:
            out.append(f"{c.category}: success rate {c.successes / c.episodes:.3f} < {g.success_rate}")
        if g.throughput_ratio and c.useful_throughput < g.throughput_ratio * c.reference_throughput:
            out.append(f"{c.category}: throughput below {g.throughput_ratio:.0%} of the scripted reference")
        if c.useful_throughput < g.min_useful_throughput:
            out.append(f"{c.category}: useful throughput below minimum")
    return out


def evaluate_promotion(state: CurriculumState, result: EvaluationResult, *, retention_results=()) -> PromotionDecision:
    """Consume one validation round; mutates only progression state. A failing
    round (or failing retention) resets the scenario's streak."""
    if result.evaluation_id in state.seen_evaluation_ids:
        return PromotionDecision(False, False, ("duplicate evaluation ID",))
    if result.split != "validation":
        return PromotionDecision(False, False, ("promotion requires the validation split",))
    failures = gate_failures(result)
    anc = ancestors(result.scenario_id)
    if not anc <= state.qualified:
        failures.append("unqualified prerequisites")
    retained = {r.scenario_id: r for r in retention_results}
    if set(retained) != anc:
        failures.append("retention must cover every transitive prerequisite exactly")
    for name, r in retained.items():
        base = state.qualified_throughput.get(name, {})
        failures += [f"{name}: {f}" for f in gate_failures(r) if "throughput" not in f]
        for c in r.categories:
            if c.category not in base or c.useful_throughput < .9 * base[c.category]:
                failures.append(f"{name}/{c.category}: retention throughput regression")
    if result.evaluation_id:
        state.seen_evaluation_ids.add(result.evaluation_id)
    sid = result.scenario_id
    if failures:
        state.consecutive_passes[sid] = 0
        return PromotionDecision(False, False, tuple(failures))
    gate = get_scenario(sid).gate
    streak = min(gate.consecutive_evaluations, state.consecutive_passes.get(sid, 0) + 1)
    state.consecutive_passes[sid] = streak
    promoted = sid not in state.qualified and streak >= gate.consecutive_evaluations
    if promoted:
        state.qualified.add(sid)
        state.qualified_checkpoint[sid] = result.checkpoint_id
        state.qualified_throughput[sid] = {c.category: c.useful_throughput for c in result.categories}
    return PromotionDecision(promoted, True, ())


def eligible_scenarios(state: CurriculumState) -> tuple[str, ...]:
    return tuple(s for s in SCENARIOS if set(SCENARIOS[s].prerequisites) <= state.qualified)


def task_mixture(state: CurriculumState, current_ids, next_ids=()) -> dict[str, float]:
    cur, nxt = set(current_ids), set(next_ids)
    if not cur:
        raise ValueError("at least one current scenario is required")
    elig = set(eligible_scenarios(state))
    if not cur <= elig or not nxt <= elig:
        raise ValueError("unknown scenario or unqualified prerequisites")
    if cur & nxt:
        raise ValueError("current and next tasks must be disjoint")
    earlier = state.qualified - cur - nxt
    groups = [(cur, .7), (earlier, .2), (nxt, .1)]
    total = sum(w for g, w in groups if g)
    return {s: w / total / len(g) for g, w in groups if g for s in sorted(g)}


# ----------------------------------------------------------------------------- environment
def _hub_phase_time(active: bool, remaining: float = 24.) -> float:
    """Match-elapsed time (s) at which the red HUB (slot 0's alliance) is
    active / inactive with `remaining` seconds before it switches. With no
    AUTO winner the red HUB is inactive in the first shift (30-55 s) and
    active in the second (55-80 s)."""
    return (80. if active else 55.) - remaining


class CurriculumEnv:
    """Batched curriculum worlds: slot 0 is the neural offense robot, the
    other slots are parked, scripted teammates or scripted defenders per
    scenario. Placements are written straight into the device state."""

    def __init__(self, scenario_id: str, category: str, num_envs: int, device, seed: int = 0,
                 fuel_physics=False, action_ticks: int = 12):
        from ..sim.env3v3 import TensorThreeVsThreeEnv
        self.scenario = get_scenario(scenario_id)
        if category not in self.scenario.required_categories:
            raise ValueError(f"category {category!r} is not part of {scenario_id}")
        self.category = category
        modes = ["nn", "none", "none", "none", "none", "none"]
        level = category.rsplit("/", 1)[-1]
        if scenario_id in ("offense_vs_scripted_pressure", "full_match_offense"):
            # parked robots (mode none) are static blockers; deterministic
            # defense-role robots defend reactively
            if level in ("level_2_patrol", "level_4_reactive", "level_5_mixed"):
                modes[3] = "deterministic"
            if level in ("level_4_reactive", "level_5_mixed") or (scenario_id == "full_match_offense"
                                                                   and level != "level_0"):
                modes[4] = "deterministic"
        if scenario_id == "full_match_offense" or category.endswith("/multiple_teammates"):
            modes[1] = modes[2] = "deterministic"
        elif category.endswith("/receiver"):
            modes[1] = "deterministic"
        elif category.endswith("/opponents"):
            modes[3] = modes[4] = "deterministic"
        self.env = TensorThreeVsThreeEnv(num_envs=num_envs, device=device, seed=seed, fuel_physics=fuel_physics,
                                         control_modes=tuple(modes), allow_nn_offense=True,
                                         horizon=int(self.scenario.time_budget_s / .02) + 1)
        self.n, self.device = self.env.n, self.env.device
        self.action_ticks = int(action_ticks)
        self.budget_ticks = int(round(self.scenario.time_budget_s / self.env.dt))
        self.obs_dim, self.action_dim = 137, 8
        self.seed = int(seed)
        self.gen = torch.Generator(device="cpu")
        self.metrics = CurriculumMetrics(self.env)

    # scenario placement ---------------------------------------------------------
    def _place(self, mask: torch.Tensor, seed: int) -> None:
        env, ws, sid, cat = self.env, self.env.ws, self.scenario.scenario_id, self.category
        g = self.gen
        g.manual_seed(seed & 0x7FFFFFFFFFFFFFFF)
        n, P = self.n, env.fuel_count
        L, W = env.field_length, env.field_width
        depth = env.alliance_zone_depth
        m = mask.to(self.device)

        def rand(*shape):
            return torch.rand(shape, generator=g).to(self.device)

        parts = cat.split("/")
        route = next((r for r in _ROUTES if r in parts), None)
        # robot 0 pose: routes home through the open field, a trench or a bump
        x0 = depth + 1. + rand(n) * (L / 2 - depth - 2.)
        y0 = 1. + rand(n) * (W - 2.)
        if route == "trench":
            y0 = torch.where(rand(n) < .5, .6 + rand(n) * .5, W - 1.1 + rand(n) * .5)
            x0 = depth + 1.8 + rand(n) * 2.
        elif route == "bump":
            y0 = torch.where(rand(n) < .5, 2.2 + rand(n) * .6, W - 2.8 + rand(n) * .6)
            x0 = depth + 1.8 + rand(n) * 2.
        elif route == "open":
            y0 = W / 2 + (rand(n) * 2 - 1) * .6
        th0 = (rand(n) * 2 - 1) * math.pi
        hub = env.hub_centers[0].to(self.device)
        if sid in ("active_shoot_preloaded",):
            x0 = depth + .4 + rand(n) * 1.5
            if cat == "active/approach":
                x0 = depth + 1.5 + rand(n) * 1.5
            if cat == "active/heading_error":   # facing away from the HUB
                th0 = torch.atan2(hub[1] - y0, hub[0] - x0) + math.pi + (rand(n) * 2 - 1) * .5
        if sid == "inactive_ferry_preloaded":
            x0 = {"inactive/approach": depth + 4. + rand(n) * 2., "inactive/landing": depth + .8 + rand(n) * .4
                  }.get(cat, depth + 2. + rand(n) * 2.)
            if cat == "inactive/alignment":     # facing away from home
                th0 = rand(n) * .6 - .3
        transition = sid == "hub_transition_cycles" and "/" in cat
        if transition:
            situation = parts[-1]
            x0 = {"collecting": L / 2 - 1. + rand(n) * 1.5, "carrying_home": depth + 2. + rand(n) * 2.,
                  "approaching_shot": depth + .6 + rand(n) * .8, "before_release": depth + 2.5 + rand(n) * 2.,
                  "after_release": depth + 1.5 + rand(n) * 1.5, "staged_at_home": depth * .5 + rand(n) * 1.
                  }[situation]
        pose = ws["r_pose"].clone()
        pose[:, 0, 0], pose[:, 0, 1], pose[:, 0, 2] = x0, y0, th0
        ws["r_pose"].copy_(torch.where(m[:, None, None], pose, ws["r_pose"]))
        ws["est_pose"].copy_(torch.where(m[:, None, None], ws["r_pose"], ws["est_pose"]))
        ws["policy_pose"].copy_(torch.where(m[:, None, None], ws["r_pose"], ws["policy_pose"]))
        # FUEL: keep the match layout, then clear / place per scenario
        active = ws["f_active"].clone()
        owner = ws["f_owner"].clone()
        fx, fy = ws["f_pos"][:, 0].clone(), ws["f_pos"][:, 1].clone()
        if sid.startswith("pickup") or sid in ("active_carry_to_zone",) or cat == "empty_collection":
            keep = {"single": 1, "cluster": 6, "sparse": 10, "dense": 30, "initially_hidden": 8, "productive": 24,
                    "empty": 16, "depleted": 8, "empty_collection": 12}.get(cat, 12)
            active.zero_()
            owner.fill_(-1)
            idx = torch.arange(keep)
            if cat in ("single", "cluster", "dense", "initially_hidden"):
                # around a point ahead of the robot, or behind it (outside every camera's view)
                ahead = -1.5 if cat == "initially_hidden" else 1.5
                cx = (x0 + ahead * torch.cos(th0)).clamp(1., L - 1.)
                cy = (y0 + ahead * torch.sin(th0)).clamp(1., W - 1.)
                spread = {"dense": .8, "initially_hidden": .3}.get(cat, .15)
                px = cx[:, None] + (rand(n, keep) * 2 - 1) * spread
                py = cy[:, None] + (rand(n, keep) * 2 - 1) * spread
            elif cat in ("empty", "empty_collection"):
                # nothing within 3.5 m: the FUEL waits on the far side of the field
                far_x = torch.where(x0 < L / 2, x0 + 4.5, x0 - 4.5).clamp(1., L - 1.)
                px = far_x[:, None] + (rand(n, keep) * 2 - 1) * .8
                py = (W - y0)[:, None] + (rand(n, keep) * 2 - 1) * .8
            else:
                px = 1. + rand(n, keep) * (L - 2.)
                py = .5 + rand(n, keep) * (W - 1.)
            fx[:, idx], fy[:, idx] = px.clamp(.1, L - .1), py.clamp(.1, W - .1)
            active[:, idx] = 1
        load = 0
        if sid in ("active_shoot_preloaded", "inactive_ferry_preloaded", "active_carry_to_zone"):
            load = 3 if cat.endswith("partial_load") else (8 if cat.endswith("full_load") else 5)
        if transition:
            load = {"empty": 0, "partial": 3, "full": 8}[parts[1]]
            if parts[-1] == "staged_at_home":   # FUEL already staged in the home zone, robot empty
                staged = torch.arange(P - 12, P - 4)
                active[:, staged] = 1
                owner[:, staged] = -1
                fx[:, staged] = .3 + rand(n, 8) * (depth - .6)
                fy[:, staged] = .5 + rand(n, 8) * (W - 1.)
                load = 0
        if cat == "hold_useful_load":
            load = 5
        if load:
            slots = torch.arange(P - load, P)
            active[:, slots] = 1
            owner[:, slots] = 0
            fx[:, slots] = ws["r_pose"][:, 0, 0:1]
            fy[:, slots] = ws["r_pose"][:, 0, 1:2]
        fpos = ws["f_pos"].clone()
        fpos[:, 0], fpos[:, 1] = fx, fy
        fpos[:, 2] = env._spawn_height(torch.stack((fx, fy), -1))
        ws["f_pos"].copy_(torch.where(m[:, None, None], fpos, ws["f_pos"]))
        ws["f_active"].copy_(torch.where(m[:, None], active, ws["f_active"]))
        ws["f_owner"].copy_(torch.where(m[:, None], owner, ws["f_owner"]))
        # scripted blockers of the pressure scenarios: parked robots on the
        # route home, in a trench, on a bump or at a seeded choice of those
        level = parts[-1]
        if level in ("level_1_stationary", "level_3_trench", "level_3_bump", "level_3_seeded_choice",
                     "level_5_mixed"):
            upper = y0 > W / 2
            bx = torch.full((n,), 4.63, device=self.device)
            by_trench = torch.where(upper, torch.full_like(y0, 7.24), torch.full_like(y0, .83))
            by_bump = torch.where(upper, torch.full_like(y0, 5.56), torch.full_like(y0, 2.51))
            if level == "level_3_trench":
                by = by_trench
            elif level == "level_3_bump":
                by = by_bump
            elif level == "level_3_seeded_choice":
                by = torch.where(rand(n) < .5, by_trench, by_bump)
            else:   # on the straight line home, halfway
                bx, by = (x0 + depth) * .5, y0
            slot = 5 if level == "level_5_mixed" else 3
            bpose = ws["r_pose"].clone()
            bpose[:, slot, 0], bpose[:, slot, 1], bpose[:, slot, 2] = bx, by, 0.
            ws["r_pose"].copy_(torch.where(m[:, None, None], bpose, ws["r_pose"]))
            for name in ("est_pose", "policy_pose"):
                ws[name].copy_(torch.where(m[:, None, None], ws["r_pose"], ws[name]))
        # match clock / HUB phase
        hub_active = cat.startswith("active") or sid.startswith("active")
        if sid.startswith("inactive") or cat.startswith("inactive"):
            hub_active = False
        t = _hub_phase_time(hub_active)
        if sid == "hub_transition_cycles":
            if transition:    # now in the first phase, `timing` seconds before the switch
                remaining = 12. if parts[2] == "enough_time" else 2.5
                t = _hub_phase_time(parts[0] == "active_to_inactive", remaining)
            else:
                t = _hub_phase_time(cat == "empty_collection", 12.)
        if sid == "full_match_offense":
            t = 0.
        if not sid.startswith("pickup") or sid == "full_match_offense":
            ws["g_time"][:, 0].masked_fill_(m, t)
            ws["g_time"][:, 1].masked_fill_(m, 160. - t)

    def reset(self, seed: int | None = None) -> torch.Tensor:
        if seed is not None:
            self.seed = int(seed)
        self.env.reset(seed=self.seed & 0x7FFFFFFF, defer_perception=True)
        allm = torch.ones(self.n, dtype=torch.bool, device=self.device)
        self._place(allm, self.seed)
        self.env._perceive_and_observe(allm)
        self.elapsed = 0
        self.metrics.snapshot()
        return self.obs()

    def obs(self) -> torch.Tensor:
        return self.env.ws["obs"][:, 0].clone()

    def step(self, actions: torch.Tensor, ticks: int | None = None):
        ticks = self.action_ticks if ticks is None else int(ticks)
        ticks = max(1, min(ticks, self.budget_ticks - self.elapsed))
        full = torch.full((self.n, 6), 7, dtype=torch.int32, device=self.device)
        full[:, 0] = actions.to(torch.int32)
        before = self.metrics.progress()
        self.env.step_held(full, ticks)
        self.elapsed += ticks
        after = self.metrics.progress()
        reward = (after - before) - .001 * ticks
        done = torch.full((self.n,), self.elapsed >= self.budget_ticks, device=self.device)
        return self.obs(), reward, done


class CurriculumMetrics:
    """Physical outcome counters of slot 0 relative to the episode start:
    acquisitions, scored FUEL (team 0 score) and FUEL staged in the friendly
    alliance zone."""

    def __init__(self, env):
        self.env = env
        self.base = None

    def _raw(self):
        ws = self.env.ws
        acquired = ws["g_rcount"][:, 0, 0].float()
        scored = ws["g_scores"][:, 2].float()  # red (slot 0's team) FUEL scored, auto included
        free = ws["f_active"].bool() & (ws["f_owner"] < 0)
        staged = (free & (ws["f_pos"][:, 0] < self.env.alliance_zone_depth)).float().sum(-1)
        held = (ws["f_active"].bool() & (ws["f_owner"] == 0)).float().sum(-1)
        return torch.stack((acquired, scored, staged, held), -1)

    def snapshot(self):
        self.base = self._raw()

    def counts(self) -> dict:
        d = self._raw() - self.base
        raw = self._raw()
        return {"acquired": d[:, 0], "scored": d[:, 1], "staged": d[:, 2], "held": raw[:, 3]}

    def progress(self) -> torch.Tensor:
        c = self.counts()
        return .5 * c["acquired"] + 2. * c["scored"] + c["staged"].clamp_min(0.)


def episode_success(scenario_id: str, category: str, counts: dict, env: CurriculumEnv) -> torch.Tensor:
    a, s, st, held = counts["acquired"], counts["scored"], counts["staged"], counts["held"]
    if scenario_id == "pickup_simple":
        return a >= (1 if category == "single" else 3)
    if scenario_id == "pickup_scattered":
        return a >= (3 if category == "sparse" else 6)
    if scenario_id == "pickup_multi_zone":
        return a >= 5
    if scenario_id == "active_carry_to_zone":
        x = env.env.ws["r_pose"][:, 0, 0]
        return (held > 0) & (x < env.env.alliance_zone_depth + 1.)
    if scenario_id == "active_shoot_preloaded":
        return s >= 1
    if scenario_id == "inactive_ferry_preloaded":
        return st >= 1
    if scenario_id in ("active_collect_carry_score", "offense_vs_scripted_pressure"):
        return s >= 2
    if scenario_id == "inactive_collect_ferry":
        return st >= 2
    if scenario_id == "hub_transition_cycles":
        return s + st >= 2
    return s >= 3


# ----------------------------------------------------------------------------- teachers
class D1HandWeightedPolicy:
    """Scripted teacher: score when carrying and the HUB is active, ferry when
    carrying and it is inactive, otherwise collect the nearest candidate."""

    name = "d1_hand_weighted"

    def choose(self, env: CurriculumEnv, observation=None) -> torch.Tensor:
        ws = env.env.ws
        held = (ws["f_active"].bool() & (ws["f_owner"] == 0)).sum(-1)
        cap = env.env.robot_fuel_capacities[0]
        hub = ws["g_hub"][:, 0].bool()
        act = torch.zeros(env.n, dtype=torch.long, device=env.device)
        act = torch.where((held > 0) & hub, torch.full_like(act, 4), act)
        act = torch.where((held > 0) & ~hub, torch.full_like(act, 6), act)
        act = torch.where((held >= cap) & hub, torch.full_like(act, 4), act)
        return act


class D2PredictivePolicy(D1HandWeightedPolicy):
    """D1 plus HUB-switch prediction: keep collecting while the active window
    outlasts the expected trip, and hold a load for an imminent activation."""

    name = "d2_predictive"

    def choose(self, env: CurriculumEnv, observation=None) -> torch.Tensor:
        act = super().choose(env, observation)
        ws = env.env.ws
        elapsed = ws["g_time"][:, 0]
        teleop = (elapsed - 20.).clamp_min(0.)
        to_switch = 30. - torch.remainder(teleop, 30.)
        held = (ws["f_active"].bool() & (ws["f_owner"] == 0)).sum(-1)
        hub = ws["g_hub"][:, 0].bool()
        cap = env.env.robot_fuel_capacities[0]
        # inactive but about to activate: hold the load for a direct shot
        act = torch.where(~hub & (held > 0) & (to_switch < 4.), torch.full_like(act, 4), act)
        # active with little time left and a partial load: shoot now
        act = torch.where(hub & (held > 0) & (held < cap) & (to_switch < 6.), torch.full_like(act, 4), act)
        return act


# ----------------------------------------------------------------------------- training
@dataclass
class TrainingConfig:
    output: str
    scenarios: tuple[str, ...] = ("pickup_simple",)
    architecture: str = "baseline_mlp"
    algorithm: str = "ppo"
    envs: int = 64
    updates: int = 20
    rollout_decisions: int = 32
    eval_every: int = 5
    eval_episodes: int = 32
    learning_rate: float = 3e-4
    seed: int = 0
    device: str = "cpu"
    action_ticks: int = 12
    fuel_physics: bool = False

    def validate(self) -> None:
        for s in self.scenarios:
            get_scenario(s)
        if self.algorithm not in ("ppo", "sac"):
            raise ValueError("algorithm must be ppo or sac")
        if min(self.envs, self.updates, self.rollout_decisions, self.eval_every, self.eval_episodes) < 1:
            raise ValueError("sizes must be positive")

    def identity(self) -> str:
        d = asdict(self)
        d.pop("updates")  # a resumed run may extend its budget
        return hashlib.sha256(json.dumps(d, sort_keys=True).encode()).hexdigest()[:16]


def _atomic_json(path: Path, value: dict) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(value, indent=2, default=str))
    tmp.replace(path)


def _atomic_save(path: Path, value) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(value, tmp)
    tmp.replace(path)


@torch.no_grad()
def evaluate_scenario(policy, scenario_id: str, *, episodes: int, split: str = "validation", master_seed: int = 0,
                      device="cpu", fuel_physics=False, teacher=None, action_ticks: int = 12) -> EvaluationResult:
    """Run `episodes` seeded episodes per category (one batched env per category)."""
    sc = get_scenario(scenario_id)
    seeds = seed_partition(scenario_id, split, len(sc.required_categories))
    cats = []
    for seed, cat in zip(seeds, sc.required_categories):
        env = CurriculumEnv(scenario_id, cat, episodes, device, seed=seed ^ master_seed, fuel_physics=fuel_physics,
                            action_ticks=action_ticks)
        obs = env.reset()
        done = torch.zeros(env.n, dtype=torch.bool, device=env.device)
        while not bool(done.all()):
            if teacher is not None:
                act = teacher.choose(env, obs)
            else:
                act, _, _ = policy.sample(obs, deterministic=True, action_mask=obs[:, -8:] > .5)
            obs, _, done = env.step(act)
        counts = env.metrics.counts()
        ok = episode_success(scenario_id, cat, counts, env)
        seconds = env.elapsed * env.env.dt
        useful = float((counts["scored"] + counts["staged"].clamp_min(0) + .25 * counts["acquired"]).mean()) / seconds
        cats.append(CategoryResult(cat, episodes, int(ok.sum()), useful, 0.))
    return EvaluationResult(f"{scenario_id}/{split}/{master_seed}/{time.time_ns()}", scenario_id, split, tuple(cats))


def evaluate_curriculum(policy_or_checkpoint, scenario_ids, *, episodes: int, split: str = "validation",
                        master_seed: int = 0, device="cpu") -> dict:
    policy = policy_or_checkpoint
    if isinstance(policy_or_checkpoint, (str, Path)):
        policy, _ = load_checkpoint(policy_or_checkpoint, device=device)
    out = {}
    for sid in scenario_ids:
        res = evaluate_scenario(policy, sid, episodes=episodes, split=split, master_seed=master_seed, device=device)
        out[sid] = {"success_rate": res.successes / max(1, res.episodes),
                    "wilson_95": wilson_interval(res.successes, res.episodes),
                    "categories": [asdict(c) for c in res.categories]}
    return out


def load_checkpoint(path, *, config: TrainingConfig | None = None, device="cpu"):
    from ..utils.checkpoint import load_verified
    payload = load_verified(path, map_location=device, weights_only=False)
    if payload.get("curriculum_version") != CURRICULUM_VERSION:
        raise ValueError("checkpoint from another curriculum version")
    if config is not None and payload.get("config_identity") != config.identity():
        raise ValueError("checkpoint configuration does not match this run (strict resume)")
    from ..models.zoo import make_policy
    policy = make_policy(payload["architecture"], tensor_cores=False).to(device)
    policy.load_state_dict(payload["model_state_dict"])
    return policy, payload


def train_curriculum(config: TrainingConfig, *, resume: str | None = None) -> dict:
    """PPO (or SAC) on the scenario mixture with periodic validation and promotion."""
    from .ppo import PPOConfig, PPOLearner
    from .rollout import gae_advantages
    from .sac import DiscreteSAC, ScenarioReplayBuffer, make_sac_optimizers, sac_update
    config.validate()
    out = Path(config.output)
    out.mkdir(parents=True, exist_ok=True)
    dev = torch.device(config.device)
    torch.manual_seed(config.seed)
    state = CurriculumState()
    cfg = PPOConfig(rollout_steps=config.rollout_decisions, epochs=4, minibatch_size=max(64, config.envs * 4),
                    learning_rate=config.learning_rate, grad_backend="local")
    learner = sac = None
    if config.algorithm == "ppo":
        net = "mlp" if config.architecture == "baseline_mlp" else config.architecture
        learner = PPOLearner(137, 8, "categorical", dev, cfg, net, 1)
        model = learner.model
    else:
        sac = DiscreteSAC(config.architecture).to(dev)
        sac_opt = make_sac_optimizers(sac, config.learning_rate)
        replay = ScenarioReplayBuffer(50_000, device=dev)
        model = sac
    start = 0
    if resume:
        from ..utils.checkpoint import load_verified
        payload = load_verified(resume, map_location=dev, weights_only=False)
        if payload.get("config_identity") != config.identity():
            raise ValueError("checkpoint configuration does not match this run (strict resume)")
        model.load_state_dict(payload["model_state_dict"])
        if learner is not None:
            learner.weights_changed()
        state = CurriculumState.from_dict(payload["curriculum_state"])
        start = int(payload["update"])
        torch.set_rng_state(payload["rng"])
    history = []
    current = [s for s in config.scenarios if s not in state.qualified][:1] or [config.scenarios[-1]]
    for update in range(start, config.updates):
        elig = [s for s in eligible_scenarios(state) if s in config.scenarios or s in current]
        cur = [s for s in current if s in elig] or [s for s in config.scenarios if s in elig][:1] or list(elig[:1])
        mix = task_mixture(state, cur, [])
        names, weights = zip(*mix.items())
        sid = names[int(torch.multinomial(torch.tensor(weights), 1))]
        sc = get_scenario(sid)
        cat = sc.required_categories[update % len(sc.required_categories)]
        seed = seed_partition(sid, "train", update + 1, master_seed=config.seed)[-1]
        env = CurriculumEnv(sid, cat, config.envs, dev, seed=seed, fuel_physics=config.fuel_physics,
                            action_ticks=config.action_ticks)
        obs = env.reset()
        T = config.rollout_decisions
        bufs = {k: [] for k in ("obs", "actions", "mask", "logp", "values", "rewards", "dones", "next_obs")}
        for _ in range(T):
            mask = obs[:, -8:] > .5
            if learner is not None:
                act, logp, value, mask = learner.act(obs)
            else:
                act, logp, value = sac.sample(obs, action_mask=mask)
            nobs, rew, done = env.step(act)
            for k, v in (("obs", obs), ("actions", act), ("mask", mask), ("logp", logp), ("values", value),
                         ("rewards", rew), ("dones", done), ("next_obs", nobs)):
                bufs[k].append(v)
            obs = nobs
            if bool(done.all()):
                obs = env.reset(seed=seed + env.elapsed + 1)
        B = {k: torch.stack(v) for k, v in bufs.items()}
        if learner is not None:
            nv = torch.cat((B["values"][1:], learner.value(obs)[None]))
            stats = torch.zeros(3, dtype=torch.float64, device=dev)
            trunc = torch.zeros_like(B["dones"])
            adv = gae_advantages(B["rewards"].float(), B["dones"], trunc, B["values"].float(), nv.float(),
                                 cfg.gamma, cfg.gae_lambda, stats)
            flat = {"obs": B["obs"].reshape(-1, 137), "actions": B["actions"].reshape(-1),
                    "mask": B["mask"].reshape(-1, 8), "logp": B["logp"].reshape(-1), "adv": adv.reshape(-1),
                    "returns": (adv + B["values"]).reshape(-1)}
            upd = learner.update(flat, cfg.entropy_coef)
            info = {"entropy": float(upd["entropy_sum"]) / max(1, upd["batches"])}
        else:
            rows = {"obs": B["obs"].reshape(-1, 137), "mask": B["mask"].reshape(-1, 8),
                    "action": B["actions"].reshape(-1), "reward": B["rewards"].reshape(-1),
                    "next_obs": B["next_obs"].reshape(-1, 137), "next_mask": B["next_obs"].reshape(-1, 137)[:, -8:] > .5,
                    "done": B["dones"].reshape(-1)}
            replay.add_batch(rows, sid)
            info = {}
            for _ in range(max(1, T // 4)):
                if len(replay) >= 256:
                    info = {k: float(v) for k, v in sac_update(sac, sac_opt, replay.sample(256), gamma=.99, tau=.01,
                                                               target_entropy_fraction=.5).items()}
        entry = {"update": update, "scenario": sid, "category": cat,
                 "mean_reward": float(B["rewards"].float().mean()), **info}
        if (update + 1) % config.eval_every == 0:
            policy = learner.model if learner is not None else sac
            for target in cur:
                res = evaluate_scenario(policy, target, episodes=config.eval_episodes, device=dev,
                                        master_seed=config.seed, fuel_physics=config.fuel_physics,
                                        action_ticks=config.action_ticks)
                retention = [evaluate_scenario(policy, a, episodes=config.eval_episodes, device=dev,
                                               master_seed=config.seed, fuel_physics=config.fuel_physics,
                                               action_ticks=config.action_ticks)
                             for a in sorted(ancestors(target))]
                retention = [EvaluationResult(res.evaluation_id, r.scenario_id, r.split, r.categories)
                             for r in retention]
                dec = evaluate_promotion(state, res, retention_results=retention)
                entry.setdefault("evaluations", []).append(
                    {"scenario": target, "success_rate": res.successes / max(1, res.episodes),
                     "promoted": dec.promoted, "failures": list(dec.failures)[:6]})
                if dec.promoted:
                    nxt = [s for s in config.scenarios if s not in state.qualified and s in eligible_scenarios(state)]
                    current = nxt[:1] or current
        history.append(entry)
        payload = {"curriculum_version": CURRICULUM_VERSION, "config": asdict(config),
                   "config_identity": config.identity(), "architecture": config.architecture,
                   "algorithm": config.algorithm, "model_state_dict": model.state_dict(),
                   "curriculum_state": state.to_dict(), "update": update + 1, "rng": torch.get_rng_state()}
        _atomic_save(out / "curriculum.pt", payload)
        _atomic_json(out / "curriculum-status.json",
                     {"state": "running", "update": update + 1, "updates": config.updates,
                      "qualified": sorted(state.qualified), "current": current, "last": entry})
    result = {"state": "complete", "updates": config.updates, "qualified": sorted(state.qualified),
              "history": history}
    _atomic_json(out / "curriculum-status.json", {k: v for k, v in result.items() if k != "history"})
    return result


def build_parser(parser: argparse.ArgumentParser | None = None) -> argparse.ArgumentParser:
    p = parser or argparse.ArgumentParser(prog="curriculum", description="offense curriculum")
    p.add_argument("command", choices=("train", "evaluate", "teacher"))
    p.add_argument("--output", default="runs/curriculum")
    p.add_argument("--scenarios", default="pickup_simple")
    p.add_argument("--architecture", default="baseline_mlp")
    p.add_argument("--algorithm", choices=("ppo", "sac"), default="ppo")
    p.add_argument("--envs", type=int, default=64)
    p.add_argument("--updates", type=int, default=20)
    p.add_argument("--rollout-decisions", type=int, default=32)
    p.add_argument("--eval-every", type=int, default=5)
    p.add_argument("--episodes", type=int, default=32)
    p.add_argument("--learning-rate", type=float, default=3e-4)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default="cpu")
    p.add_argument("--checkpoint")
    p.add_argument("--resume")
    p.add_argument("--teacher", choices=("d1", "d2"), default="d1")
    return p


def main(argv=None) -> dict:
    args = build_parser().parse_args(argv)
    scenarios = tuple(s.strip() for s in args.scenarios.split(",") if s.strip())
    if args.command == "train":
        cfg = TrainingConfig(output=args.output, scenarios=scenarios, architecture=args.architecture,
                             algorithm=args.algorithm, envs=args.envs, updates=args.updates,
                             rollout_decisions=args.rollout_decisions, eval_every=args.eval_every,
                             eval_episodes=args.episodes, learning_rate=args.learning_rate, seed=args.seed,
                             device=args.device)
        res = train_curriculum(cfg, resume=args.resume)
    elif args.command == "evaluate":
        if not args.checkpoint:
            raise SystemExit("--checkpoint is required for evaluate")
        res = evaluate_curriculum(args.checkpoint, scenarios, episodes=args.episodes, device=args.device)
    else:
        teacher = D1HandWeightedPolicy() if args.teacher == "d1" else D2PredictivePolicy()
        res = {}
        for sid in scenarios:
            r = evaluate_scenario(None, sid, episodes=args.episodes, device=args.device, teacher=teacher)
            res[sid] = {"success_rate": r.successes / max(1, r.episodes),
                        "categories": [asdict(c) for c in r.categories]}
    print(json.dumps({k: v for k, v in res.items() if k != "history"}, default=str))
    return res


if __name__ == "__main__":
    main()
