"""Seeded, matched evaluation of defense checkpoints.

Mirrors frc_defense/tensor_training_evaluation.py:45-617: a checkpoint is
loaded, every world of one batch plays a seeded scenario, and the report
carries scoring, acquisition, denial, defensive delay, cycle time (simulated
seconds from a piece's acquisition to its score), passing (FUEL ferried by a
robot: attempted, completed = next acquired by the passer's alliance, failed
= next acquired by the other alliance, fuel transferred = landed in the
passer's alliance zone, pass-to-score = seconds from the pass to that
piece's score by the passer's alliance) and per-robot opponent acquisitions,
with Wilson score intervals (Wilson, "Probable inference...", JASA 1927) on
the success rate.

* `evaluate_once`: the two-robot env, the learned defender against one
  scripted attacker (the reference's evaluation path); passing needs an
  allied receiver, so its pass metrics are reported unavailable as in the
  reference.
* `evaluate_3v3_once`: full 3v3 matches, the checkpoint controlling the
  three defenders against the deterministic offense (robots 0-2), with
  observations and decisions at the strategic rate; any network the trainer
  supports (the 137-feature MLPs or the perception-input zoo).
"""
from __future__ import annotations

import math
import time
from pathlib import Path
from typing import Any

import torch

from ..models import build_policy
from .ppo import atomic_json
from .rollout import StrategicClock

SCRIPTED_BASELINES = ("offense", "adstar", "mirror", "cutoff", "velocity_intercept")


def wilson_interval(successes: int, total: int, z: float = 1.96) -> tuple[float, float]:
    if total <= 0:
        return 0., 1.
    p = successes / total
    denom = 1. + z * z / total
    centre = (p + z * z / (2 * total)) / denom
    half = z * math.sqrt(p * (1 - p) / total + z * z / (4 * total * total)) / denom
    return max(0., centre - half), min(1., centre + half)


class GameMetricTracker:
    """Per-tick bookkeeping of piece ownership for cycle-time and passing
    metrics (owner transitions of every FUEL piece), for any robot count."""

    def __init__(self, env, team_ids):
        dev = env.device
        self.env = env
        self.team = torch.as_tensor(team_ids, device=dev).long()
        n, P = env.piece_owner.shape
        R = len(team_ids)
        self.prev = env.piece_owner.clone()
        self.acquired_at = torch.zeros((n, P), device=dev)
        self.pass_team = torch.full((n, P), -1, device=dev, dtype=torch.long)
        self.pass_time = torch.zeros((n, P), device=dev)
        self.cycle_sum = torch.zeros((n, R), device=dev)
        self.cycle_count = torch.zeros((n, R), device=dev)
        z = lambda: torch.zeros((n, 2), device=dev)  # noqa: E731 - per alliance
        self.passes_attempted, self.passes_completed, self.failed_passes = z(), z(), z()
        self.fuel_transferred, self.pass_to_score_sum, self.pass_to_score_count = z(), z(), z()

    @torch.no_grad()
    def update(self, now_s: torch.Tensor, active: torch.Tensor) -> None:
        env = self.env
        owner = env.piece_owner
        prev = self.prev
        zone = env.ws["f_zone"].long()
        scored = env.fuel_scored_event > 0
        passed = env.ws["g_rcount"][:, :, 4] > 0
        t = now_s[:, None]
        act = active[:, None]
        for r in range(self.team.numel()):
            team = int(self.team[r])
            got = (owner == r) & (prev != r) & act
            # a piece acquired by robot r: resolve an open pass of that piece
            from_pass = got & (self.pass_team >= 0)
            same = from_pass & (self.pass_team == team)
            self.passes_completed[:, team] += same.sum(-1)
            other = from_pass & (self.pass_team != team)
            for k in (0, 1):
                self.failed_passes[:, k] += (other & (self.pass_team == k)).sum(-1)
            self.pass_team = torch.where(other, torch.full_like(self.pass_team, -1), self.pass_team)
            self.acquired_at = torch.where(got, t.expand_as(self.acquired_at), self.acquired_at)
            released = (prev == r) & (owner != r) & act
            as_score = released & scored[:, r:r + 1]
            held = (t - self.acquired_at).clamp_min(0.)
            self.cycle_sum[:, r] += (held * as_score).sum(-1)
            self.cycle_count[:, r] += as_score.sum(-1)
            # scores of pieces passed by this alliance close a pass-to-score cycle
            closing = as_score & (self.pass_team == team)
            self.pass_to_score_sum[:, team] += ((t - self.pass_time) * closing).sum(-1)
            self.pass_to_score_count[:, team] += closing.sum(-1)
            self.pass_team = torch.where(as_score, torch.full_like(self.pass_team, -1), self.pass_team)
            as_pass = released & passed[:, r:r + 1] & ~as_score
            self.passes_attempted[:, team] += as_pass.sum(-1)
            self.fuel_transferred[:, team] += (as_pass & (zone == team + 1)).sum(-1)
            self.pass_team = torch.where(as_pass, torch.full_like(self.pass_team, team), self.pass_team)
            self.pass_time = torch.where(as_pass, t.expand_as(self.pass_time), self.pass_time)
        self.prev = owner.clone()

    def world_row(self, k: int, robots, alliance: int) -> dict:
        """Metrics of world k for the robots `robots` of `alliance`."""
        cnt = float(self.cycle_count[k, list(robots)].sum())
        p2s = float(self.pass_to_score_count[k, alliance])
        return {"cycle_time": float(self.cycle_sum[k, list(robots)].sum()) / cnt if cnt else None,
                "passes_attempted": float(self.passes_attempted[k, alliance]),
                "passes_completed": float(self.passes_completed[k, alliance]),
                "failed_passes": float(self.failed_passes[k, alliance]),
                "fuel_transferred": float(self.fuel_transferred[k, alliance]),
                "pass_to_score_cycle_time": float(self.pass_to_score_sum[k, alliance]) / p2s if p2s else None}


def _optional_mean(rows, key):
    vals = [float(r[key]) for r in rows if r.get(key) is not None]
    return sum(vals) / len(vals) if vals else None


def load_policy(checkpoint, device):
    from ..utils.checkpoint import load_verified
    payload = load_verified(checkpoint, map_location=device)
    network = payload.get("network", "mlp")
    model = build_policy(network, int(payload["obs_dim"]), int(payload["action_dim"]), payload["action_kind"])
    model.load_state_dict(payload["model_state_dict"])
    return model.to(device).eval(), payload


@torch.no_grad()
def evaluate_once(checkpoint, task: str = "defense", episodes: int = 4, seed: int = 1000, num_envs: int = 4,
                  device="cpu", opponent: str = "offense", output=None, horizon: int = 8000,
                  strategic_rate_hz: float = 4., capture_playback: bool = False,
                  scripted_strategy: int | None = None, fuel_physics=True) -> dict[str, Any]:
    """Play `episodes` matched worlds (batched `num_envs` at a time).

    Without a checkpoint the learner slot plays the fixed strategic action
    `scripted_strategy` (default 5, defend) — the scripted ablation rows.
    """
    from ..sim.env_defense import TensorDefenseEnv
    device = torch.device(device)
    model, payload = (load_policy(checkpoint, device) if checkpoint else (None, {}))
    architecture = payload.get("architecture", "strategic_adstar")
    mode = {"direct": "direct", "tactical_adstar": "tactical", "strategic_adstar": "strategic"}.get(
        architecture, "strategic")
    started = time.perf_counter()
    rows, frames = [], []
    remaining, batch_index = episodes, 0
    dt = .02
    while remaining > 0:
        n = min(num_envs, remaining)
        env = TensorDefenseEnv(num_envs=n, task="defense", device=device, seed=seed + batch_index * 7919,
                               opponent=opponent,
                               horizon=horizon, action_mode=mode, randomize=True, fuel_physics=fuel_physics)
        dt = env.dt
        obs, _ = env.reset(seed=seed + batch_index * 7919)
        clock = StrategicClock(strategic_rate_hz) if mode == "strategic" else None
        ticks = 0
        total = torch.zeros(n, device=device)
        first_score = torch.full((n,), float(horizon), device=device)
        tracker = GameMetricTracker(env, (0, 1))
        all_active = torch.ones(n, dtype=torch.bool, device=device)
        while ticks < env.horizon:
            if model is None:
                action = torch.full((n,), 5 if scripted_strategy is None else scripted_strategy,
                                    dtype=torch.long, device=device)
            elif mode == "strategic":
                logits, _, _ = model(obs)
                action = logits.masked_fill(~(obs[:, -8:] > .5), torch.finfo(logits.dtype).min).argmax(-1)
            else:
                action = torch.tanh(model(obs)[0])
            hold = clock.next() if clock else 1
            for _ in range(hold):
                obs, r, _, _, _ = env.step(action, _return_info=False)
                total += r
                ticks += 1
                tracker.update(env.match_elapsed, all_active)
                scored = env.fuel_score_count[:, 1] > 0
                first_score = torch.where(scored & (first_score >= horizon),
                                          torch.full_like(first_score, ticks), first_score)
                if capture_playback and batch_index == 0 and ticks % 25 == 0:
                    frames.append({"tick": ticks, "pose": env.sim.pose[0].tolist(),
                                   "fuel": env.piece_pos[0][env.piece_active[0]].tolist()[:64],
                                   "score": env.fuel_score_count[0].tolist()})
                if ticks >= env.horizon:
                    break
        own = env.fuel_score_count[:, 0].float()
        other = env.fuel_score_count[:, 1].float()
        acq = env.fuel_acquisition_count[:, 1].float()
        denied = env.fuel_denied_count[:, 1].float()
        own_acq = env.fuel_acquisition_count[:, 0].float()
        for k in range(n):
            attacker = tracker.world_row(k, (1,), 1)
            rows.append({"return": float(total[k]), "scores": float(own[k]), "opponent_scores": float(other[k]),
                         "acquisitions": float(own_acq[k]), "opponent_acquisitions": float(acq[k]),
                         "opponent_acquisitions_by_robot": [float(acq[k])], "denied": float(denied[k]),
                         "defensive_delay_s": float(first_score[k]) * dt, "success": bool(other[k] == 0),
                         "cycle_time": tracker.world_row(k, (0,), 0)["cycle_time"],
                         "opponent_cycle_time": attacker["cycle_time"]})
        remaining -= n
        batch_index += 1
    elapsed = time.perf_counter() - started
    successes = sum(r["success"] for r in rows)
    lo, hi = wilson_interval(successes, len(rows))

    def mean(key):
        return sum(float(r[key]) for r in rows) / max(1, len(rows))

    metrics = {"task": task, "opponent": opponent, "episodes": len(rows), "seed": seed, "horizon": horizon,
               "checkpoint": str(checkpoint) if checkpoint else None,
               "mean_return": mean("return"), "mean_scores": mean("scores"),
               "mean_opponent_scores": mean("opponent_scores"), "mean_acquisitions": mean("opponent_acquisitions"),
               "mean_own_acquisitions": mean("acquisitions"),
               "mean_opponent_acquisitions": mean("opponent_acquisitions"),
               "mean_denied_objectives": mean("denied"), "mean_defensive_delay": mean("defensive_delay_s"),
               "mean_cycle_time": _optional_mean(rows, "cycle_time"),
               "mean_opponent_cycle_time": _optional_mean(rows, "opponent_cycle_time"),
               "mean_passes_attempted": None, "mean_passes_completed": None, "mean_fuel_transferred": None,
               "mean_failed_passes": None, "mean_pass_to_score_cycle_time": None,
               "cycle_time_units": "simulated seconds from piece acquisition to scoring",
               "unavailable_metrics": ["passing (no allied teammate in the two-robot simulator)"],
               "mean_success": successes / max(1, len(rows)), "success_wilson_95": [lo, hi],
               "elapsed_seconds": elapsed,
               "physics_world_ticks_per_second": len(rows) * horizon / max(elapsed, 1e-9),
               "episodes_detail": rows}
    if output is not None:
        out = Path(output)
        out.parent.mkdir(parents=True, exist_ok=True)
        atomic_json(out, metrics)
        if capture_playback:
            atomic_json(out.with_name("playback.json"), {"frames": frames})
    return metrics


@torch.no_grad()
def evaluate_3v3_once(checkpoint, episodes: int = 4, seed: int = 1000, num_envs: int = 4, device="cpu",
                      output=None, horizon: int = 8000, strategic_rate_hz: float = 4., fuel_physics=True,
                      scripted_strategy: int | None = None, env_kwargs: dict | None = None) -> dict[str, Any]:
    """Full 3v3 matches: the checkpoint's policy controls robots 3-5 (blue
    defense) with greedy masked actions at the strategic rate; robots 0-2 play
    the deterministic offense. Without a checkpoint the three defenders hold
    the fixed strategic action `scripted_strategy` (default 5, defend)."""
    from ..sim.env3v3 import TensorThreeVsThreeEnv
    from .rollout import ThreeVsThreeAgents
    device = torch.device(device)
    model, payload = (load_policy(checkpoint, device) if checkpoint else (None, {}))
    perception = model is not None and hasattr(model, "input_keys")
    started = time.perf_counter()
    rows = []
    remaining, batch_index = episodes, 0
    dt = .02
    while remaining > 0:
        n = min(num_envs, remaining)
        env = TensorThreeVsThreeEnv(num_envs=n, device=device, seed=seed + batch_index * 7919, horizon=horizon,
                                    control_modes=("deterministic",) * 3 + ("nn",) * 3, fuel_physics=fuel_physics,
                                    **(env_kwargs or {}))
        dt = env.dt
        agents = ThreeVsThreeAgents(env)
        if perception:
            agents.use_perception(model.field_shape, model.input_keys)
        obs = agents.reset()
        tracker = GameMetricTracker(env, env.team_ids)
        clock = StrategicClock(strategic_rate_hz)
        total = torch.zeros(n, device=device)
        active = torch.ones(n, dtype=torch.bool, device=device)
        first_score = torch.full((n,), float(horizon), device=device)
        full = torch.full((n, 6), 7, dtype=torch.int32, device=device)
        ticks = 0
        while ticks < horizon:
            if model is None:
                action = torch.full((n * 3,), 5 if scripted_strategy is None else scripted_strategy,
                                    dtype=torch.long, device=device)
            else:
                with torch.autocast(device.type, dtype=torch.bfloat16, enabled=perception and device.type == "cuda"):
                    logits = model(obs)[0].float()
                scalars = obs["scalars"] if isinstance(obs, dict) else obs
                action = logits.masked_fill(~(scalars[:, -8:] > .5), torch.finfo(logits.dtype).min).argmax(-1)
            full[:, 3:] = action.reshape(n, 3).to(torch.int32)
            env._set_actions(full)
            hold = min(clock.next(), horizon - ticks)
            for k in range(hold):
                _, r, _, _, _ = env.step(None, capture_observation=k == hold - 1, capture_info=False)
                total += r[:, 3]
                ticks += 1
                tracker.update(env.match_elapsed, active)
                scored = env.fuel_score_count[:, 0] > 0
                first_score = torch.where(scored & (first_score >= horizon), torch.full_like(first_score, ticks),
                                          first_score)
            obs = agents._agent_obs()
        red = env.fuel_score_count[:, 0].float()
        blue = env.fuel_score_count[:, 1].float()
        acq = env.fuel_acquisition_count.float()
        denied = env.fuel_denied_count.float()
        for k in range(n):
            offense = tracker.world_row(k, (0, 1, 2), 0)
            defense = tracker.world_row(k, (3, 4, 5), 1)
            rows.append({"return": float(total[k]), "scores": float(blue[k]), "opponent_scores": float(red[k]),
                         "acquisitions": float(acq[k, 3:].sum()), "opponent_acquisitions": float(acq[k, :3].sum()),
                         "opponent_acquisitions_by_robot": acq[k, :3].tolist(),
                         "denied": float(denied[k, :3].sum()), "defensive_delay_s": float(first_score[k]) * dt,
                         "success": bool(blue[k] >= red[k]), "cycle_time": defense["cycle_time"],
                         "opponent_cycle_time": offense["cycle_time"],
                         **{f"opponent_{key}": val for key, val in offense.items() if key != "cycle_time"},
                         **{key: val for key, val in defense.items() if key != "cycle_time"}})
        remaining -= n
        batch_index += 1
    elapsed = time.perf_counter() - started
    successes = sum(r["success"] for r in rows)
    lo, hi = wilson_interval(successes, len(rows))
    per_robot = [sum(r["opponent_acquisitions_by_robot"][i] for r in rows) / max(1, len(rows)) for i in range(3)]
    metrics = {"task": "defense", "env": "3v3", "opponent": "deterministic_offense", "episodes": len(rows),
               "seed": seed, "horizon": horizon, "checkpoint": str(checkpoint) if checkpoint else None,
               "network": payload.get("network"),
               "mean_return": _optional_mean(rows, "return"), "mean_scores": _optional_mean(rows, "scores"),
               "mean_opponent_scores": _optional_mean(rows, "opponent_scores"),
               "mean_acquisitions": _optional_mean(rows, "opponent_acquisitions"),
               "mean_own_acquisitions": _optional_mean(rows, "acquisitions"),
               "mean_opponent_acquisitions": _optional_mean(rows, "opponent_acquisitions"),
               "mean_opponent_acquisitions_by_robot": per_robot,
               "mean_denied_objectives": _optional_mean(rows, "denied"),
               "mean_defensive_delay": _optional_mean(rows, "defensive_delay_s"),
               "mean_cycle_time": _optional_mean(rows, "cycle_time"),
               "mean_opponent_cycle_time": _optional_mean(rows, "opponent_cycle_time"),
               **{f"mean_{key}": _optional_mean(rows, key) for key in (
                   "passes_attempted", "passes_completed", "failed_passes", "fuel_transferred",
                   "pass_to_score_cycle_time", "opponent_passes_attempted", "opponent_passes_completed",
                   "opponent_failed_passes", "opponent_fuel_transferred", "opponent_pass_to_score_cycle_time")},
               "cycle_time_units": "simulated seconds from piece acquisition to scoring",
               "success_definition": "defense alliance score >= offense alliance score",
               "mean_success": successes / max(1, len(rows)), "success_wilson_95": [lo, hi],
               "elapsed_seconds": elapsed,
               "physics_world_ticks_per_second": len(rows) * horizon / max(elapsed, 1e-9),
               "episodes_detail": rows}
    if output is not None:
        out = Path(output)
        out.parent.mkdir(parents=True, exist_ok=True)
        atomic_json(out, metrics)
    return metrics


def evaluate(checkpoint, *, task="defense", episodes=32, seed=1000, num_envs=32, device="cuda",
             opponent="random", output="metrics/tensor-evaluation.json", horizon=8000, env_kind=None) -> dict:
    """Evaluate a checkpoint; 3v3 checkpoints (perception networks, or
    `env_kind="3v3"`) play full 3v3 matches, others the two-robot env."""
    if env_kind is None and checkpoint:
        from ..utils.checkpoint import load_verified
        payload = load_verified(checkpoint, map_location="cpu")
        env_kind = payload.get("env", "defense")
    if env_kind == "3v3":
        return evaluate_3v3_once(checkpoint, episodes, seed, num_envs, device, output, horizon)
    return evaluate_once(checkpoint, task, episodes, seed, num_envs, device, opponent, output, horizon,
                         capture_playback=True)


def evaluate_game_ablations(*, defense_checkpoint=None, episodes=8, seed=4100, num_envs=8, device="cuda",
                            output="metrics/ablations.json", horizon=8000, strategic_rate_hz=4.,
                            capture_playback=False) -> dict:
    """Each scripted attacker vs the learned defender, a fixed 'defend' and a fixed 'hold' learner."""
    rows = []
    for opponent in SCRIPTED_BASELINES:
        for name, ckpt, fixed in (("learned", defense_checkpoint, None), ("scripted_defend", None, 5),
                                  ("scripted_hold", None, 7)):
            if name == "learned" and defense_checkpoint is None:
                rows.append({"name": name, "opponent": opponent, "missing_reason": "no defense checkpoint"})
                continue
            m = evaluate_once(ckpt, "defense", episodes, seed, num_envs, device, opponent, None, horizon,
                              strategic_rate_hz, False, fixed)
            m.pop("episodes_detail", None)
            rows.append({"name": name, **m})
    result = {"ablations": rows, "seed": seed, "episodes": episodes, "horizon": horizon}
    out = Path(output)
    out.parent.mkdir(parents=True, exist_ok=True)
    atomic_json(out, result)
    return result
