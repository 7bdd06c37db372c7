"""Seeded, matched evaluation of defense checkpoints against scripted attackers.

Mirrors frc_defense/tensor_training_evaluation.py:45-184: a checkpoint is
loaded, every world of one batch plays the same seeded scenario against a
fixed scripted attacker, and the report carries scoring, acquisition, denial
and defensive-delay statistics with Wilson score intervals
(Wilson, "Probable inference...", JASA 1927) on the success rate.
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
        env = TensorDefenseEnv(num_envs=n, device=device, seed=seed + batch_index * 7919, opponent=opponent,
                               horizon=horizon, action_mode=mode, randomize=True, fuel_physics=fuel_physics)
        dt = env.dt
        obs, _ = env.reset(seed=seed + batch_index * 7919)
        clock = StrategicClock(strategic_rate_hz) if mode == "strategic" else None
        ticks = 0
        total = torch.zeros(n, device=device)
        first_score = torch.full((n,), float(horizon), device=device)
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
        for k in range(n):
            rows.append({"return": float(total[k]), "scores": float(own[k]), "opponent_scores": float(other[k]),
                         "acquisitions": float(acq[k]), "denied": float(denied[k]),
                         "defensive_delay_s": float(first_score[k]) * dt, "success": bool(other[k] == 0)})
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
               "mean_opponent_scores": mean("opponent_scores"), "mean_acquisitions": mean("acquisitions"),
               "mean_denied_objectives": mean("denied"), "mean_defensive_delay": mean("defensive_delay_s"),
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


def evaluate(checkpoint, *, task="defense", episodes=32, seed=1000, num_envs=32, device="cuda",
             opponent="random", output="metrics/tensor-evaluation.json", horizon=8000) -> dict:
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
