"""Generational PPO with a strong/diverse checkpoint archive.

Per generation (frc_defense/tensor_training_generational.py:13-384): continue
PPO from the previous checkpoint on every rank, evaluate the new checkpoint on
rank 0 against the fixed scripted baselines on a shared seeded batch, snapshot
it into ``opponent-population/generation-NNNN.pt``, keep the top-``elite``
fitness snapshots plus max-min cosine-diverse ones up to the pool capacity,
and publish ``generation-history.json`` / ``population.json`` /
``status.json``. A restarted run resumes from the recorded history.
"""
from __future__ import annotations

import json
import math
import shutil
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Any

import torch

from ..parallel import dist as pdist
from .evaluation import SCRIPTED_BASELINES, evaluate_3v3_once, evaluate_once
from .ppo import atomic_json, train_once


def checkpoint_vector(path) -> torch.Tensor:
    from ..utils.checkpoint import load_verified
    payload = load_verified(path)
    return torch.cat([v.detach().float().reshape(-1) for v in payload["model_state_dict"].values()])


def select_checkpoint_population(entries: list[dict], capacity: int, elite_count: int) -> list[dict]:
    """Top-fitness elites first, then the candidate whose minimum cosine distance
    to the kept set is largest (ties broken by fitness)."""
    ranked = sorted(entries, key=lambda e: float(e.get("fitness", -math.inf)), reverse=True)
    if len(ranked) <= capacity:
        return ranked
    shortlist = ranked[:max(capacity * 4, elite_count)]
    selected = shortlist[:min(elite_count, capacity)]
    vectors = {e["checkpoint"]: checkpoint_vector(e["checkpoint"]) for e in shortlist}
    while len(selected) < capacity:
        remaining = [e for e in shortlist if e not in selected]
        if not remaining:
            break

        def key(e):
            dmin = min((float(1. - torch.nn.functional.cosine_similarity(
                vectors[e["checkpoint"]], vectors[k["checkpoint"]], dim=0)) for k in selected), default=0.)
            return dmin, float(e.get("fitness", -math.inf))
        selected.append(max(remaining, key=key))
    return selected


def dispatch_evaluations(specs, evaluator, workers: int = 1, device="cpu"):
    """Ordered evaluations, optionally on worker threads with private CUDA streams."""
    if workers < 1:
        raise ValueError("evaluation_workers must be positive")
    if workers == 1:
        return [evaluator(i, s, None) for i, s in enumerate(specs)]
    dev = torch.device(device)

    def run(i, spec):
        if dev.type != "cuda":
            return evaluator(i, spec, None)
        stream = torch.cuda.Stream(device=dev)
        with torch.cuda.device(dev), torch.cuda.stream(stream):
            result = evaluator(i, spec, stream)
            stream.synchronize()
            return result
    with ThreadPoolExecutor(max_workers=workers, thread_name_prefix="ppo-opponent-eval") as pool:
        futures = [pool.submit(run, i, s) for i, s in enumerate(specs)]
        return [f.result() for f in futures]


def generational_train(task: str, generations: int, output, *, seed: int = 7, num_envs: int = 1024,
                       device="cuda", opponent: str | None = None, initial_checkpoint=None, horizon: int = 8000,
                       population_size: int = 8, elite_count: int = 2, l2_coef: float = 1e-5,
                       architecture: str = "strategic_adstar", timesteps: int | None = None,
                       rollout_steps: int = 128, epochs: int = 4, minibatch_size: int = 4096,
                       learning_rate: float = 3e-4, gamma: float = .993, gae_lambda: float = .95,
                       clip_coef: float = .2, value_coef: float = .5, entropy_coef: float = .01,
                       max_grad_norm: float = .5, evaluation_episodes: int = 4, strategic_rate_hz: float = 4.,
                       evaluation_workers: int = 1, network: str = "mlp", env_kind: str = "defense",
                       fuel_physics=True, grad_backend: str = "auto", **_ignored) -> dict[str, Any]:
    if task != "defense":
        raise ValueError("only defense policies are trainable; offense is deterministic")
    if min(generations, num_envs, horizon, population_size, elite_count, rollout_steps, epochs,
           minibatch_size, evaluation_episodes) < 1:
        raise ValueError("generation, environment, horizon, population, PPO, and evaluation sizes must be positive")
    if elite_count > population_size:
        raise ValueError("elite_count cannot exceed opponent population capacity")
    state = pdist.distributed_state(device)
    rank, world = state.rank, state.world
    try:
        if num_envs % world:
            raise ValueError(f"global num_envs={num_envs} must divide evenly across {world} ranks")
        if minibatch_size % world:
            raise ValueError(f"global minibatch_size={minibatch_size} must divide evenly across {world} ranks")
        local_envs = num_envs // world
        out = Path(output)
        archive = out / "opponent-population"
        if rank == 0:
            archive.mkdir(parents=True, exist_ok=True)
        pdist.barrier()
        checkpoint, status_path = out / "policy.pt", out / "status.json"
        history_path, population_path = out / "generation-history.json", archive / "population.json"
        history, members, start_gen = [], [], 0
        if history_path.exists():
            prior = json.loads(history_path.read_text())
            history = list(prior.get("generations", []))
            start_gen = max((int(h.get("generation", 0)) for h in history), default=0)
            if population_path.exists():
                members = json.loads(population_path.read_text()).get("members", [])
        previous = checkpoint if (start_gen and checkpoint.exists()) else initial_checkpoint
        per_generation = timesteps // max(1, generations) if timesteps else rollout_steps * num_envs * 2
        train_opponent = opponent or "mixed"
        started = time.perf_counter()
        final: dict[str, Any] = {}
        for generation in range(start_gen, generations):
            number = generation + 1
            spec = pdist.broadcast_object({"name": train_opponent, "mode": train_opponent})
            gen_started = time.perf_counter()
            ppo = train_once(task, max(1, per_generation // world), out, seed=seed + generation * 1009,
                             num_envs=local_envs, device=state.device, opponent=spec["mode"],
                             initial_checkpoint=previous, rollout_steps=rollout_steps, epochs=epochs,
                             minibatch_size=minibatch_size // world, learning_rate=learning_rate, gamma=gamma,
                             gae_lambda=gae_lambda, clip_coef=clip_coef, value_coef=value_coef,
                             entropy_coef=entropy_coef, max_grad_norm=max_grad_norm, l2_coef=l2_coef,
                             horizon=horizon, architecture=architecture, curriculum=True,
                             strategic_rate_hz=strategic_rate_hz, env_kind=env_kind, network=network,
                             fuel_physics=fuel_physics, grad_backend=grad_backend,
                             status_context={"generation": number, "total_generations": generations},
                             dist_state=state)
            previous = checkpoint
            pdist.barrier()
            if rank != 0:
                pdist.barrier()
                continue
            scenario_seed = 500_000 + generation * 1009
            eval_dir = out / "generation-evaluations" / f"generation-{number:04d}"
            if env_kind == "3v3":   # the 3v3 defenders always face the deterministic offense
                specs = [{"name": "deterministic_offense", "mode": "deterministic_offense"}]
            else:
                specs = [{"name": m, "mode": m} for m in SCRIPTED_BASELINES]

            def run(index, s, _stream):
                path = eval_dir / f"{s['name']}.json"
                try:
                    if env_kind == "3v3":
                        return evaluate_3v3_once(checkpoint, evaluation_episodes, scenario_seed,
                                                 evaluation_episodes, state.device, path, horizon,
                                                 strategic_rate_hz, fuel_physics=fuel_physics), None
                    return evaluate_once(checkpoint, task, evaluation_episodes, scenario_seed,
                                         evaluation_episodes, state.device, s["mode"], path, horizon,
                                         strategic_rate_hz, fuel_physics=fuel_physics), None
                except (OSError, RuntimeError, ValueError, KeyError) as exc:
                    return None, str(exc)
            results = {}
            for s, (metrics, error) in zip(specs, dispatch_evaluations(specs, run, evaluation_workers,
                                                                        state.device)):
                if error is not None:
                    results[s["name"]] = {"opponent": s["mode"], "error": error}
                    continue
                results[s["name"]] = {
                    "opponent": s["mode"], "success_rate": metrics["mean_success"],
                    "mean_return": metrics["mean_return"], "score": metrics["mean_scores"],
                    "score_differential": metrics["mean_scores"] - metrics["mean_opponent_scores"],
                    "mean_opponent_score": metrics["mean_opponent_scores"],
                    "fuel_acquired": metrics["mean_acquisitions"],
                    "defensive_delay": metrics["mean_defensive_delay"],
                    "denied_per_episode": metrics["mean_denied_objectives"],
                    "seed": scenario_seed, "episodes": metrics["episodes"]}
            ok = [r for r in results.values() if "error" not in r]
            fitness = sum(float(r.get("success_rate") or 0.) + 1e-3 * float(r.get("mean_return") or 0.)
                          for r in ok) / max(1, len(ok))
            snapshot = archive / f"generation-{number:04d}.pt"
            tmp = snapshot.with_suffix(".pt.tmp")
            shutil.copy2(checkpoint, tmp)
            tmp.replace(snapshot)
            members = [m for m in members if m.get("checkpoint") != str(snapshot.resolve())]
            members.append({"generation": number, "checkpoint": str(snapshot.resolve()), "fitness": fitness,
                            "evaluation_seed": scenario_seed, "evaluated_opponents": sorted(results)})
            kept = select_checkpoint_population(members, population_size, elite_count)
            keep = {str(Path(m["checkpoint"]).resolve()) for m in kept}
            for m in members:
                if str(Path(m["checkpoint"]).resolve()) not in keep:
                    Path(m["checkpoint"]).unlink(missing_ok=True)
            members = kept
            atomic_json(population_path, {"task": task, "capacity": population_size,
                                          "strong_elites": min(elite_count, population_size), "members": members})
            record = {"generation": number, "training_optimizer": "PPO", "training_opponent": spec["name"],
                      "ppo": {k: v for k, v in ppo.items() if k != "history"}, "fitness": fitness,
                      "opponent_metrics": results, "scenario_seed": scenario_seed,
                      "generation_wall_clock_seconds": time.perf_counter() - gen_started,
                      "population_members": [m["checkpoint"] for m in members], "population_size": len(members)}
            history = [h for h in history if int(h.get("generation", 0)) != number] + [record]
            atomic_json(history_path, {"algorithm": "ppo_opponent_population", "task": task,
                                       "generations": history})
            final = {"status": "running" if number < generations else "completed", "algorithm": "generational",
                     "optimizer": "PPO", "task": task, "generation": number, "total_generations": generations,
                     "population_size": len(members), "population_capacity": population_size,
                     "elite_count": min(elite_count, population_size), "opponent_metrics": results,
                     "best_fitness": max(float(h.get("fitness", -math.inf)) for h in history),
                     "transitions_per_second": ppo.get("transitions_per_second"),
                     "physics_world_ticks_per_second": ppo.get("physics_world_ticks_per_second"),
                     "elapsed_seconds": time.perf_counter() - started, "world_size": world,
                     "population_manifest": str(population_path), "generation_history_path": str(history_path),
                     "checkpoint": str(checkpoint)}
            atomic_json(status_path, final)
            pdist.barrier()
        if rank != 0:
            return {"status": "completed", "rank": rank, "world_size": world, "task": task,
                    "checkpoint": str(checkpoint)}
        final = {**final, "status": "completed", "generation_history": history}
        atomic_json(status_path, final)
        atomic_json(out / "metadata.json", {k: v for k, v in final.items() if k != "generation_history"})
        return final
    finally:
        pdist.teardown(state)
