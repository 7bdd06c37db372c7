"""Command-line interface: ``python -m frc_defense.tensor_training <command>``.

Commands and flags follow frc_defense/tensor_training.py:343-433 (``train``,
``evaluate``, ``evaluate-game-ablations``, ``curriculum``), plus:

* ``--network``       policy network (``mlp``, ``mlp256``, ``entity``, ``cnn`` ...);
                      ``--architecture`` keeps its meaning (action mode)
* ``--env``           ``defense`` (two-robot env, default) or ``3v3`` (three learned defenders)
* ``--fuel-physics``  / ``--no-fuel-physics``
* ``--grad-backend``  ``auto`` | ``nccl`` | ``p2p`` (fused peer-memory all-reduce + clip + Adam)
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
from pathlib import Path

from .ppo import DEFENSE_TRAINING_OPPONENTS


def train(task="defense", timesteps=1_000_000, output="checkpoints/tensor-ppo", *, seed=7, num_envs=1024,
          device="cuda", opponent=None, initial_checkpoint=None, rollout_steps=128, epochs=4,
          minibatch_size=4096, learning_rate=3e-4, gamma=.993, gae_lambda=.95, clip_coef=.2, value_coef=.5,
          entropy_coef=.01, max_grad_norm=.5, l2_coef=1e-5, horizon=8000, algorithm="generational",
          generations=20, population_size=8, elite_count=2, architecture="strategic_adstar",
          strategic_rate_hz=4., evaluation_episodes=4, evaluation_workers=1, network="mlp",
          env_kind="defense", fuel_physics=True, grad_backend="auto"):
    if task != "defense":
        raise ValueError("only defense policies are trainable; offense is deterministic")
    if opponent is not None and opponent not in (*DEFENSE_TRAINING_OPPONENTS, "mixed"):
        raise ValueError("opponent must be a deterministic defense-training baseline")
    if algorithm not in ("generational", "ppo"):
        raise ValueError("algorithm must be 'generational' or 'ppo'")
    if min(timesteps, num_envs, rollout_steps, epochs, minibatch_size, horizon) < 1:
        raise ValueError("timesteps, num_envs, rollout_steps, epochs, minibatch_size and horizon must be positive")
    if not math.isfinite(l2_coef) or l2_coef < 0:
        raise ValueError("l2_coef must be finite and non-negative")
    common = dict(seed=seed, num_envs=num_envs, initial_checkpoint=initial_checkpoint,
                  rollout_steps=rollout_steps, epochs=epochs,
                  minibatch_size=min(minibatch_size, rollout_steps * num_envs),
                  learning_rate=learning_rate, gamma=gamma, gae_lambda=gae_lambda, clip_coef=clip_coef,
                  value_coef=value_coef, entropy_coef=entropy_coef, max_grad_norm=max_grad_norm,
                  l2_coef=l2_coef, horizon=horizon, architecture=architecture,
                  strategic_rate_hz=strategic_rate_hz, network=network, env_kind=env_kind,
                  fuel_physics=fuel_physics, grad_backend=grad_backend)
    if algorithm == "generational":
        from .generational import generational_train
        return generational_train(task, generations, output, device=device, opponent=opponent,
                                  timesteps=timesteps, population_size=population_size, elite_count=elite_count,
                                  evaluation_episodes=evaluation_episodes,
                                  evaluation_workers=evaluation_workers, **common)
    # Unlike the reference (generational only), plain PPO also runs under torchrun.
    from ..parallel import dist as pdist
    from .ppo import train_once
    state = pdist.distributed_state(device)
    try:
        return train_once(task, timesteps, output, opponent=opponent or "mixed",
                          curriculum=(opponent is None or opponent == "mixed"), dist_state=state,
                          device=state.device, **common)
    finally:
        pdist.teardown(state)


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(description="Tensor-resident FRC defense learning (B200-native)")
    commands = parser.add_subparsers(dest="command", required=True)
    commands.add_parser("curriculum", help="Outcome-gated offense curriculum: plan, train, evaluate, teacher")
    p = commands.add_parser("train")
    p.add_argument("--task", choices=("defense",), default="defense")
    p.add_argument("--steps", type=int, default=1_000_000)
    p.add_argument("--envs", type=int, default=1024)
    p.add_argument("--rollout-steps", type=int, default=128)
    p.add_argument("--strategic-rate-hz", type=float, default=4.)
    p.add_argument("--gamma", type=float, default=.993)
    p.add_argument("--entropy-coef", type=float, default=.01)
    p.add_argument("--horizon", type=int, default=8000)
    p.add_argument("--seed", type=int, default=7)
    p.add_argument("--opponent")
    p.add_argument("--epochs", type=int, default=4)
    p.add_argument("--minibatch-size", type=int, default=4096)
    p.add_argument("--algorithm", choices=("generational", "ppo"), default="generational")
    p.add_argument("--architecture", choices=("strategic_adstar", "tactical_adstar", "direct"),
                   default="strategic_adstar")
    p.add_argument("--network", default="mlp")
    p.add_argument("--env", dest="env_kind", choices=("defense", "3v3"), default="defense")
    p.add_argument("--fuel-physics", action=argparse.BooleanOptionalAction, default=True)
    p.add_argument("--grad-backend", choices=("auto", "nccl", "p2p", "gloo"), default="auto")
    p.add_argument("--generations", type=int, default=20)
    p.add_argument("--evaluation-episodes", type=int, default=4,
                   help="seeded episodes per opponent at each generation boundary")
    p.add_argument("--evaluation-workers", type=int, default=1,
                   help="concurrent CUDA stream workers for generation evaluation")
    p.add_argument("--population", "--opponent-pool-size", dest="population", type=int, default=8)
    p.add_argument("--elites", "--strong-checkpoints", dest="elites", type=int, default=2)
    p.add_argument("--l2-coef", type=float, default=1e-5)
    p.add_argument("--initial-checkpoint")
    p.add_argument("--output", default="checkpoints/tensor-ppo")
    p.add_argument("--device", default="cuda")
    e = commands.add_parser("evaluate")
    e.add_argument("--task", choices=("defense",), default="defense")
    e.add_argument("--checkpoint", required=True)
    e.add_argument("--episodes", type=int, default=32)
    e.add_argument("--horizon", type=int, default=8000)
    e.add_argument("--envs", type=int, default=32)
    e.add_argument("--seed", type=int, default=1000)
    e.add_argument("--opponent", default="random")
    e.add_argument("--output", default="metrics/tensor-evaluation.json")
    e.add_argument("--device", default="cuda")
    a = commands.add_parser("evaluate-game-ablations")
    a.add_argument("--defense-checkpoint")
    a.add_argument("--episodes", type=int, default=8)
    a.add_argument("--horizon", type=int, default=8000)
    a.add_argument("--envs", type=int, default=8)
    a.add_argument("--seed", type=int, default=4100)
    a.add_argument("--output", default="metrics/ablations.json")
    a.add_argument("--device", default="cuda")
    return parser


def main(argv=None) -> None:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "curriculum":
        from .curriculum import main as curriculum_main
        curriculum_main(argv[1:])
        return
    parser = build_parser()
    args = parser.parse_args(argv)
    try:
        if args.command == "train":
            result = train(args.task, args.steps, args.output, seed=args.seed, num_envs=args.envs,
                           device=args.device, opponent=args.opponent, rollout_steps=args.rollout_steps,
                           epochs=args.epochs, minibatch_size=args.minibatch_size,
                           initial_checkpoint=args.initial_checkpoint, horizon=args.horizon,
                           l2_coef=args.l2_coef, algorithm=args.algorithm, generations=args.generations,
                           population_size=args.population, elite_count=args.elites,
                           architecture=args.architecture, strategic_rate_hz=args.strategic_rate_hz,
                           gamma=args.gamma, entropy_coef=args.entropy_coef,
                           evaluation_episodes=args.evaluation_episodes,
                           evaluation_workers=args.evaluation_workers, network=args.network,
                           env_kind=args.env_kind, fuel_physics=args.fuel_physics,
                           grad_backend=args.grad_backend)
        elif args.command == "evaluate":
            from .evaluation import evaluate
            result = evaluate(args.checkpoint, task=args.task, episodes=args.episodes, seed=args.seed,
                              num_envs=args.envs, device=args.device, opponent=args.opponent,
                              output=args.output, horizon=args.horizon)
            result.pop("episodes_detail", None)
        elif args.command == "evaluate-game-ablations":
            from .evaluation import evaluate_game_ablations
            result = evaluate_game_ablations(defense_checkpoint=args.defense_checkpoint, episodes=args.episodes,
                                             seed=args.seed, num_envs=args.envs, device=args.device,
                                             output=args.output, horizon=args.horizon)
        else:
            parser.error("use `curriculum` as the first argument for the curriculum CLI")
            return
    except Exception as exc:
        if args.command == "train" and int(os.environ.get("RANK", "0")) == 0:
            out = Path(args.output)
            out.mkdir(parents=True, exist_ok=True)
            (out / "status.json").write_text(json.dumps({"status": "failed", "error": str(exc)}))
        raise
    print(json.dumps(result, sort_keys=True, default=str))


if __name__ == "__main__":
    main()
