"""Headline benchmark: 3v3 env-ticks/s and PPO samples/s on 1..8 B200 (one process per GPU).

Default workload (`--mode train`), one step = one PPO training iteration of
the 3v3 defense configuration on every GPU:
  * TensorThreeVsThreeEnv, 2048 worlds per GPU, fuel physics on (400 FUEL,
    64 robot+FUEL substeps per 20 ms tick), stereo perception and strategic
    observations every tick, route replanning every 20 ticks on the
    reference's 0.3 m grid (56 x 27 cells), three scripted offense robots and three learned
    defenders sharing one 137->8 ActorCritic (random init, fp32);
  * a rollout of `--decisions` strategic decisions held 12/13 ticks each
    (4 Hz), the GAE kernel, then PPO with 4 epochs x 8 minibatches, gradient
    averaging over the ranks and the fused clip + Adam kernels.
`value` is simulated env-ticks per second over the whole job (all GPUs);
`ppo_samples_per_s` is agent transitions per second trained on.

`--mode sim` times the simulator alone: every world advances
`--ticks-per-step` ticks under held actions and builds observations.

Timing: CUDA events on the launching stream, W warm-up steps, K timed steps
bracketed by barrier + synchronize, max over ranks. The state touched per
step (FUEL, tracks, routes: ~0.25 GB per GPU) exceeds the 126 MB L2.

End-to-end (`e2e`): the same step through the public training/env API with
the step's control inputs copied from pinned host memory every step and the
step's result statistics read back to the host every step.

`--impl reference` runs the unmodified reference package from baseline/_ref
through its own public API on the same configuration.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "3v3 env-ticks/sec and PPO samples/sec, 1/2/4/8 B200, device-timed max over ranks"
# The 3v3 full-match benchmark world: 400 FUEL, perception and strategic
# observations every tick. Routes are planned on the 0.3 m grid (56 x 27)
# that the reference's 3v3 environment always uses (it has no resolution
# keyword), so both arms plan on the same grid; the finer 0.1 m grid is
# available through `planner_resolution`. (The reference's own defaults are
# 504 FUEL and perception every 2nd tick.)
BENCH_ENV = {"fuel_count": 400, "perception_interval": 1, "planner_resolution": .3}


def _dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def _max_over_ranks(value: float, world: int) -> float:
    import torch
    import torch.distributed as dist
    if world <= 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _timed(fn, steps, world):
    import torch
    _barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    stop.record()
    _barrier(world)
    return _max_over_ranks(start.elapsed_time(stop), world)


def run_train(args, rank, world, local):
    import torch
    sys.path.insert(0, HERE)
    from autodrive_b200.train.ppo import PPOConfig, PPOLearner, collect_rollout, make_env
    from autodrive_b200.train.rollout import StrategicClock, gae_advantages
    from autodrive_b200.utils.clocks import ClockSampler
    dev = torch.device("cuda", local)
    agents = make_env("3v3", args.envs, dev, args.seed + rank * 1_000_003, "offense", 8000, fuel_physics=True,
                      **BENCH_ENV)
    samples = agents.n_agents * args.decisions
    cfg = PPOConfig(rollout_steps=args.decisions, epochs=args.epochs,
                    minibatch_size=samples // args.minibatches, grad_backend=args.grad_backend)
    learner = PPOLearner(agents.obs_dim, agents.action_dim, "categorical", dev, cfg, "mlp", world)
    state = {"obs": agents.reset(), "clock": StrategicClock(4.), "ep": [0], "ticks": 0}
    control_dev = torch.tensor([cfg.entropy_coef, 0.], device=dev)
    stats_dev = torch.zeros(4, device=dev)

    phases = {"on": False, "events": []}

    def mark():
        if phases["on"]:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            phases["events"][-1].append(ev)

    def step():
        if phases["on"]:
            phases["events"].append([])
        mark()
        buf, state["obs"], ticks = collect_rollout(agents, learner, state["obs"], args.decisions,
                                                   state["clock"], state["ep"])
        state["ticks"] += ticks
        mark()
        stats = torch.zeros(3, dtype=torch.float64, device=dev)
        adv = gae_advantages(buf["rewards"], buf["dones"], buf["truncated"], buf["values"],
                             buf["next_values"], cfg.gamma, cfg.gae_lambda, stats)
        flat = {"obs": buf["obs"].reshape(-1, agents.obs_dim), "actions": buf["actions"].reshape(-1),
                "mask": buf["mask"].reshape(-1, agents.action_dim), "logp": buf["logp"].reshape(-1),
                "adv": adv.reshape(-1), "returns": (adv + buf["values"]).reshape(-1)}
        mark()
        upd = learner.update(flat, control_dev[0])
        mark()
        stats_dev[0] = buf["rewards"].mean()
        stats_dev[1] = upd["approx_kl_sum"] / max(1, upd["samples"])
        stats_dev[2] = upd["entropy_sum"] / max(1, upd["batches"])
        stats_dev[3] = learner.opt.last_norm[0]

    for _ in range(args.warmup):
        step()
    ticks_before = state["ticks"]
    phases["on"] = True
    with ClockSampler(local) as clocks:
        ms = _timed(step, args.steps, world)
    phases["on"] = False
    torch.cuda.synchronize()
    breakdown = {"rollout": 0., "gae": 0., "update": 0.}
    for ev in phases["events"]:
        breakdown["rollout"] += ev[0].elapsed_time(ev[1])
        breakdown["gae"] += ev[1].elapsed_time(ev[2])
        breakdown["update"] += ev[2].elapsed_time(ev[3])
    breakdown = {k: round(v / max(1, len(phases["events"])), 3) for k, v in breakdown.items()}
    ticks_timed = state["ticks"] - ticks_before
    env_ticks = args.envs * ticks_timed * world
    value = env_ticks / (ms / 1e3)
    samples_total = samples * args.steps * world
    # end to end: H2D control block and D2H result statistics every step
    host_control = torch.tensor([cfg.entropy_coef, 0.]).pin_memory()
    host_stats = torch.zeros(4).pin_memory()

    def e2e_step():
        control_dev.copy_(host_control, non_blocking=True)
        step()
        host_stats.copy_(stats_dev, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        _ = float(host_stats[0])

    for _ in range(args.warmup):
        e2e_step()
    t0 = state["ticks"]
    e2e_ms = _timed(e2e_step, args.steps, world)
    e2e_ticks = args.envs * (state["ticks"] - t0) * world
    decisions_ticks = ticks_timed / max(1, args.steps)
    minibatches = args.epochs * args.minibatches
    # own kernels per step: control+plan+tick+sense per tick, observe + policy act per decision, the
    # bootstrap value, GAE, and per minibatch either (adv stats, fused fwd+bwd, partial reduce,
    # sum-of-squares, Adam, weight pack) on the tensor-core path or (sum-of-squares, Adam)
    per_mb = 6 if learner.tc is not None else 2
    per_decision = 2 if learner.tc is not None else 1
    launches = int(args.steps * (decisions_ticks * 4 + per_decision * args.decisions + 2 + per_mb * minibatches))
    return {
        "metric": METRIC, "value": value, "unit": "env-ticks/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (random-init seeded REBUILT matches and policy; no external data)",
        "ppo_samples_per_s": samples_total / (ms / 1e3), "ppo_samples_per_step_per_gpu": samples,
        "config": {"model": "TensorThreeVsThreeEnv 3v3 full match (fuel physics on, 400 FUEL, 64 substeps/tick, "
                            "perception every tick, 0.3 m planner grid 56x27 as in the reference, replan every 20 ticks) "
                            "+ PPO on the strategic_adstar ActorCritic 137->128->128->8 for 3 learned defenders",
                   "global_batch": args.envs * world, "envs_per_gpu": args.envs,
                   "seq_len": args.decisions, "decisions_per_step": args.decisions,
                   "env_ticks_per_step_per_world": decisions_ticks, "ppo_epochs": args.epochs,
                   "ppo_minibatches": args.minibatches, "grad_backend": learner.sync.backend,
                   "parallelism": f"env-batch x dp{world}",
                   "l2": "working set > 126 MB L2 (no flush needed)"},
        "clocks": clocks.summary(),
        "e2e": {"value": e2e_ticks / (e2e_ms / 1e3), "unit": "env-ticks/s",
                "ppo_samples_per_s": samples_total / (e2e_ms / 1e3),
                "h2d_bytes_per_step": host_control.numel() * 4, "d2h_bytes_per_step": host_stats.numel() * 4},
        "gpu_launches": launches,
        "breakdown_ms_per_step": breakdown,
        "policy_kernels": "tcgen05" if learner.tc is not None else "torch",
        "final_stats": {"mean_reward": float(stats_dev[0]), "approx_kl": float(stats_dev[1]),
                        "entropy": float(stats_dev[2]), "grad_norm": float(stats_dev[3])},
    }


def run_train_zoo(args, rank, world, local):
    """PPO step with a perception-input zoo policy (e.g. the ~4M-parameter
    entity encoder, d = 256, 4 heads, 2 blocks) in bf16 autocast."""
    import torch
    sys.path.insert(0, HERE)
    from autodrive_b200.bench.zoo_ppo import ZooPPO
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    from autodrive_b200.utils.clocks import ClockSampler
    dev = torch.device("cuda", local)
    env = TensorThreeVsThreeEnv(num_envs=args.envs, device=dev, seed=args.seed + rank * 1_000_003,
                                control_modes=("deterministic",) * 3 + ("nn",) * 3, fuel_physics=True,
                                horizon=8000, **BENCH_ENV)
    ppo = ZooPPO(env, args.network, world, epochs=args.epochs, minibatches=args.minibatches,
                 grad_backend=args.grad_backend)
    state = {"ticks": 0, "upd": None, "events": None}
    stats_dev = torch.zeros(3, device=dev)

    def step():
        ev = None
        if state["events"] is not None:
            ev = []
            state["events"].append(ev)
        ticks, upd = ppo.step(args.decisions, ev)
        state["ticks"] += ticks
        stats_dev[0] = upd["mean_reward"]
        stats_dev[1] = upd["approx_kl_sum"] / max(1, upd["batches"])
        stats_dev[2] = upd["entropy_sum"] / max(1, upd["batches"])

    for _ in range(args.warmup):
        step()
    t0 = state["ticks"]
    state["events"] = []
    with ClockSampler(local) as clocks:
        ms = _timed(step, args.steps, world)
    torch.cuda.synchronize()
    breakdown = {"rollout": sum(e[0].elapsed_time(e[1]) for e in state["events"]) / args.steps,
                 "update": sum(e[1].elapsed_time(e[2]) for e in state["events"]) / args.steps}
    state["events"] = None
    ticks_timed = state["ticks"] - t0
    value = args.envs * ticks_timed * world / (ms / 1e3)
    samples = args.envs * 3 * args.decisions
    host_stats = torch.zeros(3).pin_memory()
    host_seed = torch.tensor([float(args.seed)]).pin_memory()
    seed_dev = torch.zeros(1, device=dev)

    def e2e_step():
        seed_dev.copy_(host_seed, non_blocking=True)
        step()
        host_stats.copy_(stats_dev, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        _ = float(host_stats[0])

    t1 = state["ticks"]
    e2e_ms = _timed(e2e_step, args.steps, world)
    e2e_ticks = args.envs * (state["ticks"] - t1) * world
    return {
        "metric": METRIC, "value": value, "unit": "env-ticks/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init seeded REBUILT matches and policy; no external data)",
        "ppo_samples_per_s": samples * args.steps * world / (ms / 1e3), "ppo_samples_per_step_per_gpu": samples,
        "config": {"model": f"TensorThreeVsThreeEnv 3v3 full match (fuel physics on, 400 FUEL, perception every "
                            f"tick) + PPO on PerceptionActorCritic {args.network} ({ppo.params} parameters, "
                            f"bf16 autocast, fp32 master) for 3 learned defenders",
                   "global_batch": args.envs * world, "envs_per_gpu": args.envs, "seq_len": args.decisions,
                   "ppo_epochs": args.epochs, "ppo_minibatches": args.minibatches,
                   "grad_backend": ppo.sync.backend, "parallelism": f"env-batch x dp{world}",
                   "l2": "working set > 126 MB L2 (no flush needed)"},
        "clocks": clocks.summary(),
        "e2e": {"value": e2e_ticks / (e2e_ms / 1e3), "unit": "env-ticks/s",
                "h2d_bytes_per_step": host_seed.numel() * 4, "d2h_bytes_per_step": host_stats.numel() * 4},
        "gpu_launches": None,
        "breakdown_ms_per_step": {k: round(v, 3) for k, v in breakdown.items()},
    }


def run_sim(args, rank, world, local):
    import torch
    sys.path.insert(0, HERE)
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    from autodrive_b200.utils.clocks import ClockSampler
    dev = torch.device("cuda", local)
    env = TensorThreeVsThreeEnv(num_envs=args.envs, device=dev, seed=args.seed + rank,
                                fuel_physics=True, horizon=8000, **BENCH_ENV)
    ticks = args.ticks_per_step
    actions = torch.full((args.envs, 6), 7, dtype=torch.int32, device=dev)
    for _ in range(args.warmup):
        env.step_held(actions, ticks)
    with ClockSampler(local) as clocks:
        ms = _timed(lambda: env.step_held(actions, ticks), args.steps, world)
    env_ticks = args.envs * ticks * args.steps * world
    host_actions = torch.full((args.envs, 6), 7, dtype=torch.int32).pin_memory()
    host_rewards = torch.empty((args.envs, 6), dtype=torch.float32).pin_memory()

    def e2e_step():
        _, rew, _ = env.step_held(host_actions.to(dev, non_blocking=True), ticks)
        host_rewards.copy_(rew, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        _ = float(host_rewards.sum())
    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = _timed(e2e_step, args.steps, world)
    return {
        "metric": METRIC, "value": env_ticks / (ms / 1e3), "unit": "env-ticks/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (random-init seeded REBUILT matches, deterministic scripted controllers)",
        "config": {"model": "TensorThreeVsThreeEnv 3v3 full match, fuel physics on (400 FUEL, 64 substeps/tick), "
                            "perception every tick, 0.3 m planner grid 56x27 as in the reference, replan every 20 ticks, "
                            "simulator only",
                   "global_batch": args.envs * world, "envs_per_gpu": args.envs, "seq_len": ticks,
                   "parallelism": f"env-batch x dp{world}", "l2": "working set > 126 MB L2 (no flush needed)"},
        "clocks": clocks.summary(),
        "e2e": {"value": env_ticks / (e2e_ms / 1e3), "unit": "env-ticks/s",
                "h2d_bytes_per_step": host_actions.numel() * 4, "d2h_bytes_per_step": host_rewards.numel() * 4},
        "gpu_launches": (ticks * 4 + 1) * args.steps,
    }


def run_reference(args, rank, world, local):
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "frc_defense")):
        return {"impl": "reference", "unavailable": "baseline/_ref is not installed"}
    sys.path.insert(0, ref)
    import torch
    from frc_defense.tensor_3v3 import TensorThreeVsThreeEnv as RefEnv
    dev = torch.device("cuda", local)
    # The reference's CUDA path builds FUEL contact pairs with per-world Python
    # loops on the host (frc_defense/fuel_physics.py:337-382). Calibrate one
    # tick at a small batch first and refuse configurations that cannot finish.
    calib = min(args.envs, 4)
    modes = ("deterministic",) * 3 + (("nn",) * 3 if args.mode == "train" else ("deterministic",) * 3)
    env = RefEnv(num_envs=calib, device=dev, seed=args.seed + rank, control_modes=modes,
                 robot_roles=("offense",) * 3 + ("defense",) * 3, horizon=8000, randomize=True,
                 fuel_count=BENCH_ENV["fuel_count"], perception_interval=BENCH_ENV["perception_interval"],
                 fused_sensor_rng=True, fuel_physics=True)
    actions = torch.full((calib, 6), 7, dtype=torch.long, device=dev)
    env.step(actions, capture_observation=False, capture_info=False)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    env.step(actions, capture_observation=False, capture_info=False)
    torch.cuda.synchronize()
    per_tick = time.perf_counter() - t0
    ticks_per_step = args.decisions * 12.5 if args.mode == "train" else args.ticks_per_step
    projected = per_tick * args.envs / calib * ticks_per_step * (args.steps + args.warmup)
    if projected > args.reference_budget_s:
        return {"impl": "reference",
                "unavailable": (f"reference 3v3 with fuel physics measured {per_tick:.2f} s per tick at {calib} "
                                f"worlds ({calib / per_tick:.2f} env-ticks/s) on this GPU; {args.envs} worlds x "
                                f"{ticks_per_step * (args.steps + args.warmup):.0f} ticks projects to "
                                f"{projected / 3600:.1f} h"),
                "calibration_env_ticks_per_s": calib / per_tick, "n_gpus": world}
    raise SystemExit("reference configuration fits the budget; extend run_reference before using it")


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--envs", type=int, default=2048)
    p.add_argument("--mode", choices=("train", "sim"), default="train")
    p.add_argument("--decisions", type=int, default=8, help="strategic decisions per PPO rollout (train mode)")
    p.add_argument("--epochs", type=int, default=4)
    p.add_argument("--minibatches", type=int, default=8)
    p.add_argument("--grad-backend", default="auto")
    p.add_argument("--network", default="mlp",
                   help="train mode policy: mlp (strategic_adstar ActorCritic, fused tcgen05 kernels) or a "
                        "perception zoo architecture such as entity_attention_256")
    p.add_argument("--ticks-per-step", type=int, default=20, help="ticks per step (sim mode)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--reference-budget-s", type=float, default=900.)
    args = p.parse_args()
    if args.warmup < 3:
        p.error("at least 3 warm-up steps are required")
    rank, world, local = _dist_init()
    if world != args.gpus:
        p.error(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.impl == "reference":
        result = run_reference(args, rank, world, local)
    else:
        train = run_train if args.network == "mlp" else run_train_zoo
        result = (train if args.mode == "train" else run_sim)(args, rank, world, local)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
