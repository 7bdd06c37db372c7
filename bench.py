"""Headline benchmark: 3v3 env-ticks/s and PPO samples/s on 1..8 B200 (one process per GPU).

Default workload (`--mode train`), one step = one PPO training iteration of
the 3v3 defense configuration on every GPU:
  * TensorThreeVsThreeEnv, 2048 worlds per GPU, fuel physics on (400 FUEL,
    64 robot+FUEL substeps per 20 ms tick), stereo perception and the
    137-feature strategic observations built every tick, route replanning
    every 20 ticks on a 0.1 m occupancy grid (166 x 81 cells), three scripted
    offense robots and three learned defenders sharing one 137->8
    ActorCritic (random init; fp32 master weights, bf16 tensor-core matmul
    operands with fp32 accumulation);
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
through its own public API on the same configuration: it first times two
ticks of the reference's TensorThreeVsThreeEnv at a few worlds on this GPU,
and when the full configuration projects past `--reference-budget-s` it
prints an `unavailable` line carrying that calibration instead of a value.
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
# observations every tick, routes planned on a 0.1 m occupancy grid
# (166 x 81 cells). The reference's 3v3 environment plans on a fixed 0.3 m
# grid (it has no resolution keyword) and defaults to 504 FUEL with
# perception every 2nd tick.
BENCH_ENV = {"fuel_count": 400, "perception_interval": 1, "planner_resolution": .1}
OBSERVE_EVERY_TICK = True
BENCH_DESC = ("TensorThreeVsThreeEnv 3v3 full match (fuel physics on, 400 FUEL, 64 substeps/tick, perception "
              "and strategic observations every tick, AD*-style replanning every 20 ticks on a 0.1 m grid "
              "166x81)")
DTYPES = {"simulator": "fp32", "policy_matmul": "bf16 operands, fp32 accumulate (tcgen05)",
          "master_weights_and_optimizer": "fp32"}


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
    from autodrive_b200.train.ppo import PPOConfig, PPOLearner, collect_rollout, flatten_rollout, make_env
    from autodrive_b200.train.rollout import StrategicClock, gae_advantages
    from autodrive_b200.utils import launches
    from autodrive_b200.utils.clocks import ClockSampler
    dev = torch.device("cuda", local)
    agents = make_env("3v3", args.envs, dev, args.seed + rank * 1_000_003, "offense", 8000, fuel_physics=True,
                      observe_every_tick=OBSERVE_EVERY_TICK, **BENCH_ENV)
    samples = agents.n_agents * args.decisions
    cfg = PPOConfig(rollout_steps=args.decisions, epochs=args.epochs,
                    minibatch_size=samples // args.minibatches, grad_backend=args.grad_backend)
    learner = PPOLearner(agents.obs_dim, agents.action_dim, "categorical", dev, cfg, args.network, world)
    if learner.perception:
        agents.use_perception(learner.model.field_shape, learner.model.input_keys)
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
        flat = flatten_rollout(buf, adv, agents.obs_dim, agents.action_dim, "categorical")
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
    launches_before = launches.read()
    phases["on"] = True
    with ClockSampler(local) as clocks:
        ms = _timed(step, args.steps, world)
    phases["on"] = False
    wrapper_launches = launches.read() - launches_before
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
    profile = _profile_step(step, args.profile) if args.profile else None
    decisions_ticks = ticks_timed / max(1, args.steps)
    minibatches = args.epochs * args.minibatches
    # own kernels per step: control+plan+tick+sense+observe per tick (C++ launches); on the fused
    # MLP path the policy act per decision, the bootstrap value and per minibatch adv stats, fused
    # fwd+bwd, partial reduce and weight pack; plus the kernels the Python wrappers count (GAE,
    # GEMMs, LayerNorm, Adam, peer all-reduce)
    per_tick = 5 if OBSERVE_EVERY_TICK else 4
    sim_launches = decisions_ticks * per_tick + (0 if OBSERVE_EVERY_TICK else args.decisions)
    tc_launches = (args.decisions + 1 + 4 * minibatches) if learner.tc is not None else 0
    gpu_launches = int(args.steps * (sim_launches + tc_launches) + wrapper_launches)
    return {
        "metric": METRIC, "value": value, "unit": "env-ticks/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16" if (learner.tc is not None or learner.cfg.bf16) else "fp32",
        "dtypes": DTYPES,
        "data": "synthetic (random-init seeded REBUILT matches and policy; no external data)",
        "ppo_samples_per_s": samples_total / (ms / 1e3), "ppo_samples_per_step_per_gpu": samples,
        "config": {"model": BENCH_DESC + (" + PPO on the strategic_adstar ActorCritic 137->128->128->8 for 3 "
                                          "learned defenders" if args.network == "mlp" else
                                          f" + PPO on {args.network} ({sum(p.numel() for p in learner.model.parameters())}"
                                          " parameters, bf16 autocast, fp32 master) for 3 learned defenders"),
                   "network": args.network,
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
        "gpu_launches": gpu_launches,
        "breakdown_ms_per_step": breakdown,
        "policy_kernels": ("tcgen05 fused MLP kernels" if learner.tc is not None else
                           "tcgen05 GEMM + fused LayerNorm kernels with torch attention/elementwise"),
        "final_stats": {"mean_reward": float(stats_dev[0]), "approx_kl": float(stats_dev[1]),
                        "entropy": float(stats_dev[2]), "grad_norm": float(stats_dev[3])},
        **({"profile": profile} if profile else {}),
    }


def _profile_step(step, path: str) -> dict:
    """One extra (untimed) step under torch.profiler: device time per kernel
    name, written to `path` as JSON (top 40) and summarised in the result."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    rows = []
    for e in prof.key_averages():
        dev = getattr(e, "device_time_total", None)
        if dev is None:
            dev = getattr(e, "cuda_time_total", 0.)
        if dev > 0:
            rows.append({"name": e.key[:160], "device_ms": dev / 1e3, "calls": e.count})
    rows.sort(key=lambda r: -r["device_ms"])
    total = sum(r["device_ms"] for r in rows)
    for r in rows:
        r["share"] = r["device_ms"] / max(total, 1e-9)
    with open(path, "w") as f:
        json.dump({"device_ms_total": total, "kernels": rows[:40]}, f, indent=1)
    return {"device_ms_total": round(total, 3), "top": [(r["name"][:60], round(r["share"], 4)) for r in rows[:8]],
            "file": path}


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
    held = dict(observe_every_tick=OBSERVE_EVERY_TICK)
    for _ in range(args.warmup):
        env.step_held(actions, ticks, **held)
    with ClockSampler(local) as clocks:
        ms = _timed(lambda: env.step_held(actions, ticks, **held), args.steps, world)
    env_ticks = args.envs * ticks * args.steps * world
    host_actions = torch.full((args.envs, 6), 7, dtype=torch.int32).pin_memory()
    host_rewards = torch.empty((args.envs, 6), dtype=torch.float32).pin_memory()

    def e2e_step():
        _, rew, _ = env.step_held(host_actions.to(dev, non_blocking=True), ticks, **held)
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
        "config": {"model": BENCH_DESC + ", simulator only",
                   "global_batch": args.envs * world, "envs_per_gpu": args.envs, "seq_len": ticks,
                   "parallelism": f"env-batch x dp{world}", "l2": "working set > 126 MB L2 (no flush needed)"},
        "clocks": clocks.summary(),
        "e2e": {"value": env_ticks / (e2e_ms / 1e3), "unit": "env-ticks/s",
                "h2d_bytes_per_step": host_actions.numel() * 4, "d2h_bytes_per_step": host_rewards.numel() * 4},
        "gpu_launches": (ticks * (5 if OBSERVE_EVERY_TICK else 4) + (0 if OBSERVE_EVERY_TICK else 1)) * args.steps,
    }


def run_reference(args, rank, world, local):
    """The unmodified reference (baseline/_ref) through its public API.

    Calibration: the reference's TensorThreeVsThreeEnv on this GPU at a few
    worlds with the benchmark world's settings (400 FUEL, perception every
    tick, observations every tick, fuel physics on), one warm-up tick and two
    timed ticks. Its CUDA path builds FUEL contact pairs with per-world
    Python loops on the host (frc_defense/fuel_physics.py:337-382), so the
    full configuration is projected first; when it fits the budget the
    reference's own loop runs and is timed (`--mode sim`: env.step ticks as in
    scripts/benchmark_3v3_full_match.py:15-58; `--mode train`: one
    train_3v3_generation call of `--decisions` rollout steps per step,
    frc_defense/tensor_training.py:137-157).
    """
    ref = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "frc_defense")):
        return {"impl": "reference", "unavailable": "baseline/_ref is not installed"}
    sys.path.insert(0, ref)
    import torch
    from frc_defense.tensor_3v3 import TensorThreeVsThreeEnv as RefEnv
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    calib = min(args.envs, 4)
    modes = ("deterministic",) * 3 + (("nn",) * 3 if args.mode == "train" else ("deterministic",) * 3)
    env_kw = dict(robot_roles=("offense",) * 3 + ("defense",) * 3, horizon=8000, randomize=True,
                  fuel_count=BENCH_ENV["fuel_count"], perception_interval=BENCH_ENV["perception_interval"],
                  fused_sensor_rng=True, fuel_physics=True)
    env = RefEnv(num_envs=calib, device=dev, seed=args.seed + rank, control_modes=modes, **env_kw)
    env.reset(seed=args.seed + rank)
    actions = torch.full((calib, 6), 7, dtype=torch.long, device=dev)
    env.step(actions, capture_observation=OBSERVE_EVERY_TICK, capture_info=False)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(2):
        env.step(actions, capture_observation=OBSERVE_EVERY_TICK, capture_info=False)
    stop.record()
    torch.cuda.synchronize()
    per_tick = _max_over_ranks(start.elapsed_time(stop) / 2e3, world)
    del env
    ticks_per_step = args.decisions * 12.5 if args.mode == "train" else args.ticks_per_step
    projected = per_tick * args.envs / calib * ticks_per_step * (args.steps + args.warmup)
    calibration = {"envs": calib, "ticks": 2, "seconds_per_tick": per_tick,
                   "env_ticks_per_s": calib / per_tick, "device_timed": True,
                   "settings": "400 FUEL, perception and observations every tick, fuel physics on, reference "
                               "planner grid 0.3 m (no resolution keyword)"}
    if projected > args.reference_budget_s:
        return {"impl": "reference", "n_gpus": world,
                "unavailable": (f"reference 3v3 (fuel physics on) measured {per_tick:.2f} s per tick at {calib} "
                                f"worlds ({calib / per_tick:.2f} env-ticks/s) on this GPU; {args.envs} worlds x "
                                f"{ticks_per_step * (args.steps + args.warmup):.0f} ticks projects to "
                                f"{projected / 3600:.1f} h, over the {args.reference_budget_s:.0f} s budget"),
                "calibration": calibration, "calibration_env_ticks_per_s": calib / per_tick}
    if args.mode == "sim":
        env = RefEnv(num_envs=args.envs, device=dev, seed=args.seed + rank, control_modes=modes, **env_kw)
        env.reset(seed=args.seed + rank)
        actions = torch.full((args.envs, 6), 7, dtype=torch.long, device=dev)

        def step():
            for _ in range(args.ticks_per_step):
                env.step(actions, capture_observation=OBSERVE_EVERY_TICK, capture_info=False)
        work = args.envs * args.ticks_per_step
    else:
        import tempfile
        from frc_defense.tensor_training import train_3v3_generation
        out_dir = tempfile.mkdtemp(prefix="ref_bench_")
        counter = [0]
        samples = args.envs * 3 * args.decisions

        def step():
            counter[0] += 1
            train_3v3_generation("defense", counter[0], out_dir, seed=args.seed, num_envs=args.envs * world,
                                 device=str(dev), rollout_steps=args.decisions, epochs=args.epochs,
                                 minibatch_size=max(world, samples * world // args.minibatches))
        work = args.envs * args.decisions * 12.5
    for _ in range(args.warmup):
        step()
    ms = _timed(step, args.steps, world)
    value = work * args.steps * world / (ms / 1e3)
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": "env-ticks/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (reference package, random init)", "calibration": calibration,
            "config": {"model": "reference TensorThreeVsThreeEnv (400 FUEL, perception every tick, fuel physics on)",
                       "global_batch": args.envs * world, "envs_per_gpu": args.envs, "mode": args.mode,
                       "parallelism": f"env-batch x dp{world}"}}


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
    p.add_argument("--profile", help="train mode: also run one step under torch.profiler and write the device "
                                     "time per kernel to this JSON file")
    args = p.parse_args()
    if args.warmup < 3:
        p.error("at least 3 warm-up steps are required")
    rank, world, local = _dist_init()
    if world != args.gpus:
        p.error(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if args.impl == "reference":
        result = run_reference(args, rank, world, local)
    else:
        result = (run_train if args.mode == "train" else run_sim)(args, rank, world, local)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
