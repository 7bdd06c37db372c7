"""Headline benchmark: 3v3 full-match env-ticks/s on 1..8 B200 (one process per GPU).

Workload (one step): every world of a TensorThreeVsThreeEnv batch (2048 worlds
per GPU, fuel physics on: 504 FUEL, 64 FUEL+robot substeps per 20 ms tick,
perception every 2 ticks, route replanning every 20 ticks, deterministic
scripted controllers for all six robots, seed 0..N per rank) advances one
held decision interval of `--ticks-per-step` ticks (default 20) and builds the
137-feature observations. Synthetic data, random-init state; nothing is
cached or skipped inside the timed region.

Device timing: CUDA events on the launching stream, W warm-up steps, K timed
steps bracketed by barrier + synchronize, max over ranks. The state touched
per step (FUEL, tracks, routes: ~0.25 GB at 2048 worlds) exceeds the 126 MB L2,
so no explicit flush is needed.

End-to-end (`e2e`): the same metric through the public API
(`TensorThreeVsThreeEnv.step_held`) with the step's action tensor copied from
pinned host memory every step and the rewards read back to the host every step.

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


def _dist_init():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        import datetime
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


def run_ours(args, rank, world, local):
    import torch
    sys.path.insert(0, HERE)
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    from autodrive_b200.utils.clocks import ClockSampler
    dev = torch.device("cuda", local)
    env = TensorThreeVsThreeEnv(num_envs=args.envs, device=dev, seed=args.seed + rank,
                                fuel_physics=True, horizon=8000)
    ticks = args.ticks_per_step
    actions = torch.full((args.envs, 6), 7, dtype=torch.int32, device=dev)
    # device-timed region
    for _ in range(args.warmup):
        env.step_held(actions, ticks)
    _barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps):
            env.step_held(actions, ticks)
        stop.record()
        _barrier(world)
    ms = start.elapsed_time(stop)
    ms = _max_over_ranks(ms, world)
    env_ticks = args.envs * ticks * args.steps * world
    value = env_ticks / (ms / 1000.)
    # end-to-end through the public API with H2D inputs and D2H results each step
    host_actions = torch.full((args.envs, 6), 7, dtype=torch.int32).pin_memory()
    host_rewards = torch.empty((args.envs, 6), dtype=torch.float32).pin_memory()
    env.reset(seed=args.seed + rank)
    for _ in range(args.warmup):
        dev_actions = host_actions.to(dev, non_blocking=True)
        _, rew, _ = env.step_held(dev_actions, ticks)
        host_rewards.copy_(rew, non_blocking=True)
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        dev_actions = host_actions.to(dev, non_blocking=True)
        _, rew, _ = env.step_held(dev_actions, ticks)
        host_rewards.copy_(rew, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        _ = float(host_rewards.sum())
    e1.record()
    _barrier(world)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = env_ticks / (e2e_ms / 1000.)
    scores = env.fuel_score_count.sum().item()
    launches_per_step = ticks * 3 + 1
    return {
        "metric": "3v3 env-ticks/sec and PPO samples/sec, 1/2/4/8 B200, device-timed max over ranks",
        "value": value, "unit": "env-ticks/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (random-init seeded REBUILT matches, deterministic scripted controllers)",
        "config": {"model": "TensorThreeVsThreeEnv 3v3 full match, fuel physics on (504 FUEL, "
                            "64 substeps/tick), perception every 2 ticks, replan every 20 ticks",
                   "global_batch": args.envs * world, "envs_per_gpu": args.envs,
                   "seq_len": ticks, "ticks_per_step": ticks, "parallelism": f"env-batch x dp{world}",
                   "l2": "working set > 126 MB L2 (no flush needed)"},
        "clocks": clocks.summary(),
        "e2e": {"value": e2e_value, "unit": "env-ticks/s",
                "h2d_bytes_per_step": host_actions.numel() * 4,
                "d2h_bytes_per_step": host_rewards.numel() * 4},
        "gpu_launches": launches_per_step * args.steps,
        "team_scores_total": scores,
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
    calib_envs = min(args.envs, 4)
    env = RefEnv(num_envs=calib_envs, device=dev, seed=args.seed + rank,
                 control_modes=("deterministic",) * 6, robot_roles=("offense",) * 3 + ("defense",) * 3,
                 horizon=8000, randomize=True, fuel_count=504, fused_sensor_rng=True, fuel_physics=True)
    actions = torch.full((calib_envs, 6), 7, dtype=torch.long, device=dev)
    env.step(actions, capture_observation=False, capture_info=False)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    env.step(actions, capture_observation=False, capture_info=False)
    torch.cuda.synchronize()
    per_tick = time.perf_counter() - t0
    projected = per_tick * args.envs / calib_envs * args.ticks_per_step * (args.steps + args.warmup)
    if projected > args.reference_budget_s:
        value = calib_envs / per_tick
        return {"impl": "reference",
                "unavailable": (f"reference 3v3 with fuel physics measured {per_tick:.2f} s per tick at "
                                f"{calib_envs} worlds ({value:.2f} env-ticks/s) on this GPU; "
                                f"{args.envs} worlds x {args.ticks_per_step * (args.steps + args.warmup)} "
                                f"ticks projects to {projected / 3600:.1f} h"),
                "calibration_env_ticks_per_s": value, "n_gpus": world}
    env = RefEnv(num_envs=args.envs, device=dev, seed=args.seed + rank,
                 control_modes=("deterministic",) * 6, robot_roles=("offense",) * 3 + ("defense",) * 3,
                 horizon=8000, randomize=True, fuel_count=504, fused_sensor_rng=True, fuel_physics=True)
    actions = torch.full((args.envs, 6), 7, dtype=torch.long, device=dev)
    for _ in range(args.warmup * args.ticks_per_step):
        env.step(actions, capture_observation=False, capture_info=False)
    _barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        for t in range(args.ticks_per_step):
            env.step(actions, capture_observation=(t == args.ticks_per_step - 1), capture_info=False)
    stop.record()
    _barrier(world)
    ms = _max_over_ranks(start.elapsed_time(stop), world)
    value = args.envs * args.ticks_per_step * args.steps * world / (ms / 1000.)
    return {"impl": "reference", "metric": "3v3 env-ticks/sec and PPO samples/sec, 1/2/4/8 B200, "
            "device-timed max over ranks", "value": value, "unit": "env-ticks/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "dtype": "fp32", "data": "synthetic",
            "config": {"model": "reference TensorThreeVsThreeEnv", "global_batch": args.envs * world,
                       "seq_len": args.ticks_per_step, "parallelism": f"dp{world}"}}


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--envs", type=int, default=2048)
    p.add_argument("--ticks-per-step", type=int, default=20)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--reference-budget-s", type=float, default=900.)
    args = p.parse_args()
    if args.warmup < 3:
        p.error("at least 3 warm-up steps are required")
    rank, world, local = _dist_init()
    if world != args.gpus:
        p.error(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    result = run_reference(args, rank, world, local) if args.impl == "reference" else run_ours(args, rank, world, local)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
