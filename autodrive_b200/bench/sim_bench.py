"""Simulator micro-benchmarks (per-kernel device time, FUEL microbench).

Examples::

    python -m autodrive_b200.bench.sim_bench stages --envs 2048 --ticks 40
    python -m autodrive_b200.bench.sim_bench fuel --envs 4096 --pieces 400 --ticks 1000

``stages`` times the control / plan / tick / observe kernels of the 3v3
environment separately with CUDA events (eager launches, after warm-up).
``fuel`` is the FUEL-physics microbenchmark: worlds of spheres placed
uniformly over the field with N(0, 1.5 m/s) planar velocities and six robots
driving at up to 4.5 m/s, 10 substeps of 2 ms per tick, all ticks in one
kernel with the state resident in shared memory.
"""
from __future__ import annotations

import argparse
import json
import math

import torch


def _events():
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def stages(args):
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    dev = torch.device("cuda", 0)
    env = TensorThreeVsThreeEnv(num_envs=args.envs, device=dev, seed=args.seed, fuel_physics=not args.static,
                                fuel_count=args.fuel_count, perception_interval=args.perception_interval,
                                planner_resolution=args.planner_resolution)
    if args.threads:
        env.ws.sim.threads = args.threads
    sim = env.ws.sim
    nn_slots = [i for i, m in enumerate(env.control_modes) if m == "nn"]
    gen = torch.Generator(device=dev).manual_seed(args.seed)

    def random_actions():
        # uniformly random valid strategic action for every neural slot (an untrained policy)
        full = torch.full((env.n, 6), 7, dtype=torch.int32, device=dev)
        if nn_slots:
            mask = env.ws["obs"][:, nn_slots, -8:] > .5
            score = torch.rand(mask.shape, device=dev, generator=gen).masked_fill(~mask, -1.)
            full[:, nn_slots] = score.argmax(-1).to(torch.int32)
        return full

    for _ in range(args.warmup):
        env.step_held(random_actions() if args.actions == "random" else None, 20, use_graph=False)
    torch.cuda.synchronize()
    totals = {"control": 0., "plan": 0., "tick": 0., "sense": 0., "observe": 0.}
    sim.sense_in_tick = False   # the sensor stage is timed on its own
    for t in range(args.ticks):
        if args.actions == "random" and t % 12 == 0:
            env._set_actions(random_actions())
        for name, fn in (("control", lambda: sim.control(env._actions_buf)), ("plan", lambda: sim.plan(0)),
                         ("tick", lambda: sim.tick(0, 1)), ("sense", lambda: sim.sense(0))):
            a, b = _events()
            a.record()
            fn()
            b.record()
            b.synchronize()
            totals[name] += a.elapsed_time(b)
        if (t + 1) % 12 == 0:
            a, b = _events()
            a.record()
            sim.observe()
            b.record()
            b.synchronize()
            totals["observe"] += a.elapsed_time(b)
    per_tick = {k: v / args.ticks for k, v in totals.items()}
    total = sum(per_tick.values())
    phases = None
    if args.phases:
        from autodrive_b200.ops import require_extension
        ext = require_extension()
        ext.phase_profile_read()
        ext.sense_profile_read()
        ext.plan_profile_read()
        ext.phase_profile_enable(True)
        for _ in range(args.ticks):
            sim.control(env._actions_buf)
            sim.plan(0)
            sim.tick(0, 1)
            sim.sense(0)
        torch.cuda.synchronize()
        ext.phase_profile_enable(False)
        cyc = ext.phase_profile_read()
        scyc = ext.sense_profile_read()
        pcyc = ext.plan_profile_read()
        pnames = ("occupancy_grid", "endpoint_projection", "move_table_init", "sweeps", "greedy_descent",
                  "line_of_sight", "smoothing_resample", "speed_profile")
        plan_phases = {n: round(c / max(1, sum(pcyc)), 4) for n, c in zip(pnames, pcyc)}
        snames = ("load", "lens_visibility", "lens_geometry_sort", "lens_depth_buffer", "lens_objects",
                  "stereo_fusion", "packing", "association")
        sense_phases = {n: round(c / max(1, sum(scyc)), 4) for n, c in zip(snames, scyc)}
        # robot_* and the join wait of warp 0 are on warp 0's timeline; fuel_integrate..fuel_apply and
        # their join wait on the FUEL warps' timeline (concurrent); the rest on the whole CTA's
        names = ("robot_swerve", "robot_sweep", "robot_contacts", "robot_tail", "fuel_integrate_clear",
                 "fuel_scatter", "fuel_pairs", "fuel_apply", "fuel_chassis_reduce", "fuel_static",
                 "pre_substeps", "post_substeps", "robot_warp_join_wait", "fuel_warps_join_wait",
                 "fuel_count", "fuel_scan", "fuel_chassis_loop", "fuel_pairs_loop")
        robot_line = sum(cyc[k] for k in (0, 1, 2, 3, 12))
        crit = max(1, robot_line + sum(cyc[k] for k in (8, 9, 10, 11, 16)))
        phases = {n: round(c / crit, 4) for n, c in zip(names, cyc)}
    sim.sense_in_tick = True
    awake = (env.ws["f_active"].bool() & (env.ws["f_sleep"] == 0)).float().sum(-1).mean().item()
    sweeps = env.ws["p_sweeps"].float()
    planned = sweeps != 0
    sweep_stats = {"mean": float(sweeps[planned].abs().mean()) if bool(planned.any()) else 0.,
                   "max": float(sweeps.abs().max()), "not_converged": int((sweeps < 0).sum())}
    print(json.dumps({"mode": "stages", "envs": args.envs, "ticks": args.ticks, "actions": args.actions,
                      "awake_fuel_per_world": awake, "planner_sweeps": sweep_stats, "phase_share": phases,
                      "sense_phase_share": sense_phases if args.phases else None,
                      "plan_phase_share": plan_phases if args.phases else None,
                      "ms_per_tick": per_tick, "env_ticks_per_s": args.envs / (total / 1e3),
                      "threads": sim.threads}))


def fuel(args):
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    from autodrive_b200.sim.world import FuelPhysicsConfig
    dev = torch.device("cuda", 0)
    cfg = FuelPhysicsConfig(adaptive_substeps=False, substeps=10, broadphase="grid", contact_mode="fused",
                            solver="jacobi", sleep=True)
    # (0.2 m grid cells: a 0.15 m grid would exceed the 4096-cell shared-memory
    # grid; the broadphase is exact, so the cell size changes speed, not contacts)
    env = TensorThreeVsThreeEnv(num_envs=args.envs, device=dev, seed=args.seed, fuel_physics=cfg,
                                fuel_count=max(args.pieces, 96))
    if args.threads:
        env.ws.sim.threads = args.threads
    ws = env.ws
    g = torch.Generator(device="cpu").manual_seed(args.seed)
    n, P = args.envs, env.fuel_count
    r = cfg.radius
    active = torch.zeros((n, P), dtype=torch.uint8)
    active[:, :args.pieces] = 1
    x = r + torch.rand((n, P), generator=g) * (16.54 - 2 * r)
    y = r + torch.rand((n, P), generator=g) * (8.07 - 2 * r)
    vx = torch.randn((n, P), generator=g) * 1.5
    vy = torch.randn((n, P), generator=g) * 1.5
    ws["f_pos"][:, 0] = x.to(dev)
    ws["f_pos"][:, 1] = y.to(dev)
    ws["f_pos"][:, 2] = env._spawn_height(torch.stack((x, y), -1).to(dev))
    ws["f_vel"].zero_()
    ws["f_vel"][:, 0] = vx.to(dev)
    ws["f_vel"][:, 1] = vy.to(dev)
    ws["f_ang"].zero_()
    ws["f_sleep"].zero_()
    ws["f_active"].copy_(active.to(dev))
    ws["f_owner"].fill_(-1)
    heading = torch.rand((n, 6), generator=g) * 2 * math.pi
    speed = torch.rand((n, 6), generator=g) * 4.5
    cmd = torch.stack((speed * heading.cos(), speed * heading.sin(), torch.zeros_like(speed)), -1)
    ws["c_command"].copy_(cmd.to(dev))
    ws.sim.physics(args.warmup)
    torch.cuda.synchronize()
    a, b = _events()
    a.record()
    ws.sim.physics(args.ticks)
    b.record()
    b.synchronize()
    ms = a.elapsed_time(b)
    print(json.dumps({"mode": "fuel", "envs": n, "pieces": args.pieces, "ticks": args.ticks,
                      "substeps": 10, "ms_per_tick": ms / args.ticks,
                      "env_ticks_per_s": n * args.ticks / (ms / 1e3),
                      "finite": bool(torch.isfinite(ws["f_pos"]).all())}))


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("mode", choices=("stages", "fuel"))
    p.add_argument("--envs", type=int, default=2048)
    p.add_argument("--pieces", type=int, default=400)
    p.add_argument("--ticks", type=int, default=40)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--threads", type=int, default=0)
    p.add_argument("--static", action="store_true")
    p.add_argument("--fuel-count", type=int, default=504, help="stages: FUEL pieces per world")
    p.add_argument("--perception-interval", type=int, default=2, help="stages: ticks between sensor updates")
    p.add_argument("--planner-resolution", type=float, default=.3, help="stages: planner grid cell (m)")
    p.add_argument("--phases", action="store_true", help="stages: also report the tick kernel's per-phase cycle shares")
    p.add_argument("--actions", choices=("held", "random"), default="held",
                   help="stages: default held actions, or random valid strategic actions every 12 ticks")
    args = p.parse_args()
    (stages if args.mode == "stages" else fuel)(args)


if __name__ == "__main__":
    main()
