"""Seeded 3v3 match-outcome statistics for either simulator.

Runs batches of full REBUILT matches with all six robots under their
deterministic controllers (robots 0-2 offense, 3-5 defense role), the
configuration of the reference's offense batch evaluator
(scripts/evaluate_3v3_offense_batch.py:190-230 in the reference: 504 FUEL,
randomized drivetrains, fuel physics on, replanning every 20 ticks,
perception every 2nd tick, action 7 for every robot), and records every
world's alliance scores and per-robot FUEL acquisitions at fixed checkpoints.

    python -m autodrive_b200.bench.match_outcomes run --impl ours --seeds 827104 827105 191873 \
        --envs 12 --ticks 8000 --output outcomes.json
    python -m autodrive_b200.bench.match_outcomes run --impl reference --device cpu --seeds 827104 \
        --envs 4 --ticks 8000 --output ref.json
    python -m autodrive_b200.bench.match_outcomes summarize outcomes.json ref.json
    python -m autodrive_b200.bench.match_outcomes compare --ours outcomes.json --reference ref*.json

`--impl reference` imports the unmodified reference package installed in
``baseline/_ref`` and drives it through its public ``TensorThreeVsThreeEnv``
API exactly as its evaluator does. `summarize` prints per-checkpoint means
and 95 % confidence intervals (Student t over worlds) for one or more files.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _make_env(impl: str, envs: int, device, seed: int, ticks: int, fuel_count: int,
              perception_interval: int, planner_resolution: float):
    kw = dict(num_envs=envs, device=device, seed=seed, control_modes=("deterministic",) * 6,
              robot_roles=("offense",) * 3 + ("defense",) * 3, horizon=ticks, dt=.02, randomize=True,
              fuel_count=fuel_count, fuel_physics=True, replan_interval=20,
              perception_interval=perception_interval)
    if impl == "reference":
        ref = os.path.join(REPO, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref, "frc_defense")):
            raise SystemExit("baseline/_ref is not installed")
        sys.path.insert(0, ref)
        from frc_defense.tensor_3v3 import TensorThreeVsThreeEnv
        return TensorThreeVsThreeEnv(fused_sensor_rng=True, **kw)
    sys.path.insert(0, REPO)
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    return TensorThreeVsThreeEnv(planner_resolution=planner_resolution, **kw)


def run(args) -> dict:
    import torch
    if args.threads:
        torch.set_num_threads(args.threads)
    device = torch.device(args.device)
    out = {"impl": args.impl, "device": str(device), "envs": args.envs, "ticks": args.ticks,
           "fuel_count": args.fuel_count, "perception_interval": args.perception_interval,
           "planner_resolution": args.planner_resolution if args.impl == "ours" else .3,
           "checkpoint_every": args.every, "seeds": {}}
    for seed in args.seeds:
        env = _make_env(args.impl, args.envs, device, seed, args.ticks, args.fuel_count,
                        args.perception_interval, args.planner_resolution)
        env.reset(seed=seed)
        actions = torch.full((args.envs, 6), 7, device=device, dtype=torch.long)
        record = {"checkpoints": []}
        started = time.perf_counter()
        for tick in range(1, args.ticks + 1):
            env.step(actions, capture_observation=False, capture_info=False)
            if tick % args.every == 0 or tick == args.ticks:
                record["checkpoints"].append({
                    "tick": tick,
                    "score_by_team": env.fuel_score_count.detach().cpu().tolist(),
                    "acquisitions_by_robot": env.fuel_acquisition_count.detach().cpu().tolist(),
                    "elapsed_s": time.perf_counter() - started})
                out["seeds"][str(seed)] = record
                if args.output:
                    tmp = args.output + ".tmp"
                    with open(tmp, "w") as f:
                        json.dump(out, f)
                    os.replace(tmp, args.output)
        del env
    return out


def _mean_ci(values):
    n = len(values)
    if n == 0:
        return None
    mean = sum(values) / n
    if n < 2:
        return {"n": n, "mean": mean, "ci95": None}
    var = sum((v - mean) ** 2 for v in values) / (n - 1)
    # two-sided 97.5 % Student t quantiles for small samples, normal beyond 30
    t_table = {1: 12.706, 2: 4.303, 3: 3.182, 4: 2.776, 5: 2.571, 6: 2.447, 7: 2.365, 8: 2.306, 9: 2.262,
               10: 2.228, 11: 2.201, 12: 2.179, 13: 2.160, 14: 2.145, 15: 2.131, 20: 2.086, 25: 2.060,
               30: 2.042}
    dof = n - 1
    t = t_table.get(dof) or (1.96 if dof > 30 else t_table[max(k for k in t_table if k <= dof)])
    half = t * math.sqrt(var / n)
    return {"n": n, "mean": mean, "ci95": [mean - half, mean + half], "std": math.sqrt(var)}


def summarize(paths, tick=None) -> dict:
    """Per-world red-alliance score and per-robot acquisitions pooled over
    every seed of every file, at checkpoint `tick` (default: the last tick
    that every seed reached)."""
    result = {}
    for path in paths:
        with open(path) as f:
            run_ = json.load(f)
        seeds = run_["seeds"]
        reached = min(r["checkpoints"][-1]["tick"] for r in seeds.values()) if seeds else 0
        at = tick or reached
        score, acq = [], [[] for _ in range(6)]
        for r in seeds.values():
            cp = next((c for c in r["checkpoints"] if c["tick"] == at), None)
            if cp is None:
                continue
            for world_score, world_acq in zip(cp["score_by_team"], cp["acquisitions_by_robot"]):
                score.append(world_score[0])
                for k in range(6):
                    acq[k].append(world_acq[k])
        result[f"{run_['impl']}:{os.path.basename(path)}"] = {
            "tick": at, "red_score_per_world": _mean_ci(score),
            "acquisitions_per_robot": [_mean_ci(a) for a in acq[:3]]}
    return result


def _t975(dof: float) -> float:
    table = {1: 12.706, 2: 4.303, 3: 3.182, 4: 2.776, 5: 2.571, 6: 2.447, 7: 2.365, 8: 2.306, 9: 2.262,
             10: 2.228, 11: 2.201, 12: 2.179, 13: 2.160, 14: 2.145, 15: 2.131, 20: 2.086, 25: 2.060, 30: 2.042}
    if dof > 30:
        return 1.96
    return table[max(k for k in table if k <= max(1, int(dof)))]


def _pooled(paths, tick):
    """Per-world red scores and per-robot acquisitions of all seeds of `paths` at `tick`."""
    score, acq = [], [[] for _ in range(3)]
    for path in paths:
        with open(path) as f:
            for r in json.load(f)["seeds"].values():
                cp = next((c for c in r["checkpoints"] if c["tick"] == tick), None)
                if cp is None:
                    continue
                for world_score, world_acq in zip(cp["score_by_team"], cp["acquisitions_by_robot"]):
                    score.append(world_score[0])
                    for k in range(3):
                        acq[k].append(world_acq[k])
    return score, acq


def _welch(a, b) -> dict:
    """Difference of means a - b with a Welch 95 % interval (Welch-Satterthwaite dof)."""
    na, nb = len(a), len(b)
    ma, mb = sum(a) / na, sum(b) / nb
    va = sum((x - ma) ** 2 for x in a) / max(1, na - 1)
    vb = sum((x - mb) ** 2 for x in b) / max(1, nb - 1)
    se2 = va / na + vb / nb
    if se2 == 0:
        return {"difference": ma - mb, "ci95": [ma - mb, ma - mb], "dof": None}
    dof = se2 ** 2 / ((va / na) ** 2 / max(1, na - 1) + (vb / nb) ** 2 / max(1, nb - 1) + 1e-300)
    half = _t975(dof) * math.sqrt(se2)
    return {"difference": ma - mb, "ci95": [ma - mb - half, ma - mb + half], "dof": dof}


def compare(ours, reference, tick=None) -> dict:
    """Our simulator's outcome files against the reference's at one checkpoint
    tick (default: the last tick every seed of both sides reached): pooled
    means with 95 % intervals and the Welch difference of means for the red
    score per world and each offense robot's acquisitions."""
    def reached(paths):
        ticks = []
        for path in paths:
            with open(path) as f:
                ticks += [r["checkpoints"][-1]["tick"] for r in json.load(f)["seeds"].values() if r["checkpoints"]]
        return min(ticks) if ticks else 0
    at = tick or min(reached(ours), reached(reference))
    (so, ao), (sr, ar) = _pooled(ours, at), _pooled(reference, at)
    if not so or not sr:
        raise ValueError(f"no worlds reached tick {at} on both sides")
    return {"tick": at,
            "red_score_per_world": {"ours": _mean_ci(so), "reference": _mean_ci(sr), "ours_minus_reference": _welch(so, sr)},
            "acquisitions_per_robot": [{"ours": _mean_ci(ao[k]), "reference": _mean_ci(ar[k]),
                                        "ours_minus_reference": _welch(ao[k], ar[k])} for k in range(3)]}


def main():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = p.add_subparsers(dest="cmd")
    r = sub.add_parser("run")
    r.add_argument("--impl", choices=("ours", "reference"), default="ours")
    r.add_argument("--device", default="cuda:0")
    r.add_argument("--seeds", type=int, nargs="+", default=[64821])
    r.add_argument("--envs", type=int, default=12)
    r.add_argument("--ticks", type=int, default=8000)
    r.add_argument("--every", type=int, default=500)
    r.add_argument("--fuel-count", type=int, default=504)
    r.add_argument("--perception-interval", type=int, default=2)
    r.add_argument("--planner-resolution", type=float, default=.3)
    r.add_argument("--threads", type=int, default=0)
    r.add_argument("--output")
    s = sub.add_parser("summarize")
    s.add_argument("files", nargs="+")
    s.add_argument("--tick", type=int)
    c = sub.add_parser("compare")
    c.add_argument("--ours", nargs="+", required=True)
    c.add_argument("--reference", nargs="+", required=True)
    c.add_argument("--tick", type=int)
    args = p.parse_args()
    if args.cmd == "summarize":
        print(json.dumps(summarize(args.files, args.tick), indent=1))
    elif args.cmd == "compare":
        print(json.dumps(compare(args.ours, args.reference, args.tick), indent=1))
    else:
        if args.cmd is None:
            p.error("choose run or summarize")
        print(json.dumps(run(args))[:2000])


if __name__ == "__main__":
    main()
