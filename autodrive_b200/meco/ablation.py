"""Paired ablation matrix of MECO scorer tracks (frc_defense/meco_ablation_matrix.py).

For every track x scenario, the full scorer and each ablation
(``meco.train.ABLATIONS``) play the same matched seeds of every category, so
each episode yields a paired outcome (full, ablated). Per cell the matrix
reports both success rates with Wilson intervals, the discordant pairs, the
exact two-sided McNemar test (binomial on the discordant pairs, McNemar 1947)
and the success difference with a Newcombe hybrid-score interval for paired
proportions (Newcombe, Statistics in Medicine 1998, method 10). Records go to
an append-only hash-chained ledger when one is given.

    python -m autodrive_b200.meco.ablation --checkpoint C1=runs/c1/meco.pt \\
        --scenarios pickup_simple pickup_scattered --episodes 8 --output matrix.json
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from ..train.evaluation import wilson_interval
from .train import ABLATIONS, MecoPolicy, MetricLedger, evaluate_meco


def mcnemar_exact(b: int, c: int) -> float:
    """Two-sided exact McNemar p-value for b and c discordant pairs."""
    n = b + c
    if n == 0:
        return 1.
    k = min(b, c)
    tail = sum(math.comb(n, i) for i in range(k + 1)) / 2 ** n
    return min(1., 2. * tail)


def paired_difference_interval(a: int, b: int, c: int, d: int, z: float = 1.96) -> tuple[float, float, float]:
    """Difference p2 - p1 of paired proportions (p1 = success of the first
    arm, p2 of the second) with Newcombe's hybrid-score interval; a = both
    succeed, b = first only, c = second only, d = neither."""
    n = a + b + c + d
    if n == 0:
        return 0., -1., 1.
    p1, p2 = (a + b) / n, (a + c) / n
    l1, u1 = wilson_interval(a + b, n, z)
    l2, u2 = wilson_interval(a + c, n, z)
    denom = math.sqrt(max((a + b) * (c + d) * (a + c) * (b + d), 0))
    num = a * d - b * c
    if num > 0:                       # Newcombe's continuity correction of phi
        num = max(num - n / 2, 0.)
    phi = 0. if denom == 0 else num / denom
    diff = p2 - p1
    dl = math.sqrt(max((p2 - l2) ** 2 - 2 * phi * (p2 - l2) * (u1 - p1) + (u1 - p1) ** 2, 0.))
    du = math.sqrt(max((u2 - p2) ** 2 - 2 * phi * (u2 - p2) * (p1 - l1) + (p1 - l1) ** 2, 0.))
    return diff, max(-1., diff - dl), min(1., diff + du)


def _outcomes(result: dict) -> list[bool]:
    return [v for row in result["categories"] for v in row.get("meco_episodes", [])]


def ablation_matrix(policies: dict[str, MecoPolicy], scenarios, *, episodes: int = 4, ablations=ABLATIONS,
                    split: str = "validation", master_seed: int = 0, device="cpu",
                    ledger: MetricLedger | None = None) -> dict:
    """The full matrix; `policies` maps track ids to scorer policies."""
    if "full" not in ablations:
        ablations = ("full",) + tuple(ablations)
    cells = []
    for track, policy in policies.items():
        for scenario in scenarios:
            runs = {ab: evaluate_meco(policy, scenario, episodes=episodes, split=split, master_seed=master_seed,
                                      device=device, ablation=ab) for ab in ablations}
            full = _outcomes(runs["full"])
            teacher = runs["full"].get("teacher", {})
            for ab in ablations:
                if ab == "full":
                    continue
                arm = _outcomes(runs[ab])
                if len(arm) != len(full):
                    raise RuntimeError("ablation arms did not play the same matched episodes")
                a = sum(f and x for f, x in zip(full, arm))
                b = sum(f and not x for f, x in zip(full, arm))
                c = sum(x and not f for f, x in zip(full, arm))
                d = len(full) - a - b - c
                diff, lo, hi = paired_difference_interval(a, b, c, d)
                cell = {"track": track, "scenario": scenario, "ablation": ab, "episodes": len(full),
                        "full_success": (a + b) / max(1, len(full)),
                        "full_wilson_95": wilson_interval(a + b, len(full)),
                        "ablated_success": (a + c) / max(1, len(full)),
                        "ablated_wilson_95": wilson_interval(a + c, len(full)),
                        "discordant": {"full_only": b, "ablated_only": c},
                        "difference": diff, "difference_95": [lo, hi],
                        "mcnemar_p": mcnemar_exact(b, c),
                        "teacher_success": teacher.get("success_rate")}
                cells.append(cell)
                if ledger is not None:
                    ledger.append("meco_ablation", cell)
    return {"split": split, "master_seed": master_seed, "episodes_per_category": episodes,
            "ablations": [a for a in ablations if a != "full"], "cells": cells}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description="Paired ablation matrix of MECO scorer tracks")
    p.add_argument("--checkpoint", action="append", default=[],
                   help="TRACK=PATH of a trained scorer (meco.pt); repeat per track")
    p.add_argument("--untrained", nargs="*", default=[], help="tracks to include with random weights")
    p.add_argument("--scenarios", nargs="+", default=["pickup_simple"])
    p.add_argument("--ablations", nargs="+", default=list(ABLATIONS))
    p.add_argument("--episodes", type=int, default=4)
    p.add_argument("--split", default="validation")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--device", default="cpu")
    p.add_argument("--output", required=True)
    p.add_argument("--ledger")
    args = p.parse_args(argv)
    policies = {}
    for spec in args.checkpoint:
        track, _, path = spec.partition("=")
        from ..utils.checkpoint import load_verified
        payload = load_verified(path, map_location=args.device, weights_only=False)
        if payload["track"] != track:
            p.error(f"{path} holds track {payload['track']}, not {track}")
        pol = MecoPolicy(track)
        pol.load_state_dict(payload["model_state_dict"])
        policies[track] = pol.to(args.device).eval()
    for track in args.untrained:
        torch.manual_seed(args.seed)
        policies[track] = MecoPolicy(track).to(args.device).eval()
    if not policies:
        p.error("give at least one --checkpoint TRACK=PATH or --untrained TRACK")
    ledger = MetricLedger(args.ledger) if args.ledger else None
    result = ablation_matrix(policies, args.scenarios, episodes=args.episodes, ablations=tuple(args.ablations),
                             split=args.split, master_seed=args.seed, device=args.device, ledger=ledger)
    out = Path(args.output)
    out.parent.mkdir(parents=True, exist_ok=True)
    out.write_text(json.dumps(result, indent=1))
    print(json.dumps({"cells": len(result["cells"]), "output": str(out)}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
