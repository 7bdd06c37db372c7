"""Controlled PPO screening of the policy architecture zoo.

    python -m autodrive_b200.train.architecture_study --architectures deep_sets entity_attention \
        --scenarios pickup defense_3v3 --seeds 7 19 --device cuda:0

Parity with frc_defense/architecture_benchmark.py:26-374: every (architecture,
scenario, seed, learning rate) case trains the network with PPO on
perception-only inputs (``PerceptionInputs``: simulated tracks, own/team
localization, public field map and match state; truth only in rewards and
evaluation records), evaluates on held-fixed worlds every ``--eval-every``
updates, and writes ``metadata.json`` (configuration, parameter count, source
provenance, perception contract) and ``curve.json`` (evaluation curve,
throughput) under ``<output>/<architecture>/<scenario>/seed-<s>-lr-<lr>/``.

Scenarios:
* ``pickup``       one neural offense robot collecting scattered FUEL
                   (curriculum ``pickup_scattered/dense`` worlds); reward =
                   acquisitions;
* ``defense_3v3``  three neural defenders against the scripted offense in a
                   full 3v3 match; reward = blue minus red scoring.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import subprocess
import time
from pathlib import Path

import torch

from ..models.perception import PerceptionInputs
from ..models.zoo import ARCHITECTURES, PerceptionActorCritic, parameter_count
from .rollout import gae_reference

SCENARIOS = {
    "pickup": {"robots": (0,), "reward": "acquisitions per decision"},
    "defense_3v3": {"robots": (3, 4, 5), "reward": "blue score delta minus red score delta"},
}
PERCEPTION_CONTRACT = {
    "version": 2,
    "opponents": "simulated sensor track of the nearest opponent only",
    "fuel": "retained simulated FUEL tracks only",
    "own_and_team": "policy pose estimate, team telemetry and possession",
    "geometry": "public fixed field map",
    "public_match": "clock, HUB activity and score",
    "truth_allowed": "physical dynamics, task rewards and evaluation records",
}


def source_provenance() -> dict:
    root = Path(__file__).resolve().parents[2]
    files = sorted(p for p in (root / "autodrive_b200").rglob("*") if p.suffix in (".py", ".cu", ".h", ".cpp"))
    hashes = {str(p.relative_to(root)): hashlib.sha256(p.read_bytes()).hexdigest() for p in files}
    try:
        commit = subprocess.check_output(["git", "rev-parse", "HEAD"], cwd=root, text=True,
                                         stderr=subprocess.DEVNULL).strip()
    except (OSError, subprocess.CalledProcessError):
        commit = "unknown"
    return {"commit": commit, "source_sha256": hashlib.sha256(json.dumps(hashes, sort_keys=True).encode()).hexdigest(),
            "files": len(hashes)}


class _Case:
    """One scenario's batched worlds plus its perception builder and reward."""

    def __init__(self, scenario: str, n: int, device, seed: int, field_shape):
        if scenario not in SCENARIOS:
            raise ValueError(f"unknown scenario {scenario!r}")
        self.scenario = scenario
        self.ids = SCENARIOS[scenario]["robots"]
        if scenario == "pickup":
            from .curriculum import CurriculumEnv
            self.cenv = CurriculumEnv("pickup_scattered", "dense", n, device, seed=seed)
            self.env = self.cenv.env
        else:
            from ..sim.env3v3 import TensorThreeVsThreeEnv
            self.cenv = None
            self.env = TensorThreeVsThreeEnv(num_envs=n, device=device, seed=seed, fuel_physics=False,
                                             control_modes=("deterministic",) * 3 + ("nn",) * 3)
        self.builder = PerceptionInputs(self.env, self.ids, field_shape=field_shape)
        self.seed = seed

    def reset(self, seed=None):
        if self.cenv is not None:
            self.cenv.reset(seed=self.seed if seed is None else seed)
        else:
            self.env.reset(seed=self.seed if seed is None else seed)
        return self.builder()

    def step(self, actions: torch.Tensor, ticks: int):
        k = len(self.ids)
        if self.cenv is not None:
            _, rew, done = self.cenv.step(actions.reshape(-1), ticks)
            return self.builder(), rew, done
        full = torch.full((self.env.n, 6), 7, dtype=torch.int32, device=self.env.device)
        full[:, list(self.ids)] = actions.reshape(self.env.n, k).to(torch.int32)
        _, rew, trunc = self.env.step_held(full, ticks)
        r = rew[:, list(self.ids)].reshape(-1)
        return self.builder(), r, trunc[:, None].expand(-1, k).reshape(-1)

    def metrics(self) -> dict:
        ws = self.env.ws
        acquired = ws["g_rcount"][:, list(self.ids), 0].sum(-1).float()
        score = ws["g_scores"][:, 2:4].float()
        return {"mean_acquired": float(acquired.mean()), "mean_score_red": float(score[:, 0].mean()),
                "mean_score_blue": float(score[:, 1].mean()),
                "mean_score_difference": float((score[:, 1] - score[:, 0]).mean())}


def _index(d: dict, idx):
    return {k: v[idx] for k, v in d.items()}


def _stack(rows: list) -> dict:
    return {k: torch.stack([r[k] for r in rows]) for k in rows[0]}


def _flatten(d: dict) -> dict:
    return {k: v.reshape(-1, *v.shape[2:]) for k, v in d.items()}


@torch.no_grad()
def evaluate(model, case: _Case, seed: int, ticks: int, repeat: int) -> dict:
    obs = case.reset(seed)
    for _ in range(max(1, ticks // repeat)):
        act, _, _ = model.sample(obs, deterministic=True)
        obs, _, _ = case.step(act, repeat)
    return case.metrics()


def train_case(args, architecture: str, scenario: str, seed: int, lr: float) -> Path:
    torch.manual_seed(seed)
    dev = torch.device(args.device)
    model = PerceptionActorCritic(architecture, tensor_cores=dev.type == "cuda").to(dev)
    opt = torch.optim.Adam(model.parameters(), lr=lr, eps=1e-5)
    out = Path(args.output) / architecture / scenario / f"seed-{seed}-lr-{lr:g}"
    out.mkdir(parents=True, exist_ok=True)
    train = _Case(scenario, args.envs, dev, seed, model.field_shape)
    evalc = _Case(scenario, args.eval_envs, dev, seed + 100000, model.field_shape)
    meta = {"architecture": architecture, "scenario": scenario, "seed": seed, "learning_rate": lr,
            "parameters": parameter_count(model), "config": {k: str(v) for k, v in vars(args).items()},
            "perception_only_dynamic_inputs": True, "perception_contract": PERCEPTION_CONTRACT,
            "provenance": source_provenance(), "reward": SCENARIOS[scenario]["reward"],
            "runtime": {"torch": torch.__version__, "device": str(dev),
                        "device_name": torch.cuda.get_device_name(dev) if dev.type == "cuda" else "CPU",
                        "tensor_cores": dev.type == "cuda"}, "status": "running"}
    (out / "metadata.json").write_text(json.dumps(meta, indent=2))
    curve, t_train, transitions = [], 0., 0
    obs = train.reset()
    for update in range(args.updates + 1):
        if update % args.eval_every == 0 or update == args.updates:
            res = evaluate(model, evalc, seed + 100000, args.eval_ticks, args.action_repeat)
            res.update(update=update, transitions=transitions, train_seconds=round(t_train, 3))
            curve.append(res)
            (out / "curve.json").write_text(json.dumps(curve, indent=2))
        if update == args.updates:
            break
        t0 = time.perf_counter()
        rows, acts, logps, vals, rews, dones = [], [], [], [], [], []
        with torch.no_grad():
            for _ in range(args.rollout_steps):
                act, logp, val = model.sample(obs)
                nobs, rew, done = train.step(act, args.action_repeat)
                rows.append(obs)
                acts.append(act)
                logps.append(logp)
                vals.append(val)
                rews.append(rew.float())
                dones.append(done.bool())
                obs = nobs
                if bool(done.all()):
                    obs = train.reset(seed + update + 1)
            last_v = model(obs)[2]
        T = len(rows)
        val_t = torch.stack(vals)
        next_v = torch.cat((val_t[1:], last_v[None]))
        done_t = torch.stack(dones)
        adv = gae_reference(torch.stack(rews), done_t, torch.zeros_like(done_t), val_t, next_v, args.gamma, .95)
        ret = adv + val_t
        flat = _flatten(_stack(rows))
        a_f, lp_f = torch.stack(acts).reshape(-1), torch.stack(logps).reshape(-1)
        adv_f, ret_f = adv.reshape(-1), ret.reshape(-1)
        n = a_f.numel()
        for _ in range(args.epochs):
            for idx in torch.randperm(n, device=dev).split(args.minibatch_size):
                logp, ent, v, _ = model.score(_index(flat, idx), a_f[idx])
                ratio = (logp - lp_f[idx]).exp()
                a = adv_f[idx]
                a = (a - a.mean()) / (a.std(unbiased=False) + 1e-8)
                pg = torch.maximum(-a * ratio, -a * ratio.clamp(.8, 1.2)).mean()
                loss = pg + .5 * (v - ret_f[idx]).square().mean() - .01 * ent.mean()
                opt.zero_grad(set_to_none=True)
                loss.backward()
                torch.nn.utils.clip_grad_norm_(model.parameters(), .5)
                opt.step()
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        t_train += time.perf_counter() - t0
        transitions += n
    meta.update(status="complete", train_seconds=round(t_train, 3),
                transitions_per_second=round(transitions / max(t_train, 1e-9), 1))
    (out / "metadata.json").write_text(json.dumps(meta, indent=2))
    return out


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--architectures", nargs="+", choices=sorted(ARCHITECTURES), default=sorted(ARCHITECTURES))
    p.add_argument("--scenarios", nargs="+", choices=sorted(SCENARIOS), default=sorted(SCENARIOS))
    p.add_argument("--seeds", nargs="+", type=int, default=[7, 19, 43])
    p.add_argument("--learning-rates", nargs="+", type=float, default=[3e-4])
    p.add_argument("--output", type=Path, default=Path("evaluations/architecture-study"))
    p.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    p.add_argument("--envs", type=int, default=8)
    p.add_argument("--eval-envs", type=int, default=4)
    p.add_argument("--eval-ticks", type=int, default=400)
    p.add_argument("--updates", type=int, default=12)
    p.add_argument("--rollout-steps", type=int, default=40)
    p.add_argument("--action-repeat", type=int, default=10)
    p.add_argument("--epochs", type=int, default=2)
    p.add_argument("--minibatch-size", type=int, default=32)
    p.add_argument("--eval-every", type=int, default=4)
    p.add_argument("--gamma", type=float, default=.993)
    return p


def main(argv=None) -> list[Path]:
    p = build_parser()
    args = p.parse_args(argv)
    for name in ("envs", "eval_envs", "eval_ticks", "rollout_steps", "action_repeat", "epochs",
                 "minibatch_size", "eval_every"):
        if getattr(args, name) < 1:
            p.error(f"--{name.replace('_', '-')} must be positive")
    if args.updates < 0 or not 0 < args.gamma <= 1 or any(lr <= 0 for lr in args.learning_rates):
        p.error("updates must be nonnegative; gamma and learning rates must be positive")
    outs = []
    for arch in args.architectures:
        for sc in args.scenarios:
            for seed in args.seeds:
                for lr in args.learning_rates:
                    outs.append(train_case(args, arch, sc, seed, lr))
    return outs


if __name__ == "__main__":
    main()
