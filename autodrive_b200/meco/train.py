"""MECO track training and evaluation on the offense curriculum.

Parity with frc_defense/meco_track_training.py (``train_meco`` :2441,
``evaluate_meco`` :3452, ``_parser`` :5671), meco_supervised.py (teacher
warm start), meco_counterfactual.py (branch-rollout labels) and
meco_metric_ledger.py (append-only provenance ledger):

* ``MecoPolicy``        wraps one scorer track (A1/A2/A3/C1/C2) with a value
                         head; every strategic action of the learned robot
                         (slot 0 of a ``CurriculumEnv``) is a candidate. Candidate
                         tracks (C1/C2) score the candidate table directly; dense
                         tracks (A1 raster, A2/A3 SE(2) lattice) are read at each
                         candidate's goal cell and approach heading. Logits are
                         utility - penalty over the valid candidates.
* ``train_meco``        recurrent PPO (GRU context carried through the episode,
                         stored per decision for the update), optional teacher
                         warm start.
* ``supervised_warm_start``  cross-entropy towards a scripted teacher's choices.
* ``counterfactual_labels``  for every row, each candidate is executed for one
                         decision in a cloned world and the teacher continues
                         for the horizon; the label is the best candidate by
                         curriculum progress.
* ``evaluate_meco``     matched-seed evaluation against the scripted teacher,
                         decisions routed through the fail-closed arbiter
                         (``choose_candidate``); success rates with Wilson
                         intervals and arbiter fallback counts.
* ``MetricLedger``      JSON-lines ledger, each record chained to the previous
                         by SHA-256.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import math
import time
from dataclasses import asdict, dataclass
from pathlib import Path

import torch
from torch import nn
from torch.nn import functional as F

from ..train.curriculum import (SCENARIOS, CurriculumEnv, D2PredictivePolicy, episode_success, get_scenario,
                                seed_partition, wilson_interval)
from .inputs import CELL, build_globals, build_raster, safe_action_candidates, se2_lattice
from .tracks import HIDDEN, DecisionRequest, ScorerOutput, candidate_policy_logits, choose_candidate, make_meco_track

SLOT = 0          # the learned robot of the offense curriculum
ACTIONS = 8


# --------------------------------------------------------------------------- policy
def candidate_goals(env, slot: int = SLOT) -> torch.Tensor:
    """Goal point [n, 8, 2] of every strategic action: the four FUEL candidates,
    the own HUB, the tracked opponent, the mid-field ferry lane, staying put."""
    ws = env.ws
    pose = ws["policy_pose"][:, slot, :2]
    n = env.n
    goals = pose[:, None, :].repeat(1, ACTIONS, 1)
    cand = ws["c_cand"][:, slot].long()                                  # [n, 4], -1 = none
    tpos = ws["t_pos"][:, slot].transpose(1, 2)                          # [n, P, 2]
    fuel = tpos.gather(1, cand.clamp_min(0)[..., None].expand(-1, -1, 2))
    goals[:, :4] = torch.where((cand >= 0)[..., None], fuel, goals[:, :4])
    team = int(env.team_ids[slot])
    goals[:, 4] = env.hub_centers[team]
    opp_ok = ws["o_valid"][:, slot].bool()
    goals[:, 5] = torch.where(opp_ok[:, None], ws["o_pose"][:, slot, :2], pose)
    lane_x = env.field_length * .5 + (-.45 if team == 0 else .45)
    goals[:, 6, 0] = lane_x
    return torch.nan_to_num(goals)


def _heading_bins(env, goals, slot: int = SLOT) -> torch.Tensor:
    pose = env.ws["policy_pose"][:, slot, :2]
    d = goals - pose[:, None]
    ang = torch.atan2(d[..., 1], d[..., 0])
    return torch.remainder(torch.round(ang / (2 * math.pi / 8)).long(), 8)


class MecoPolicy(nn.Module):
    """One MECO scorer track as a candidate policy with a value head."""

    def __init__(self, track: str):
        super().__init__()
        self.track_id = track
        self.track = make_meco_track(track)
        self.value_head = nn.Linear(HIDDEN, 1)

    def forward(self, env, hidden=None, slot: int = SLOT):
        """(utility [n, 8], penalty [n, 8], valid [n, 8], value [n], hidden)."""
        raster = build_raster(env, slot)
        glob = build_globals(env, slot)
        _, valid, feats = safe_action_candidates(env, slot)
        if self.track_id == "C1":
            out = self.track(globals_=glob, candidate_features=feats, hidden=hidden)
            util, pen = out["utility"], out["penalty"]
        elif self.track_id == "C2":
            out = self.track(raster=raster, globals_=glob, candidate_features=feats, hidden=hidden)
            util, pen = out["utility"], out["penalty"]
        else:
            goals = candidate_goals(env, slot)
            hb = _heading_bins(env, goals, slot)
            h, w = raster.shape[-2:]
            if self.track_id == "A1":
                out = self.track(raster=raster, globals_=glob, hidden=hidden)
                cx = (goals[..., 0] / CELL).floor().long().clamp(0, w - 1)
                cy = (goals[..., 1] / CELL).floor().long().clamp(0, h - 1)
                flat_u = out["utility"].reshape(env.n, -1)               # [n, 8 * h * w]
                flat_p = out["penalty"].reshape(env.n, -1)
                idx = (hb * h + cy) * w + cx
            else:
                stride = 4
                lat = se2_lattice(raster, stride=stride)
                out = self.track(**lat, globals_=glob, hidden=hidden)
                cw, ch = math.ceil(w / stride), math.ceil(h / stride)
                cx = (goals[..., 0] / (CELL * stride)).floor().long().clamp(0, cw - 1)
                cy = (goals[..., 1] / (CELL * stride)).floor().long().clamp(0, ch - 1)
                flat_u, flat_p = out["utility"], out["penalty"]
                idx = (cy * cw + cx) * 8 + hb
            util, pen = flat_u.gather(1, idx), flat_p.gather(1, idx)
        hid = out["hidden"]
        return util, pen, valid, self.value_head(hid).squeeze(-1), hid

    def distribution(self, env, hidden=None):
        util, pen, valid, value, hid = self(env, hidden)
        logits = candidate_policy_logits(util, valid, pen)
        return torch.distributions.Categorical(logits=logits), value, hid, util, pen, valid


# --------------------------------------------------------------------------- config
@dataclass
class MecoConfig:
    track: str = "C1"
    scenario: str = "pickup_simple"
    envs: int = 32
    updates: int = 10
    epochs: int = 2
    learning_rate: float = 3e-4
    clip: float = .2
    gamma: float = .99
    lam: float = .95
    entropy: float = .01
    warm_start_decisions: int = 0
    seed: int = 0
    device: str = "cpu"
    output: str = ""

    def identity(self) -> str:
        return hashlib.sha256(json.dumps(asdict(self), sort_keys=True).encode()).hexdigest()[:16]


# --------------------------------------------------------------------------- ledger
class MetricLedger:
    """Append-only JSON-lines ledger; record k stores the SHA-256 of record k-1,
    so any edit or deletion breaks ``verify()``."""

    def __init__(self, path):
        self.path = Path(path)

    def _last_hash(self) -> str:
        if not self.path.exists():
            return "0" * 64
        last = "0" * 64
        for line in self.path.read_text().splitlines():
            if line.strip():
                last = json.loads(line)["sha256"]
        return last

    def append(self, kind: str, payload: dict) -> dict:
        body = {"kind": kind, "time": time.time(), "prev": self._last_hash(), "payload": payload}
        canon = json.dumps(body, sort_keys=True, allow_nan=False)
        rec = {**body, "sha256": hashlib.sha256(canon.encode()).hexdigest()}
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with self.path.open("a") as fh:
            fh.write(json.dumps(rec, sort_keys=True) + "\n")
        return rec

    def records(self) -> list[dict]:
        if not self.path.exists():
            return []
        return [json.loads(line) for line in self.path.read_text().splitlines() if line.strip()]

    def verify(self) -> bool:
        prev = "0" * 64
        for rec in self.records():
            body = {k: rec[k] for k in ("kind", "time", "prev", "payload")}
            canon = json.dumps(body, sort_keys=True, allow_nan=False)
            if rec["prev"] != prev or hashlib.sha256(canon.encode()).hexdigest() != rec["sha256"]:
                return False
            prev = rec["sha256"]
        return True


# --------------------------------------------------------------------------- teacher / labels
def supervised_warm_start(policy: MecoPolicy, cenv: CurriculumEnv, optimizer, decisions: int,
                          teacher=None) -> float:
    """Imitate the teacher's valid choices for `decisions` steps; returns the mean loss."""
    teacher = teacher or D2PredictivePolicy()
    cenv.reset()
    hidden, losses = None, []
    for _ in range(decisions):
        act = teacher.choose(cenv)
        dist, _, hidden, _, _, valid = policy.distribution(cenv.env, hidden)
        ok = valid.gather(1, act[:, None]).squeeze(1)
        if bool(ok.any()):
            loss = F.cross_entropy(dist.logits[ok], act[ok])
            optimizer.zero_grad()
            loss.backward()
            optimizer.step()
            losses.append(loss.item())
        hidden = hidden.detach()
        _, _, done = cenv.step(act)
        if bool(done.all()):
            cenv.reset()
            hidden = None
    return sum(losses) / max(1, len(losses))


def _clone_rows(src: CurriculumEnv, dst: CurriculumEnv, copies: int) -> None:
    """World state of every row of `src` repeated `copies` times into `dst`."""
    state = src.env.ws.state_dict()
    for name, tensor in state.items():
        if name == "raster_pts":
            continue
        dst.env.ws[name].copy_(tensor.repeat_interleave(copies, dim=0))
    dst.elapsed = src.elapsed
    dst.metrics.snapshot()


def counterfactual_labels(cenv: CurriculumEnv, horizon: int = 4, teacher=None, branch_env: CurriculumEnv | None = None):
    """(best action [n], value [n, 8]): each candidate is executed for one
    decision in a cloned world, the teacher acts for the remaining horizon;
    value = curriculum progress (invalid candidates: -inf)."""
    teacher = teacher or D2PredictivePolicy()
    n = cenv.n
    if branch_env is None:
        branch_env = CurriculumEnv(cenv.scenario.scenario_id, cenv.category, n * ACTIONS, cenv.device,
                                   seed=cenv.seed, action_ticks=cenv.action_ticks)
        branch_env.reset()
    _clone_rows(cenv, branch_env, ACTIONS)
    first = torch.arange(ACTIONS, device=cenv.device).repeat(n)
    total = torch.zeros(n * ACTIONS, device=cenv.device)
    act = first
    for k in range(horizon):
        _, reward, done = branch_env.step(act)
        total += reward
        if bool(done.all()):
            break
        act = teacher.choose(branch_env)
    value = total.reshape(n, ACTIONS)
    valid = cenv.env.ws["obs"][:, SLOT, -8:] > .5
    value = value.masked_fill(~valid, -math.inf)
    return value.argmax(-1), value


# --------------------------------------------------------------------------- PPO
def train_meco(config: MecoConfig, ledger: MetricLedger | None = None) -> tuple[MecoPolicy, list[dict]]:
    """Recurrent PPO of one MECO track on one curriculum scenario (category 0)."""
    torch.manual_seed(config.seed)
    dev = torch.device(config.device)
    sc = get_scenario(config.scenario)
    cenv = CurriculumEnv(config.scenario, sc.required_categories[0], config.envs, dev, seed=config.seed)
    policy = MecoPolicy(config.track).to(dev)
    opt = torch.optim.Adam(policy.parameters(), lr=config.learning_rate, eps=1e-5)
    history = []
    if config.warm_start_decisions:
        loss = supervised_warm_start(policy, cenv, opt, config.warm_start_decisions)
        history.append({"phase": "warm_start", "loss": loss})
    cenv.reset()
    hidden = None
    decisions = max(4, int(math.ceil(cenv.budget_ticks / cenv.action_ticks)) // 2)
    for update in range(config.updates):
        # the update replays the policy on the stored world snapshots
        snaps, buf = [], {k: [] for k in ("hidden", "act", "logp", "value", "reward", "done")}
        for _ in range(decisions):
            snaps.append({k: v.clone() for k, v in cenv.env.ws.state_dict().items() if k != "raster_pts"})
            with torch.no_grad():
                dist, value, nh, _, _, _ = policy.distribution(cenv.env, hidden)
                act = dist.sample()
            buf["hidden"].append(hidden if hidden is not None else torch.zeros_like(nh))
            buf["act"].append(act)
            buf["logp"].append(dist.log_prob(act))
            buf["value"].append(value)
            _, reward, done = cenv.step(act)
            buf["reward"].append(reward)
            buf["done"].append(done.float())
            hidden = nh
            if bool(done.all()):
                cenv.reset()
                hidden = None
        with torch.no_grad():
            _, last_value, _, _, _, _ = policy.distribution(cenv.env, hidden)
        rewards, dones, values = (torch.stack(buf[k]) for k in ("reward", "done", "value"))
        adv = torch.zeros_like(rewards)
        gae = torch.zeros_like(last_value)
        nxt = last_value
        for t in reversed(range(decisions)):
            nonterm = 1. - dones[t]
            delta = rewards[t] + config.gamma * nxt * nonterm - values[t]
            gae = delta + config.gamma * config.lam * nonterm * gae
            adv[t] = gae
            nxt = values[t]
        ret = adv + values
        adv = (adv - adv.mean()) / adv.std().clamp_min(1e-6)
        live = {k: v.clone() for k, v in cenv.env.ws.state_dict().items() if k != "raster_pts"}
        stats = []
        for _ in range(config.epochs):
            for t in range(decisions):
                cenv.env.ws.load_state_dict(snaps[t])
                dist, value, _, _, _, _ = policy.distribution(cenv.env, buf["hidden"][t])
                ratio = (dist.log_prob(buf["act"][t]) - buf["logp"][t]).exp()
                pg = -torch.minimum(ratio * adv[t], ratio.clamp(1 - config.clip, 1 + config.clip) * adv[t]).mean()
                vloss = .5 * (value - ret[t]).square().mean()
                loss = pg + .5 * vloss - config.entropy * dist.entropy().mean()
                opt.zero_grad()
                loss.backward()
                nn.utils.clip_grad_norm_(policy.parameters(), .5)
                opt.step()
                stats.append((pg.item(), vloss.item()))
        cenv.env.ws.load_state_dict(live)
        row = {"update": update, "reward": float(rewards.sum(0).mean()), "policy_loss": stats[-1][0],
               "value_loss": stats[-1][1]}
        history.append(row)
        if ledger is not None:
            ledger.append("meco_update", {"config": config.identity(), "track": config.track, **row})
    return policy, history


# --------------------------------------------------------------------------- evaluation
ABLATIONS = ("full", "no_penalty", "no_memory", "uniform_utility")


def evaluate_meco(policy: MecoPolicy | None, scenario: str, *, episodes: int, split: str = "validation",
                  master_seed: int = 0, device="cpu", max_age_s: float = .25, ablation: str = "full") -> dict:
    """Matched-seed evaluation of the track (through the fail-closed arbiter)
    and of the scripted teacher on the same seeds. `ablation` removes one
    part of the scorer at decision time: ``no_penalty`` (risk penalties
    zeroed), ``no_memory`` (recurrent state reset every decision),
    ``uniform_utility`` (every valid candidate scored alike, so the arbiter's
    tie order decides). Per-episode outcomes are kept for paired tests."""
    if ablation not in ABLATIONS:
        raise ValueError(f"ablation must be one of {ABLATIONS}")
    sc = get_scenario(scenario)
    seeds = seed_partition(scenario, split, len(sc.required_categories))
    teacher = D2PredictivePolicy()
    out = {"scenario": scenario, "split": split, "categories": []}
    totals = {"meco": [0, 0], "teacher": [0, 0]}
    fallbacks = {}
    for seed, cat in zip(seeds, sc.required_categories):
        row = {"category": cat}
        for arm in ("meco", "teacher"):
            if arm == "meco" and policy is None:
                continue
            cenv = CurriculumEnv(scenario, cat, episodes, device, seed=seed ^ master_seed)
            cenv.reset()
            hidden, done = None, torch.zeros(cenv.n, dtype=torch.bool, device=cenv.device)
            while not bool(done.all()):
                fallback = teacher.choose(cenv)
                if arm == "meco":
                    with torch.no_grad():
                        util, pen, valid, _, hidden = policy(cenv.env, None if ablation == "no_memory" else hidden)
                    if ablation == "no_penalty":
                        pen = torch.zeros_like(pen)
                    elif ablation == "uniform_utility":
                        util = torch.zeros_like(util)
                    ids = tuple(f"action-{k}" for k in range(ACTIONS))
                    now = float(cenv.elapsed) * cenv.env.dt
                    choice = []
                    for i in range(cenv.n):
                        req = DecisionRequest(ids, tuple(bool(v) for v in valid[i].tolist()), ids[int(fallback[i])],
                                              now, max_age_s)
                        res = ScorerOutput(ids, tuple(util[i].tolist()), tuple(pen[i].tolist()), now)
                        cid, why = choose_candidate(req, res)
                        fallbacks[why] = fallbacks.get(why, 0) + 1
                        choice.append(ids.index(cid))
                    act = torch.tensor(choice, device=cenv.device)
                else:
                    act = fallback
                _, _, done = cenv.step(act)
            ok = episode_success(scenario, cat, cenv.metrics.counts(), cenv)
            row[arm] = int(ok.sum())
            row[f"{arm}_episodes"] = [bool(v) for v in ok.tolist()]
            totals[arm][0] += int(ok.sum())
            totals[arm][1] += cenv.n
        out["categories"].append(row)
    for arm, (s, n) in totals.items():
        if n:
            out[arm] = {"success_rate": s / n, "wilson_95": wilson_interval(s, n), "episodes": n}
    out["arbiter"] = fallbacks
    out["ablation"] = ablation
    return out


# --------------------------------------------------------------------------- CLI
def _parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="autodrive_b200.meco.train", description=__doc__.split("\n")[0])
    sub = p.add_subparsers(dest="command", required=True)
    t = sub.add_parser("train", help="recurrent PPO of one MECO track")
    t.add_argument("--track", default="C1", choices=("A1", "A2", "A3", "C1", "C2"))
    t.add_argument("--scenario", default="pickup_simple", choices=sorted(SCENARIOS))
    t.add_argument("--envs", type=int, default=32)
    t.add_argument("--updates", type=int, default=10)
    t.add_argument("--epochs", type=int, default=2)
    t.add_argument("--learning-rate", type=float, default=3e-4)
    t.add_argument("--warm-start-decisions", type=int, default=0)
    t.add_argument("--seed", type=int, default=0)
    t.add_argument("--device", default="cpu")
    t.add_argument("--output", required=True)
    e = sub.add_parser("evaluate", help="matched-seed evaluation against the scripted teacher")
    e.add_argument("--checkpoint", default=None)
    e.add_argument("--scenario", default="pickup_simple", choices=sorted(SCENARIOS))
    e.add_argument("--episodes", type=int, default=16)
    e.add_argument("--split", default="validation")
    e.add_argument("--device", default="cpu")
    c = sub.add_parser("counterfactual", help="branch-rollout labels of the current decision")
    c.add_argument("--scenario", default="pickup_simple", choices=sorted(SCENARIOS))
    c.add_argument("--envs", type=int, default=4)
    c.add_argument("--horizon", type=int, default=4)
    c.add_argument("--device", default="cpu")
    return p


def main(argv=None) -> int:
    args = _parser().parse_args(argv)
    if args.command == "train":
        cfg = MecoConfig(track=args.track, scenario=args.scenario, envs=args.envs, updates=args.updates,
                         epochs=args.epochs, learning_rate=args.learning_rate,
                         warm_start_decisions=args.warm_start_decisions, seed=args.seed, device=args.device,
                         output=args.output)
        out = Path(args.output)
        out.mkdir(parents=True, exist_ok=True)
        ledger = MetricLedger(out / "metric-ledger.jsonl")
        policy, history = train_meco(cfg, ledger)
        from ..utils.provenance import state_dict_digest
        payload = {"track": cfg.track, "config": asdict(cfg), "model_state_dict": policy.state_dict(),
                   "history": history}
        payload["weights_sha256"] = state_dict_digest(payload["model_state_dict"])
        torch.save(payload, out / "meco.pt")
        ledger.append("checkpoint", {"path": "meco.pt", "weights_sha256": payload["weights_sha256"]})
        print(json.dumps({"output": str(out), "updates": len(history), "weights_sha256": payload["weights_sha256"]}))
    elif args.command == "evaluate":
        policy = None
        if args.checkpoint:
            from ..utils.checkpoint import load_verified
            payload = load_verified(args.checkpoint, map_location=args.device, weights_only=False)
            policy = MecoPolicy(payload["track"]).to(args.device)
            policy.load_state_dict(payload["model_state_dict"])
            policy.eval()
        print(json.dumps(evaluate_meco(policy, args.scenario, episodes=args.episodes, split=args.split,
                                       device=args.device)))
    else:
        sc = get_scenario(args.scenario)
        cenv = CurriculumEnv(args.scenario, sc.required_categories[0], args.envs, args.device)
        cenv.reset()
        best, value = counterfactual_labels(cenv, args.horizon)
        print(json.dumps({"labels": best.tolist(), "values": torch.nan_to_num(value, neginf=-1e9).tolist()}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
