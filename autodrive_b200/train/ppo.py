"""Device-resident PPO for the defense environments.

Behaviour follows frc_defense/tensor_training_ppo.py:12-631: Adam(lr 3e-4,
eps 1e-5) per train call, strategic decisions held 12/13 ticks at 4 Hz,
GAE with truncation bootstrapping, epochs x shuffled minibatches,
minibatch advantage normalisation over all ranks, loss = clipped policy
gradient + 0.5 value + linearly decayed entropy + L2 on weight matrices,
global-norm clip 0.5, checkpoints and status written atomically by rank 0.

B200 path: rollouts stay on the device (simulator kernels, one CUDA graph per
held interval for the 3v3 env), GAE is one kernel that also yields the
advantage statistics, and the update's gradient reduction + clip + Adam run
as fused kernels over one flat parameter buffer.
"""
from __future__ import annotations

import json
import math
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any

import torch

from ..models import build_policy
from ..ops import policy_tc
from ..utils import trace
from ..parallel import dist as pdist
from ..parallel.grad_sync import GradientSync, sync_parameters
from .optim import FusedAdam
from .rollout import DefenseAgents, StrategicClock, ThreeVsThreeAgents, gae_advantages, stack_inputs

OBS_NORMALIZATION = "fixed_physical_scale_v1"
DEFENSE_TRAINING_OPPONENTS = ("offense", "adstar", "mirror", "cutoff", "velocity_intercept")
CURRICULUM_STAGES = ("static_straight", "scripted", "adstar", "mixed")
STATIC_OPPONENT_FRACTION = .20


def curriculum_stage(progress: float) -> int:
    return min(len(CURRICULUM_STAGES) - 1, max(0, int(max(0., min(.999999, progress)) * len(CURRICULUM_STAGES))))


def curriculum_opponents(stage: int) -> tuple[str, ...]:
    pools = (("offense",), ("offense", "mirror"), ("offense", "mirror", "adstar"), DEFENSE_TRAINING_OPPONENTS)
    return pools[min(max(0, stage), len(pools) - 1)]


@dataclass
class PPOConfig:
    rollout_steps: int = 128
    epochs: int = 4
    minibatch_size: int = 4096
    learning_rate: float = 3e-4
    gamma: float = .993
    gae_lambda: float = .95
    clip_coef: float = .2
    value_coef: float = .5
    entropy_coef: float = .01
    max_grad_norm: float = .5
    l2_coef: float = 1e-5
    strategic_rate_hz: float = 4.
    grad_backend: str = "auto"
    bf16: bool = False
    # tcgen05 kernels for the 2 x 128 categorical policy on CUDA (act + update)
    fused_policy: bool = True


def atomic_json(path: Path, value: dict) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(value, indent=2, default=str))
    tmp.replace(path)


def atomic_save(path: Path, value: dict) -> None:
    tmp = path.with_suffix(path.suffix + ".tmp")
    torch.save(value, tmp)
    tmp.replace(path)


def make_env(kind: str, num_envs: int, device, seed: int, opponent: str, horizon: int,
             architecture: str = "strategic_adstar", fuel_physics=True, static_opponent_fraction: float = 0.,
             observe_every_tick: bool = False, **env_kwargs):
    """Environment factory (frc_defense/tensor_training_runtime.py:156-178). Extra keywords go to
    the 3v3 environment (FUEL count, perception interval, planner resolution, ...);
    `observe_every_tick` makes the 3v3 agents build observations at the physics rate."""
    if kind == "3v3":
        from ..sim.env3v3 import TensorThreeVsThreeEnv
        env = TensorThreeVsThreeEnv(num_envs=num_envs, device=device, seed=seed, horizon=horizon,
                                    control_modes=("deterministic",) * 3 + ("nn",) * 3,
                                    fuel_physics=fuel_physics, **env_kwargs)
        return ThreeVsThreeAgents(env, observe_every_tick)
    from ..sim.env_defense import TensorDefenseEnv
    mode = {"direct": "direct", "tactical_adstar": "tactical", "strategic_adstar": "strategic"}.get(
        architecture, architecture)
    env = TensorDefenseEnv(num_envs=num_envs, task="defense", device=device, seed=seed, opponent=opponent,
                           horizon=horizon, action_mode=mode, fuel_physics=fuel_physics,
                           static_opponent_fraction=static_opponent_fraction, **env_kwargs)
    return DefenseAgents(env)


class PPOLearner:
    """Policy, fused optimizer and update step shared by the trainers and bench."""

    def __init__(self, obs_dim: int, action_dim: int, action_kind: str, device, cfg: PPOConfig,
                 network: str = "mlp", world: int = 1, initial_state: dict | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        self.model = build_policy(network, obs_dim, action_dim, action_kind).to(self.device)
        from ..models.zoo import PerceptionActorCritic
        # architecture-zoo networks read perception dictionaries and train in
        # bf16 autocast on CUDA (fp32 master weights, fp32 accumulation)
        self.perception = isinstance(self.model, PerceptionActorCritic)
        if self.perception and self.device.type == "cuda":
            cfg.bf16 = True
        if initial_state is not None:
            self.model.load_state_dict(initial_state)
        self.opt = FusedAdam(self.model, lr=cfg.learning_rate, eps=1e-5, max_grad_norm=cfg.max_grad_norm)
        self.sync = GradientSync(self.opt, world, cfg.grad_backend)
        # every replica starts from rank 0's weights: one peer-memory broadcast
        # kernel on the fused path, per-parameter collectives otherwise
        if world > 1 and getattr(self.sync, "fused", None) is not None:
            self.sync.fused.broadcast_parameters(0)
            self.sync.fused.check()
        else:
            sync_parameters(self.model, world)
        self.world = world
        self.action_kind = action_kind
        self.action_dim = action_dim
        self.tc = None
        if (cfg.fused_policy and self.device.type == "cuda" and not cfg.bf16
                and policy_tc.supported(self.model)):
            self.tc = policy_tc.TensorCorePolicy(self.model, self.opt.flat)
        self.weights_version = 0
        self._loss_stats = torch.zeros(5, device=self.device)

    def weights_changed(self) -> None:
        """Call after writing parameters outside the optimizer (checkpoint loads)."""
        self.weights_version += 1

    def _tc_ready(self):
        self.tc.ensure_packed(self.weights_version)
        return self.tc

    def _mask(self, obs):
        if self.action_kind != "categorical":
            return None
        scalars = obs["scalars"] if isinstance(obs, dict) else obs
        return scalars[:, -self.action_dim:] > .5

    @torch.no_grad()
    def act(self, obs):
        if self.tc is not None:
            return self._tc_ready().act(obs)
        mask = self._mask(obs)
        with torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=self.cfg.bf16 and self.device.type == "cuda"):
            action, logp, value = self.model.sample(obs, action_mask=mask)
        return action, logp.float(), value.float(), mask

    @torch.no_grad()
    def value(self, obs: torch.Tensor) -> torch.Tensor:
        if self.tc is not None:
            return self._tc_ready().act(obs, value_only=True)
        with torch.autocast(self.device.type, dtype=torch.bfloat16, enabled=self.cfg.bf16 and self.device.type == "cuda"):
            return self.model(obs)[2].float()

    def update(self, flat: dict, entropy_coef: float) -> dict:
        """epochs x minibatches of clipped PPO on one rollout batch."""
        if self.tc is not None:
            return self._update_tc(flat, entropy_coef)
        cfg = self.cfg
        n = flat["actions"].shape[0]
        mb = min(cfg.minibatch_size, n)
        kl = torch.zeros((), device=self.device)
        clip_frac = torch.zeros((), device=self.device)
        ent = torch.zeros((), device=self.device)
        samples, batches = 0, 0
        obs_all = flat["obs"]
        for _ in range(cfg.epochs):
            perm = torch.randperm(n, device=self.device)
            for idx in perm.split(mb):
                mask = flat["mask"][idx] if flat["mask"] is not None else None
                obs = ({k: v[idx] for k, v in obs_all.items()} if isinstance(obs_all, dict) else obs_all[idx])
                with torch.autocast(self.device.type, dtype=torch.bfloat16,
                                    enabled=cfg.bf16 and self.device.type == "cuda"):
                    logp, entropy, value, _ = self.model.score(obs, flat["actions"][idx], mask)
                logp, entropy, value = logp.float(), entropy.float(), value.float()
                logratio = logp - flat["logp"][idx]
                ratio = logratio.exp()
                kl += ((ratio - 1.) - logratio).detach().sum()
                clip_frac += ((ratio - 1.).abs() > cfg.clip_coef).detach().sum()
                adv = flat["adv"][idx]
                if self.world > 1:
                    stats = torch.stack((adv.sum(), adv.square().sum(), adv.new_tensor(float(adv.numel()))))
                    pdist.all_reduce_(stats)
                    mean = stats[0] / stats[2].clamp_min(1.)
                    var = (stats[1] / stats[2].clamp_min(1.) - mean.square()).clamp_min(0.)
                    adv = (adv - mean) / (var.sqrt() + 1e-8)
                else:
                    adv = (adv - adv.mean()) / (adv.std(unbiased=False) + 1e-8)
                pg = torch.maximum(-adv * ratio, -adv * ratio.clamp(1 - cfg.clip_coef, 1 + cfg.clip_coef)).mean()
                vloss = .5 * (value - flat["returns"][idx]).square().mean()
                l2 = sum(p.square().sum() for p in self.model.parameters() if p.ndim > 1)
                loss = pg + cfg.value_coef * vloss - entropy_coef * entropy.mean() + cfg.l2_coef * l2
                self.opt.zero_grad()
                loss.backward()
                self.sync.step()
                ent += entropy.mean().detach()
                samples += int(idx.numel())
                batches += 1
        if self.perception and self.device.type == "cuda":
            from ..ops.tc_linear import check_gemm_status
            check_gemm_status(self.device, block=False)
        return {"approx_kl_sum": kl, "clip_fraction_sum": clip_frac, "entropy_sum": ent,
                "samples": samples, "batches": batches}


    def _update_tc(self, flat: dict, entropy_coef) -> dict:
        """The update on the tensor-core kernels: per minibatch one fused
        forward+backward, the partial-gradient reduction and the fused
        clip + Adam; no autograd graph and no host synchronisation."""
        cfg, tc = self.cfg, self._tc_ready()
        tc.check()
        n = flat["obs"].shape[0]
        mb = min(cfg.minibatch_size, n)
        batch = {"obs": flat["obs"].contiguous().float(), "actions": flat["actions"].reshape(-1).long().contiguous(),
                 "mask": None if flat.get("mask") is None else flat["mask"].contiguous(),
                 "logp": flat["logp"].contiguous().float(), "adv": flat["adv"].contiguous().float(),
                 "returns": flat["returns"].contiguous().float()}
        if torch.is_tensor(entropy_coef):
            ent = entropy_coef.reshape(1).to(self.device, torch.float32)
        else:
            ent = torch.full((1,), float(entropy_coef), device=self.device)
        stats = self._loss_stats
        stats.zero_()
        # every minibatch of the update is drawn up front, so the advantage
        # statistics of all of them cross the ranks in one exchange instead of
        # one synchronising all-reduce per minibatch
        plan = [idx for _ in range(cfg.epochs) for idx in torch.randperm(n, device=self.device).split(mb)]
        adv_stats = tc.minibatch_adv_stats(batch["adv"], plan)
        if self.world > 1:
            fused = getattr(self.sync, "fused", None)
            flat_stats = adv_stats.view(-1)
            if fused is not None:
                for k in range(0, flat_stats.numel(), 15):   # the peer stats kernel carries <= 16 values
                    chunk = flat_stats[k:k + 15].clone()
                    fused.stats_allreduce(chunk)
                    flat_stats[k:k + 15].copy_(chunk)
            else:
                pdist.all_reduce_(flat_stats)
        samples, batches = 0, 0
        for k, idx in enumerate(plan):
            tc.train_minibatch(batch, idx, ent, cfg.clip_coef, cfg.value_coef, cfg.l2_coef, stats,
                               adv_stats=adv_stats[k])
            self.sync.step()
            self.weights_version += 1
            tc.pack(self.weights_version)
            samples += int(idx.numel())
            batches += 1
        tc._post_status()
        return {"approx_kl_sum": stats[0], "clip_fraction_sum": stats[1], "entropy_sum": stats[2],
                "policy_loss_sum": stats[3], "value_loss_sum": stats[4], "samples": samples, "batches": batches}


def collect_rollout(agents, learner: PPOLearner, obs: torch.Tensor, steps: int, clock: StrategicClock,
                    episode_ticks: list[int]):
    """Fill one rollout of `steps` decisions; returns (buffers, next obs, tick count)."""
    dev = learner.device
    A, D = agents.n_agents, agents.obs_dim
    cont = learner.action_kind == "continuous"
    dict_obs = isinstance(obs, dict)
    buf = {
        "obs": [] if dict_obs else torch.empty((steps, A, D), device=dev),
        "actions": torch.empty((steps, A, learner.action_dim) if cont else (steps, A), device=dev,
                               dtype=torch.float32 if cont else torch.long),
        "mask": None if cont else torch.empty((steps, A, learner.action_dim), device=dev, dtype=torch.bool),
        "logp": torch.empty((steps, A), device=dev),
        "values": torch.empty((steps, A), device=dev),
        "next_values": torch.empty((steps, A), device=dev),
        "rewards": torch.empty((steps, A), device=dev),
        "dones": torch.empty((steps, A), device=dev, dtype=torch.bool),
        "truncated": torch.empty((steps, A), device=dev, dtype=torch.bool),
    }
    ticks_total = 0
    horizon = agents.horizon
    for t in range(steps):
        if dict_obs:
            buf["obs"].append(obs)
        else:
            buf["obs"][t] = obs
        action, logp, value, mask = learner.act(obs)
        if mask is not None:
            buf["mask"][t] = mask
        ticks = clock.next()
        remaining = horizon - episode_ticks[0]
        next_obs, reward, done, truncated = agents.act(action, ticks, remaining)
        used = min(ticks, remaining)
        episode_ticks[0] += used
        ticks_total += used
        boundary = episode_ticks[0] >= horizon
        buf["actions"][t], buf["logp"][t], buf["values"][t] = action, logp, value
        buf["rewards"][t] = reward
        buf["dones"][t] = done
        buf["truncated"][t] = truncated | boundary
        if t > 0:
            prev_end = buf["dones"][t - 1] | buf["truncated"][t - 1]
            buf["next_values"][t - 1] = torch.where(prev_end, buf["next_values"][t - 1], value)
        if boundary or t == steps - 1:
            buf["next_values"][t] = learner.value(next_obs)
        if boundary:
            episode_ticks[0] = 0
            next_obs = agents.reset_done(torch.ones(A, dtype=torch.bool, device=dev))
        obs = next_obs
    if dict_obs:
        buf["obs"] = stack_inputs(buf["obs"])
    return buf, obs, ticks_total


def flatten_rollout(buf: dict, adv: torch.Tensor, obs_dim: int, action_dim: int, action_kind: str) -> dict:
    """Rollout buffers [T, A, ...] -> one flat PPO batch [T*A, ...]."""
    obs = buf["obs"] if isinstance(buf["obs"], dict) else buf["obs"].reshape(-1, obs_dim)
    return {"obs": obs,
            "actions": buf["actions"].reshape((-1, action_dim) if action_kind == "continuous" else (-1,)),
            "mask": buf["mask"].reshape(-1, action_dim) if buf["mask"] is not None else None,
            "logp": buf["logp"].reshape(-1), "adv": adv.reshape(-1),
            "returns": (adv + buf["values"]).reshape(-1)}


def train_once(task: str, timesteps: int, output, *, seed: int, num_envs: int, device, opponent: str,
               initial_checkpoint=None, rollout_steps: int = 128, epochs: int = 4, minibatch_size: int = 4096,
               learning_rate: float = 3e-4, gamma: float = .993, gae_lambda: float = .95, clip_coef: float = .2,
               value_coef: float = .5, entropy_coef: float = .01, max_grad_norm: float = .5,
               l2_coef: float = 1e-5, horizon: int = 8000, architecture: str = "strategic_adstar",
               curriculum: bool = True, strategic_rate_hz: float = 4., env_kind: str = "defense",
               network: str = "mlp", fuel_physics=True, grad_backend: str = "auto", bf16: bool = False,
               status_context: dict | None = None, dist_state=None,
               env_kwargs: dict | None = None) -> dict[str, Any]:
    if task != "defense":
        raise ValueError("only defense policies are trainable; offense is deterministic")
    if opponent not in (*DEFENSE_TRAINING_OPPONENTS, "mixed"):
        raise ValueError("opponent must be a deterministic defense-training baseline")
    state = dist_state or pdist.distributed_state(device)
    rank, world, dev = state.rank, state.world, state.device
    rank_seed = seed + rank * 1_000_003
    torch.manual_seed(rank_seed)
    cfg = PPOConfig(rollout_steps=rollout_steps, epochs=epochs, minibatch_size=minibatch_size,
                    learning_rate=learning_rate, gamma=gamma, gae_lambda=gae_lambda, clip_coef=clip_coef,
                    value_coef=value_coef, entropy_coef=entropy_coef, max_grad_norm=max_grad_norm,
                    l2_coef=l2_coef, strategic_rate_hz=strategic_rate_hz, grad_backend=grad_backend, bf16=bf16)
    agents = make_env(env_kind, num_envs, dev, rank_seed, "offense" if opponent == "mixed" else opponent,
                      horizon, architecture, fuel_physics,
                      STATIC_OPPONENT_FRACTION if env_kind == "defense" else 0., **(env_kwargs or {}))
    action_kind = agents.action_kind
    initial_state = None
    # with the peer-memory broadcast, rank 0 alone reads the checkpoint and the
    # learner's initial sync moves its weights to the other ranks
    peer_broadcast = world > 1 and dev.type == "cuda" and grad_backend in ("auto", "p2p")
    if initial_checkpoint is not None and (rank == 0 or not peer_broadcast):
        from ..utils.checkpoint import load_verified
        payload = load_verified(initial_checkpoint, map_location=dev)
        if payload.get("task") != "defense":
            raise ValueError("initial checkpoint must be tagged as a defense policy")
        if payload.get("drivetrain_config") != agents.drivetrain_config:
            raise ValueError("initial checkpoint drivetrain configuration does not match this run")
        if payload.get("architecture", "direct") != architecture:
            raise ValueError("initial checkpoint architecture differs from this training run")
        if payload.get("network", "mlp") != network:
            raise ValueError("initial checkpoint network differs from this training run")
        initial_state = payload["model_state_dict"]
    learner = PPOLearner(agents.obs_dim, agents.action_dim, action_kind, dev, cfg, network, world, initial_state)
    if learner.perception:
        if not hasattr(agents, "use_perception"):
            raise ValueError(f"network {network!r} reads perception inputs of the 3v3 environment; use env_kind='3v3'")
        agents.use_perception(learner.model.field_shape, learner.model.input_keys)
    out = Path(output)
    if rank == 0:
        out.mkdir(parents=True, exist_ok=True)
    status_path, checkpoint = out / "status.json", out / "policy.pt"
    status_context = dict(status_context or {})
    updates = max(1, (timesteps + rollout_steps * num_envs - 1) // (rollout_steps * num_envs))
    if rank == 0:
        atomic_json(status_path, {**status_context, "status": "running", "task": task, "opponent": opponent,
                                  "architecture": architecture, "network": network, "action_kind": action_kind,
                                  "updates": updates, "world_size": world})
    obs = agents.reset()
    clock = StrategicClock(strategic_rate_hz) if action_kind == "categorical" else None
    clock = clock or _UnitClock()
    episode_ticks = [0]
    started = time.perf_counter()
    totals = {"transitions": 0, "physics_world_ticks": 0, "return_sum": 0., "episodes": 0}
    action_counts = torch.zeros(agents.action_dim, device=dev)
    history = []
    result: dict[str, Any] = {}
    for update in range(updates):
        if curriculum and env_kind == "defense" and hasattr(agents.env, "ws"):
            pool = curriculum_opponents(curriculum_stage(update / max(1, updates)))
            kind = pool[update % len(pool)]
            from ..sim.env_defense import OPPONENT_KINDS
            agents.env.ws.sim  # parameters are baked per world; opponent variants switch via params
            agents.env.opponent = kind
            _set_opponent(agents.env, OPPONENT_KINDS[kind])
        t0 = time.perf_counter()
        with trace.stage("rollout"):
            buf, obs, ticks = collect_rollout(agents, learner, obs, rollout_steps, clock, episode_ticks)
        stats = torch.zeros(3, dtype=torch.float64, device=dev)
        with trace.stage("gae"):
            adv = gae_advantages(buf["rewards"], buf["dones"], buf["truncated"], buf["values"],
                                 buf["next_values"], gamma, gae_lambda, stats)
        flat = flatten_rollout(buf, adv, agents.obs_dim, agents.action_dim, action_kind)
        if action_kind == "categorical":
            action_counts += torch.bincount(flat["actions"], minlength=agents.action_dim).float()
        coef = entropy_coef * max(0., 1. - update / max(1, updates - 1))
        with trace.stage("update"):
            upd = learner.update(flat, coef)
        counters = torch.tensor([float(rollout_steps * agents.n_agents), float(ticks * num_envs),
                                 float(buf["rewards"].sum().item()), float(upd["samples"]),
                                 float(upd["approx_kl_sum"].item()), float(upd["clip_fraction_sum"].item()),
                                 float(upd["entropy_sum"].item()), float(upd["batches"])],
                                dtype=torch.float64, device=dev)
        pdist.all_reduce_(counters)
        elapsed = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=dev)
        pdist.all_reduce_(elapsed, "max")
        totals["transitions"] += int(counters[0])
        totals["physics_world_ticks"] += int(counters[1])
        wall = time.perf_counter() - started
        record = {"update": update + 1, "updates": updates, "transitions": totals["transitions"],
                  "transitions_per_second": totals["transitions"] / max(wall, 1e-9),
                  "physics_world_ticks_per_second": totals["physics_world_ticks"] / max(wall, 1e-9),
                  "update_seconds_max_rank": float(elapsed), "mean_reward": float(counters[2] / max(1., counters[0])),
                  "approx_kl": float(counters[4] / max(1., counters[3])),
                  "clip_fraction": float(counters[5] / max(1., counters[3])),
                  "entropy": float(counters[6] / max(1., counters[7])),
                  "grad_norm": float(learner.opt.last_norm.item())}
        history.append(record)
        if rank == 0:
            atomic_save(checkpoint, checkpoint_payload(learner.model, agents, architecture, network, action_kind,
                                                      learner.opt))
            dist_counts = (action_counts / action_counts.sum().clamp_min(1)).tolist()
            atomic_json(status_path, {**status_context, "status": "running", "task": task, "opponent": opponent,
                                      "architecture": architecture, "network": network, **record,
                                      "action_distribution": dist_counts, "world_size": world})
        result = record
    scores, acquisitions = agents.score_counts()
    import hashlib
    digest = hashlib.sha256(learner.opt.flat.flat.detach().float().cpu().numpy().tobytes()).hexdigest()
    final = {**status_context, "status": "completed", "task": task, "opponent": opponent,
             "parameters_sha256": digest,
             "architecture": architecture, "network": network, "checkpoint": str(checkpoint),
             **result, "history": history[-20:],
             "team_scores": scores.sum(0).tolist(), "acquisitions": acquisitions.sum(0).tolist(),
             "world_size": world}
    if rank == 0:
        atomic_json(status_path, final)
        atomic_json(out / "metadata.json", {k: v for k, v in final.items() if k != "history"})
    return final


class _UnitClock:
    def next(self) -> int:
        return 1


def _set_opponent(env, code: int) -> None:
    """Switch the scripted attacker behaviour between rollouts."""
    params = dict(env.ws.params)
    if params.get("opponent_kind") == code:
        return
    params["opponent_kind"] = code
    from ..ops import require_extension
    ext = require_extension()
    tensors = [env.ws.t[name] for name, _, _ in env.ws.schema]
    env.ws.params = params
    env.ws.sim = ext.Sim(tensors, params)


def checkpoint_payload(model, agents, architecture, network, action_kind, optimizer=None) -> dict:
    """Reference-compatible policy.pt payload (frc_defense/tensor_training_ppo.py:455-459)."""
    payload = {"model_state_dict": model.state_dict(), "obs_dim": agents.obs_dim,
               "action_dim": agents.action_dim, "action_kind": action_kind, "architecture": architecture,
               "task": "defense", "observation_normalization": OBS_NORMALIZATION,
               "drivetrain_config": agents.drivetrain_config, "network": network,
               "env": "3v3" if isinstance(agents, ThreeVsThreeAgents) else "defense"}
    if isinstance(agents, ThreeVsThreeAgents):
        payload["observation_spec"] = "per-robot-3v3-v1"
    if optimizer is not None:
        payload["optimizer_state_dict"] = optimizer.state_dict()
    # provenance: SHA-256 tree digest of the weights, computed where they live
    from ..utils.provenance import state_dict_digest
    payload["weights_sha256"] = state_dict_digest(payload["model_state_dict"])
    from ..ops.ext import native_extension_identity
    ident = native_extension_identity()
    payload["native_extension"] = {k: ident.get(k) for k in ("sha256", "build_fingerprint", "sources_match_build")}
    return payload
