"""Categorical Soft Actor-Critic for the curriculum (``--algorithm sac``).

Behaviour follows frc_defense/discrete_sac.py:40-246: a categorical actor,
twin Q critics with Polyak-averaged targets, a learned temperature driven
towards a target entropy of ``fraction * log(#valid actions)``, masked
action distributions, and a replay sampled evenly across the scenarios it
currently holds.

B200 design: the replay is a device-resident ring (every field, including
perception dictionaries, is one preallocated tensor in HBM; a 100k-row
perception replay with 12 x 32 x 64 rasters is ~10 GB, small next to 180 GB),
so adding a rollout batch is one scatter and sampling a minibatch is one
gather, with no per-row host objects or host<->device copies.
"""
from __future__ import annotations

from collections.abc import Mapping

import torch
from torch import nn

from ..models.zoo import make_policy


def _logits_value(policy, obs):
    out = policy(obs)
    return (out[0], out[2]) if len(out) == 3 else (out[0], out[1])


def masked_distribution(logits: torch.Tensor, action_mask: torch.Tensor):
    """(probs, log_probs with masked entries zeroed, mask) of the masked softmax."""
    mask = action_mask.bool()
    if mask.shape != logits.shape:
        raise ValueError("action mask shape must match categorical logits")
    logp = logits.masked_fill(~mask, torch.finfo(logits.dtype).min).log_softmax(-1)
    return logp.exp().masked_fill(~mask, 0.), logp.masked_fill(~mask, 0.), mask


class DiscreteQ(nn.Module):
    """Q-values as the logits head of a policy network of the same architecture."""

    def __init__(self, architecture: str):
        super().__init__()
        self.network = make_policy(architecture)

    def forward(self, obs):
        return _logits_value(self.network, obs)[0]


class DiscreteSAC(nn.Module):
    def __init__(self, architecture: str = "baseline_mlp", initial_alpha: float = .2):
        super().__init__()
        self.algorithm, self.architecture = "sac", architecture
        self.actor = make_policy(architecture)
        self.q1, self.q2 = DiscreteQ(architecture), DiscreteQ(architecture)
        self.target_q1, self.target_q2 = DiscreteQ(architecture), DiscreteQ(architecture)
        self.target_q1.load_state_dict(self.q1.state_dict())
        self.target_q2.load_state_dict(self.q2.state_dict())
        for p in (*self.target_q1.parameters(), *self.target_q2.parameters()):
            p.requires_grad_(False)
        self.log_alpha = nn.Parameter(torch.tensor(float(initial_alpha)).log())

    @property
    def alpha(self) -> torch.Tensor:
        return self.log_alpha.exp()

    def forward(self, obs):
        logits, value = _logits_value(self.actor, obs)
        return logits, None, value

    def sample(self, obs, deterministic: bool = False, action_mask=None):
        logits, _, value = self(obs)
        if action_mask is None:
            action_mask = torch.ones_like(logits, dtype=torch.bool)
        probs, logp, _ = masked_distribution(logits, action_mask)
        action = probs.argmax(-1) if deterministic else torch.distributions.Categorical(probs=probs).sample()
        return action, logp.gather(-1, action[:, None]).squeeze(-1), value


def make_sac_optimizers(agent: DiscreteSAC, learning_rate: float) -> dict:
    return {"actor": torch.optim.Adam(agent.actor.parameters(), lr=learning_rate),
            "critic": torch.optim.Adam((*agent.q1.parameters(), *agent.q2.parameters()), lr=learning_rate),
            "alpha": torch.optim.Adam((agent.log_alpha,), lr=learning_rate)}


def _map(value, fn):
    if isinstance(value, Mapping):
        return {k: _map(v, fn) for k, v in value.items()}
    return fn(value)


def _zip_map(a, b, fn):
    if isinstance(a, Mapping):
        return {k: _zip_map(a[k], b[k], fn) for k in a}
    return fn(a, b)


class ScenarioReplayBuffer:
    """Bounded device-resident replay, sampled evenly across its scenarios.

    ``add_batch(batch, scenario)`` takes a dict with ``obs`` (tensor or dict of
    tensors), ``mask``, ``action``, ``reward``, ``next_obs``, ``next_mask``,
    ``done`` (leading dimension = rows); ``sample(batch_size, device)`` draws a
    scenario uniformly among those present, then a row of that scenario.
    """

    FIELDS = ("obs", "mask", "action", "reward", "next_obs", "next_mask", "done")

    def __init__(self, capacity: int, device=None):
        if type(capacity) is not int or capacity < 1:
            raise ValueError("replay capacity must be positive")
        self.capacity = capacity
        self.device = None if device is None else torch.device(device)
        self.store = None
        self.scenario_ids: dict[str, int] = {}
        self.scen = None
        self.position = 0
        self.size = 0

    def __len__(self) -> int:
        return self.size

    def _allocate(self, batch: dict) -> None:
        dev = self.device or batch["action"].device
        self.device = dev
        self.store = {k: _map(batch[k], lambda t: torch.zeros((self.capacity, *t.shape[1:]), dtype=t.dtype,
                                                               device=dev)) for k in self.FIELDS}
        self.scen = torch.full((self.capacity,), -1, dtype=torch.long, device=dev)

    def add_batch(self, batch: dict, scenario: str) -> None:
        rows = int(batch["action"].shape[0])
        if rows == 0:
            return
        if self.store is None:
            self._allocate(batch)
        sid = self.scenario_ids.setdefault(str(scenario), len(self.scenario_ids))
        if rows > self.capacity:  # only the newest `capacity` rows survive
            batch = {k: _map(batch[k], lambda t: t[-self.capacity:]) for k in self.FIELDS}
            rows = self.capacity
        idx = (self.position + torch.arange(rows, device=self.device)) % self.capacity
        for k in self.FIELDS:
            _zip_map(self.store[k], batch[k], lambda dst, src: dst.index_copy_(0, idx, src.to(dst.device, dst.dtype)))
        self.scen.index_fill_(0, idx, sid)
        self.position = (self.position + rows) % self.capacity
        self.size = min(self.size + rows, self.capacity)

    def sample(self, batch_size: int, device=None, generator: torch.Generator | None = None) -> dict:
        if type(batch_size) is not int or batch_size < 1 or self.size < batch_size:
            raise ValueError("replay does not contain a full training batch")
        present = torch.unique(self.scen[self.scen >= 0])
        pick = present[torch.randint(len(present), (batch_size,), device=self.device, generator=generator)]
        # a uniformly random row of each chosen scenario: rank among that scenario's rows
        order = torch.argsort(self.scen * self.capacity + torch.arange(self.capacity, device=self.device))
        counts = torch.bincount(self.scen.clamp_min(0), weights=(self.scen >= 0).float(),
                                minlength=int(present.max()) + 1).long()
        starts = torch.cumsum(counts, 0) - counts
        empty = int((self.scen < 0).sum())
        rank = (torch.rand(batch_size, device=self.device, generator=generator) * counts[pick]).long()
        rows = order[empty + starts[pick] + rank.clamp_max(counts[pick] - 1)]
        out = {k: _map(self.store[k], lambda t: t.index_select(0, rows)) for k in self.FIELDS}
        out["action"] = out["action"].long()
        out["reward"] = out["reward"].float()
        out["done"] = out["done"].float()
        if device is not None:
            out = {k: _map(v, lambda t: t.to(device, non_blocking=True)) for k, v in out.items()}
        return out

    def state_dict(self) -> dict:
        return {"capacity": self.capacity, "store": self.store, "scen": self.scen,
                "scenario_ids": dict(self.scenario_ids), "position": self.position, "size": self.size}

    def load_state_dict(self, state: dict) -> None:
        if not isinstance(state, dict) or state.get("capacity") != self.capacity:
            raise ValueError("incompatible SAC replay state")
        if not (0 <= state["position"] < self.capacity and 0 <= state["size"] <= self.capacity):
            raise ValueError("invalid SAC replay state")
        self.store, self.scen = state["store"], state["scen"]
        self.scenario_ids = dict(state["scenario_ids"])
        self.position, self.size = int(state["position"]), int(state["size"])
        if self.scen is not None:
            self.device = self.scen.device


def sac_update(agent: DiscreteSAC, optimizers: dict, batch: dict, *, gamma: float, tau: float,
               target_entropy_fraction: float) -> dict:
    """One critic, actor and temperature step plus the Polyak target update."""
    logits_next, _ = _logits_value(agent.actor, batch["next_obs"])
    p_next, logp_next, _ = masked_distribution(logits_next, batch["next_mask"])
    with torch.no_grad():
        q_next = torch.minimum(agent.target_q1(batch["next_obs"]), agent.target_q2(batch["next_obs"]))
        v_next = (p_next * (q_next - agent.alpha * logp_next)).sum(-1)
        target = batch["reward"] + gamma * (1. - batch["done"]) * v_next
    a = batch["action"][:, None]
    q1 = agent.q1(batch["obs"]).gather(-1, a).squeeze(-1)
    q2 = agent.q2(batch["obs"]).gather(-1, a).squeeze(-1)
    critic_loss = .5 * ((q1 - target).square().mean() + (q2 - target).square().mean())
    optimizers["critic"].zero_grad(set_to_none=True)
    critic_loss.backward()
    optimizers["critic"].step()

    logits, _ = _logits_value(agent.actor, batch["obs"])
    probs, logp, valid = masked_distribution(logits, batch["mask"])
    with torch.no_grad():
        q_min = torch.minimum(agent.q1(batch["obs"]), agent.q2(batch["obs"]))
    alpha = agent.alpha.detach()
    actor_loss = (probs * (alpha * logp - q_min)).sum(-1).mean()
    optimizers["actor"].zero_grad(set_to_none=True)
    actor_loss.backward()
    optimizers["actor"].step()

    entropy = -(probs * logp).sum(-1).detach()
    target_entropy = target_entropy_fraction * valid.sum(-1).float().log()
    alpha_loss = (agent.log_alpha * (entropy - target_entropy)).mean()
    optimizers["alpha"].zero_grad(set_to_none=True)
    alpha_loss.backward()
    optimizers["alpha"].step()

    with torch.no_grad():
        for tgt, src in ((agent.target_q1, agent.q1), (agent.target_q2, agent.q2)):
            for pt, ps in zip(tgt.parameters(), src.parameters()):
                pt.lerp_(ps, tau)
    return {"actor_loss": actor_loss.detach(), "critic_loss": critic_loss.detach(),
            "alpha_loss": alpha_loss.detach(), "alpha": agent.alpha.detach(),
            "entropy": entropy.mean(), "valid_action_count": valid.sum(-1).float().mean()}
