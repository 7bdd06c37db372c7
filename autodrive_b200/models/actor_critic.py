"""Actor-critic policy with the reference's state-dict layout.

Parameter names match frc_defense/tensor_training_runtime.py:40-94
(``trunk.0``, ``trunk.2``, ``actor``, ``critic``, ``log_std``) so checkpoints
load in either framework. ``hidden`` and ``layers`` widen or deepen the trunk
(the reference default is 2 x 128 tanh).
"""
from __future__ import annotations

import torch
from torch import nn
from torch.distributions import Normal

OBS_DIM = 35
ACTION_DIM = 3
STRATEGIC_OBS_DIM = 137
STRATEGIC_ACTION_DIM = 8


class ActorCritic(nn.Module):
    def __init__(self, obs_dim: int = OBS_DIM, action_dim: int = ACTION_DIM,
                 action_kind: str = "continuous", hidden: int = 128, layers: int = 2):
        super().__init__()
        if action_kind not in ("continuous", "categorical"):
            raise ValueError("action_kind must be continuous or categorical")
        self.action_kind = action_kind
        self.obs_dim, self.action_dim, self.hidden = obs_dim, action_dim, hidden
        mods: list[nn.Module] = []
        width = obs_dim
        for _ in range(layers):
            mods += [nn.Linear(width, hidden), nn.Tanh()]
            width = hidden
        self.trunk = nn.Sequential(*mods)
        self.actor = nn.Linear(hidden, action_dim)
        self.critic = nn.Linear(hidden, 1)
        if action_kind == "continuous":
            self.log_std = nn.Parameter(torch.zeros(action_dim))

    def forward(self, obs: torch.Tensor):
        features = self.trunk(obs)
        logits_or_mean = self.actor(features)
        scale = None if self.action_kind == "categorical" else self.log_std.expand_as(logits_or_mean)
        return logits_or_mean, scale, self.critic(features).squeeze(-1)

    def _masked(self, logits, action_mask):
        if action_mask is None:
            return logits
        return logits.masked_fill(~action_mask.bool(), torch.finfo(logits.dtype).min)

    def sample(self, obs: torch.Tensor, deterministic: bool = False, action_mask=None):
        mean, log_std, value = self(obs)
        if self.action_kind == "categorical":
            logits = self._masked(mean, action_mask)
            dist = torch.distributions.Categorical(logits=logits)
            action = logits.argmax(-1) if deterministic else dist.sample()
            return action, dist.log_prob(action), value
        dist = Normal(mean, log_std.exp())
        latent = mean if deterministic else dist.rsample()
        action = torch.tanh(latent)
        log_prob = dist.log_prob(latent).sum(-1) - torch.log(1 - action.square() + 1e-6).sum(-1)
        return action, log_prob, value

    def score(self, obs: torch.Tensor, actions: torch.Tensor, action_mask=None):
        mean, log_std, value = self(obs)
        if self.action_kind == "categorical":
            logits = self._masked(mean, action_mask)
            dist = torch.distributions.Categorical(logits=logits)
            actions = actions.to(torch.long).reshape(-1)
            return dist.log_prob(actions), dist.entropy(), value, logits
        actions = actions.clamp(-0.999999, 0.999999)
        latent = torch.atanh(actions)
        dist = Normal(mean, log_std.exp())
        log_prob = dist.log_prob(latent).sum(-1) - torch.log(1 - actions.square() + 1e-6).sum(-1)
        return log_prob, dist.entropy().sum(-1), value, mean


class DDPScore(nn.Module):
    """Expose ``ActorCritic.score`` through a module forward (for DDP wrappers)."""

    def __init__(self, policy: nn.Module):
        super().__init__()
        self.policy = policy

    def forward(self, obs, actions, action_mask=None):
        return self.policy.score(obs, actions, action_mask)
