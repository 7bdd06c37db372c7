"""Policy networks.

``build_policy(network, obs_dim, action_dim, action_kind)`` returns a module
with the ActorCritic interface (``forward`` -> (logits|mean, log_std, value),
``sample``, ``score``). Networks:

* ``mlp``     the reference ActorCritic, 2 x 128 tanh (35,337 params at 137->8)
* ``mlp256``  2 x 256 tanh
* further architectures are registered by ``autodrive_b200.models.zoo``
"""
from __future__ import annotations

from .actor_critic import ActorCritic, DDPScore  # noqa: F401

_REGISTRY = {}


def register(name):
    def deco(fn):
        _REGISTRY[name] = fn
        return fn
    return deco


@register("mlp")
def _mlp(obs_dim, action_dim, action_kind):
    return ActorCritic(obs_dim, action_dim, action_kind, hidden=128, layers=2)


@register("mlp256")
def _mlp256(obs_dim, action_dim, action_kind):
    return ActorCritic(obs_dim, action_dim, action_kind, hidden=256, layers=2)


def build_policy(network: str, obs_dim: int, action_dim: int, action_kind: str):
    try:
        from . import zoo  # noqa: F401  (registers the larger architectures)
    except ImportError:
        pass
    if network not in _REGISTRY:
        raise ValueError(f"unknown network {network!r}; choose from {sorted(_REGISTRY)}")
    return _REGISTRY[network](obs_dim, action_dim, action_kind)


def available_networks():
    try:
        from . import zoo  # noqa: F401
    except ImportError:
        pass
    return sorted(_REGISTRY)
