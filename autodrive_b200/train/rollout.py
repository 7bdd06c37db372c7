"""Agent-batch adapters over the environments, GAE and held-action stepping.

PPO sees a flat batch of agents: the two-robot env has one learner per world;
the 3v3 env has one agent per neural-controlled robot slot. Strategic
decisions hold for ``ticks`` physics ticks (12 or 13 at 4 Hz, from a phase
accumulator: frc_defense/tensor_training_ppo.py:275-278).
"""
from __future__ import annotations

import torch

from ..ops import require_extension
from ..utils import launches


def gae_advantages(rewards, dones, truncated, values, next_values, gamma: float, gae_lambda: float,
                   stats: torch.Tensor | None = None) -> torch.Tensor:
    """Generalised advantage estimation. Truncations bootstrap; terminations do not.

    Runs the native reverse scan (sm_100a kernel on CUDA tensors, host loop on
    CPU) and, when ``stats`` (float64 [3]) is given, leaves sum(adv),
    sum(adv^2) and the count in it for advantage normalisation.
    """
    ext = require_extension()
    adv = torch.empty_like(rewards)
    if stats is None:
        stats = torch.zeros(3, dtype=torch.float64, device=rewards.device)
    launches.add(1)
    ext.gae(rewards.contiguous().float(), dones.contiguous().to(torch.uint8),
            truncated.contiguous().to(torch.uint8), values.contiguous().float(),
            next_values.contiguous().float(), adv, float(gamma), float(gae_lambda), stats)
    return adv


def gae_reference(rewards, dones, truncated, values, next_values, gamma, gae_lambda):
    """Plain PyTorch reverse scan (numerics oracle for the native kernel)."""
    adv = torch.zeros_like(rewards)
    last = torch.zeros_like(rewards[0])
    for t in reversed(range(rewards.shape[0])):
        nonterminal = (~dones[t]).float()
        delta = rewards[t] + gamma * next_values[t] * nonterminal - values[t]
        cont = (~(dones[t] | truncated[t])).float()
        last = delta + gamma * gae_lambda * cont * last
        adv[t] = last
    return adv


def trim_entities(inp: dict) -> dict:
    """Drop FUEL-track tokens past the highest live track slot of the batch
    (anonymous tracks fill slots from 0), rounded up to a multiple of 8, and
    keep the four robot tokens: attention cost follows the tracks held."""
    ent, mask = inp["entities"], inp["entity_mask"]
    P = ent.shape[1] - 4
    live = mask[:, :P].any(0)
    k = int(live.nonzero().max()) + 1 if bool(live.any()) else 0
    k = min(P, (k + 7) // 8 * 8)
    if k == P:
        return inp
    keep = torch.cat((torch.arange(k, device=ent.device), torch.arange(P, P + 4, device=ent.device)))
    return {**inp, "entities": ent[:, keep], "entity_mask": mask[:, keep]}


def stack_inputs(rows: list[dict]) -> dict:
    """Concatenate per-decision perception dictionaries along the batch,
    zero-padding the FUEL-track tokens (invalid, masked) to the longest."""
    if "entities" in rows[0]:
        kmax = max(r["entities"].shape[1] for r in rows)
        padded = []
        for r in rows:
            ent, mask = r["entities"], r["entity_mask"]
            extra = kmax - ent.shape[1]
            if extra:
                ent = torch.cat((ent[:, :-4], ent.new_zeros((ent.shape[0], extra, ent.shape[2])), ent[:, -4:]), 1)
                mask = torch.cat((mask[:, :-4], mask.new_zeros((mask.shape[0], extra)), mask[:, -4:]), 1)
            padded.append({**r, "entities": ent, "entity_mask": mask})
        rows = padded
    return {k: torch.cat([r[k] for r in rows]) for k in rows[0]}


class StrategicClock:
    """Ticks per strategic decision at `rate_hz` with a 50 Hz physics tick."""

    def __init__(self, rate_hz: float = 4.):
        if not 2. <= rate_hz <= 5.:
            raise ValueError("strategic_rate_hz must be between 2 and 5")
        self.rate_hz = rate_hz
        self.phase = 0.

    def next(self) -> int:
        self.phase += 50. / self.rate_hz
        ticks = max(1, int(self.phase))
        self.phase -= ticks
        return ticks


class DefenseAgents:
    """One learner per world of a TensorDefenseEnv."""

    def __init__(self, env):
        self.env = env
        self.n_agents = env.n
        self.obs_dim, self.action_dim, self.action_kind = env.obs_dim, env.action_dim, env.action_kind
        self.horizon = env.horizon
        self.drivetrain_config = env.drivetrain_config

    def reset(self) -> torch.Tensor:
        obs, _ = self.env.reset()
        return obs

    def act(self, action: torch.Tensor, ticks: int, remaining: int):
        reward = torch.zeros(self.n_agents, device=self.env.device)
        done = torch.zeros(self.n_agents, dtype=torch.bool, device=self.env.device)
        truncated = torch.zeros_like(done)
        obs = None
        for k in range(ticks):
            last = k == ticks - 1 or k + 1 == remaining
            obs, r, d, tr, _ = self.env.step(action, _return_info=False, _capture_observation=last)
            reward += r
            done |= d
            truncated |= tr
            if k + 1 == remaining:
                break
        return obs, reward, done, truncated

    def reset_done(self, mask: torch.Tensor) -> torch.Tensor:
        return self.env.reset_done(mask)

    def score_counts(self):
        return self.env.fuel_score_count, self.env.fuel_acquisition_count


class ThreeVsThreeAgents:
    """Neural-controlled slots of a TensorThreeVsThreeEnv as a flat agent batch."""

    def __init__(self, env, observe_every_tick: bool = False):
        self.env = env
        self.observe_every_tick = bool(observe_every_tick)
        self.slots = [i for i, m in enumerate(env.control_modes) if m == "nn"]
        if not self.slots:
            raise ValueError("the 3v3 environment has no neural-controlled robot slots")
        self.slot_index = torch.tensor(self.slots, device=env.device)
        self.n_agents = env.n * len(self.slots)
        self.obs_dim, self.action_dim, self.action_kind = 137, 8, "categorical"
        self.horizon = env.horizon
        self.drivetrain_config = env.drivetrain_config
        self._full = torch.full((env.n, 6), 7, dtype=torch.int32, device=env.device)
        self.perception = None
        self.perception_keys = ()

    def use_perception(self, field_shape=(32, 64), keys=("scalars", "field", "entities", "entity_mask")):
        """Observations become perception dictionaries (``PerceptionInputs``)
        holding only `keys`, for the architecture-zoo networks."""
        from ..models.perception import PerceptionInputs
        self.perception = PerceptionInputs(self.env, self.slots, field_shape=field_shape)
        self.perception_keys = tuple(keys)

    def _agent_obs(self):
        if self.perception is not None:
            inp = self.perception()
            inp = {k: inp[k] for k in self.perception_keys}
            return trim_entities(inp) if "entities" in inp else inp
        return self.env.ws["obs"].index_select(1, self.slot_index).reshape(self.n_agents, 137)

    def reset(self) -> torch.Tensor:
        self.env.reset()
        return self._agent_obs()

    def act(self, action: torch.Tensor, ticks: int, remaining: int):
        self._full.index_copy_(1, self.slot_index,
                               action.reshape(self.env.n, len(self.slots)).to(torch.int32))
        ticks = min(ticks, max(1, remaining))
        _, reward, truncated = self.env.step_held(self._full, ticks, observe_every_tick=self.observe_every_tick)
        reward = reward.index_select(1, self.slot_index).reshape(self.n_agents)
        truncated = truncated[:, None].expand(-1, len(self.slots)).reshape(self.n_agents)
        done = torch.zeros_like(truncated)
        return self._agent_obs(), reward, done, truncated

    def reset_done(self, mask: torch.Tensor) -> torch.Tensor:
        world = mask.reshape(self.env.n, len(self.slots)).any(-1)
        self.env.reset_done(world)
        return self._agent_obs()

    def score_counts(self):
        return self.env.fuel_score_count, self.env.fuel_acquisition_count
