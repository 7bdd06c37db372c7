"""PPO step for the perception-input policy zoo on the 3v3 environment.

One step = a rollout of `decisions` strategic decisions (held 12 or 13 ticks,
4 Hz) for the three learned defenders of every world, GAE, then PPO epochs x
minibatches on a ``PerceptionActorCritic`` (e.g. ``entity_attention_256``:
two pre-LN attention blocks, d = 256, 4 heads, ~4M parameters). Forward and
backward run under bf16 autocast (linear layers on the tcgen05 GEMM kernel,
fp32 accumulation) with fp32 master weights; gradients are averaged, clipped
and applied by the same fused Adam / peer all-reduce path as the MLP trainer.
"""
from __future__ import annotations

import torch

from ..models.perception import PerceptionInputs
from ..models.zoo import PerceptionActorCritic, parameter_count
from ..parallel.grad_sync import GradientSync, sync_parameters
from ..train.optim import FusedAdam

LEARNED = (3, 4, 5)


class ZooPPO:
    def __init__(self, env, network: str, world: int, *, lr: float = 3e-4, gamma: float = .999,
                 lam: float = .95, clip: float = .2, epochs: int = 4, minibatches: int = 8,
                 grad_backend: str = "auto", entropy: float = .01):
        self.env, self.world = env, world
        dev = env.device
        self.model = PerceptionActorCritic(network, tensor_cores=dev.type == "cuda").to(dev)
        sync_parameters(self.model, world)
        self.params = parameter_count(self.model)
        self.inputs = PerceptionInputs(env, LEARNED, field_shape=self.model.field_shape)
        self.opt = FusedAdam(self.model, lr=lr, eps=1e-5, max_grad_norm=.5)
        self.sync = GradientSync(self.opt, world, grad_backend)
        self.gamma, self.lam, self.clip = gamma, lam, clip
        self.epochs, self.minibatches, self.entropy = epochs, minibatches, entropy
        self.actions = torch.full((env.n, 6), 7, dtype=torch.int32, device=dev)
        self.tick_parity = 0

    def _policy_inputs(self):
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=self.env.device.type == "cuda"):
            inp = self.inputs()
        return self._trim(inp)

    @staticmethod
    def _trim(inp: dict) -> dict:
        """Drop FUEL-track tokens past the highest live slot of the batch
        (anonymous tracks fill slots from 0), keeping the four robot tokens:
        the attention cost follows the tracks actually held, not the slot count."""
        ent, mask = inp["entities"], inp["entity_mask"]
        P = ent.shape[1] - 4
        live = mask[:, :P].any(0)
        k = int(live.nonzero().max()) + 1 if bool(live.any()) else 0
        k = min(P, (k + 7) // 8 * 8)
        keep = torch.cat((torch.arange(k, device=ent.device), torch.arange(P, P + 4, device=ent.device)))
        return {**inp, "entities": ent[:, keep], "entity_mask": mask[:, keep]}

    @staticmethod
    def _pad(inp: dict, k: int) -> dict:
        ent, mask = inp["entities"], inp["entity_mask"]
        have = ent.shape[1] - 4
        if have == k:
            return inp
        pad_e = ent.new_zeros((ent.shape[0], k - have, ent.shape[2]))
        pad_m = mask.new_zeros((mask.shape[0], k - have))
        return {**inp, "entities": torch.cat((ent[:, :have], pad_e, ent[:, have:]), 1),
                "entity_mask": torch.cat((mask[:, :have], pad_m, mask[:, have:]), 1)}

    def rollout(self, decisions: int):
        rows, acts, logps, vals, rews = [], [], [], [], []
        ticks = 0
        with torch.no_grad():
            for _ in range(decisions):
                inp = self._policy_inputs()
                with torch.autocast("cuda", dtype=torch.bfloat16, enabled=self.env.device.type == "cuda"):
                    act, logp, val = self.model.sample(inp)
                self.actions[:, 3:] = act.reshape(self.env.n, 3).to(torch.int32)
                held = 12 + self.tick_parity          # 12 / 13 ticks: 4 Hz at 50 Hz
                self.tick_parity ^= 1
                _, reward, _ = self.env.step_held(self.actions, held)
                ticks += held
                rows.append(inp)
                acts.append(act)
                logps.append(logp.float())
                vals.append(val.float().reshape(-1))
                rews.append(reward[:, 3:].reshape(-1).float())
            last = self.model(self._policy_inputs())[2].float().reshape(-1)
        return rows, acts, logps, vals, rews, last, ticks

    def update(self, rows, acts, logps, vals, rews, last) -> dict:
        T = len(rows)
        vals_t, rews_t = torch.stack(vals), torch.stack(rews)
        adv = torch.zeros_like(rews_t)
        gae = torch.zeros_like(last)
        nxt = last
        for t in reversed(range(T)):            # matches run past the rollout: bootstrap, no terminal
            delta = rews_t[t] + self.gamma * nxt - vals_t[t]
            gae = delta + self.gamma * self.lam * gae
            adv[t] = gae
            nxt = vals_t[t]
        ret = (adv + vals_t).reshape(-1)
        adv = adv.reshape(-1)
        kmax = max(r["entities"].shape[1] - 4 for r in rows)
        rows = [self._pad(r, kmax) for r in rows]
        flat = {k: torch.cat([r[k] for r in rows]) for k in rows[0]}
        a_f, lp_f = torch.cat(acts), torch.cat(logps)
        n = a_f.numel()
        mb = max(1, n // self.minibatches)
        kl_sum = torch.zeros((), device=a_f.device)
        ent_sum = torch.zeros((), device=a_f.device)
        batches = 0
        for _ in range(self.epochs):
            for idx in torch.randperm(n, device=a_f.device).split(mb):
                sub = {k: v[idx] for k, v in flat.items()}
                with torch.autocast("cuda", dtype=torch.bfloat16, enabled=a_f.device.type == "cuda"):
                    logp, ent, v, _ = self.model.score(sub, a_f[idx])
                logp, ent, v = logp.float(), ent.float(), v.float().reshape(-1)
                a = adv[idx]
                a = (a - a.mean()) / (a.std(unbiased=False) + 1e-8)
                ratio = (logp - lp_f[idx]).exp()
                pg = torch.maximum(-a * ratio, -a * ratio.clamp(1 - self.clip, 1 + self.clip)).mean()
                loss = pg + .5 * (v - ret[idx]).square().mean() - self.entropy * ent.mean()
                self.opt.zero_grad()
                loss.backward()
                self.sync.step()
                kl_sum += (lp_f[idx] - logp).mean().detach()
                ent_sum += ent.mean().detach()
                batches += 1
        return {"samples": n, "batches": batches, "approx_kl_sum": kl_sum, "entropy_sum": ent_sum,
                "mean_reward": rews_t.mean()}

    def step(self, decisions: int, events: list | None = None) -> tuple[int, dict]:
        """One PPO iteration; `events` (a list) receives CUDA events around the
        rollout and the update for a device-time breakdown."""
        def mark():
            if events is not None:
                ev = torch.cuda.Event(enable_timing=True)
                ev.record()
                events.append(ev)
        mark()
        rows, acts, logps, vals, rews, last, ticks = self.rollout(decisions)
        mark()
        upd = self.update(rows, acts, logps, vals, rews, last)
        mark()
        return ticks, upd
