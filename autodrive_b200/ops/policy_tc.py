"""Tensor-core (tcgen05) execution of the 2 x 128 tanh actor-critic.

``TensorCorePolicy`` drives the fused kernels of ``csrc/policy_tc.cu`` for an
``ActorCritic`` whose parameters live in a ``FlatParameters`` buffer:

* ``pack()``            fp32 master weights -> bf16 UMMA images (one launch);
* ``act(obs)``          forward + action mask + categorical sample + log-prob +
                        value in one launch (reference: ``ActorCritic.sample``,
                        frc_defense/tensor_training_runtime.py:63-71);
* ``train_minibatch``   PPO loss gradient for one minibatch gathered by index:
                        advantage statistics, fused forward+backward, partial-
                        gradient reduction (+ L2 on weight matrices) -> the flat
                        gradient buffer; three launches
                        (frc_defense/tensor_training_ppo.py:403-430).

Matmul operands are bf16 with fp32 accumulation in tensor memory; biases,
activations, heads, softmax and the loss run in fp32. Only categorical
policies with the reference trunk (2 x 128 tanh) qualify; ``supported()``
says whether a model does.
"""
from __future__ import annotations

import math

import torch

from .ext import require_extension

_L2_NAMES = ("trunk.0.weight", "trunk.2.weight", "actor.weight", "critic.weight")
_ORDER = ("trunk.0.weight", "trunk.0.bias", "trunk.2.weight", "trunk.2.bias",
          "actor.weight", "actor.bias", "critic.weight", "critic.bias")


class PolicyKernelError(RuntimeError):
    pass


def supported(model) -> bool:
    try:
        trunk = model.trunk
        return (getattr(model, "action_kind", None) == "categorical" and len(trunk) == 4
                and trunk[0].out_features == 128 and trunk[2].in_features == 128
                and trunk[2].out_features == 128 and isinstance(trunk[1], torch.nn.Tanh)
                and isinstance(trunk[3], torch.nn.Tanh) and model.obs_dim <= 191
                and 1 <= model.action_dim <= 9)
    except AttributeError:
        return False


class TensorCorePolicy:
    def __init__(self, model, flat, seed: int | None = None):
        if not supported(model):
            raise ValueError("the tensor-core policy needs a categorical 2 x 128 tanh ActorCritic "
                             "with obs_dim <= 191 and action_dim <= 9")
        self.ext = require_extension()
        self.model, self.flat = model, flat
        self.device = flat.flat.device
        if self.device.type != "cuda":
            raise ValueError("the tensor-core policy runs on CUDA devices only")
        self.obs_dim, self.action_dim = model.obs_dim, model.action_dim
        offset_of = {}
        by_id = {id(p): o for p, (o, _) in zip(flat.params, flat.slices)}
        for name, p in model.named_parameters():
            if id(p) in by_id:
                offset_of[name] = by_id[id(p)]
        missing = [n for n in _ORDER if n not in offset_of]
        if missing:
            raise ValueError(f"parameters missing from the flat buffer: {missing}")
        self.offsets = [int(offset_of[n]) for n in _ORDER]
        if self.offsets[2] % 4:
            raise ValueError("trunk.2.weight must start on a 16-byte boundary of the flat buffer")
        sizes = {n: p.numel() for n, p in model.named_parameters()}
        self.l2_ranges = []
        for n in _L2_NAMES:
            self.l2_ranges += [int(offset_of[n]), int(sizes[n])]
        self.images = torch.zeros(int(self.ext.POLICY_TC_IMAGE_ELEMS), dtype=torch.bfloat16, device=self.device)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.adv_stats = torch.zeros(3, dtype=torch.float64, device=self.device)
        self.rows = int(self.ext.POLICY_TC_ROWS)
        self.pstride = (flat.flat.numel() + 3) // 4 * 4
        self._partials = None
        if seed is None:
            seed = int(torch.randint(0, 2 ** 62, (1,)).item())
        self.seed = int(seed)
        self.counter = 0
        self.version = -1
        self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._status_event = None

    # -- weights --------------------------------------------------------------------
    def pack(self, version: int | None = None) -> None:
        self.ext.policy_pack(self.flat.flat, self.offsets, self.obs_dim, self.images)
        self.version = -1 if version is None else int(version)

    def ensure_packed(self, version: int) -> None:
        if self.version != version:
            self.pack(version)

    # -- status -----------------------------------------------------------------------
    def _post_status(self) -> None:
        self._status_host.copy_(self.status, non_blocking=True)
        if self._status_event is None:
            self._status_event = torch.cuda.Event()
        self._status_event.record()

    def check(self) -> None:
        """Raise if an earlier launch gave up waiting on its tensor cores."""
        if self._status_event is not None:
            self._status_event.synchronize()
            code = int(self._status_host[0])
            if code:
                raise PolicyKernelError(f"policy kernel wait expired (status {code}); results are invalid")

    # -- forward ------------------------------------------------------------------------
    def act(self, obs: torch.Tensor, deterministic: bool = False, value_only: bool = False):
        obs = obs.contiguous().float()
        n = obs.shape[0]
        action = torch.empty(n, dtype=torch.long, device=self.device)
        logp = torch.empty(n, device=self.device)
        value = torch.empty(n, device=self.device)
        mask = None if value_only else torch.empty((n, self.action_dim), dtype=torch.bool, device=self.device)
        mode = 0 if value_only else (2 if deterministic else 1)
        self.ext.policy_act(obs, self.action_dim, self.images, self.flat.flat, self.offsets, mode, self.seed,
                            self.counter, action, logp, value, mask, self.status)
        self.counter += 1
        if value_only:
            return value
        return action, logp, value, mask

    # -- training -------------------------------------------------------------------------
    def partials(self, rows: int) -> torch.Tensor:
        nblk = max(1, math.ceil(rows / self.rows))
        if self._partials is None or self._partials.shape[0] < nblk:
            self._partials = torch.empty((nblk, self.pstride), device=self.device)
        return self._partials

    def minibatch_adv_stats(self, adv: torch.Tensor, batches) -> torch.Tensor:
        """Local (sum, sum of squares, count) of the advantages of every
        minibatch in `batches`, one row each (float64 [len(batches), 3])."""
        out = torch.empty((len(batches), 3), dtype=torch.float64, device=adv.device)
        for k, idx in enumerate(batches):
            self.ext.policy_adv_stats(adv, idx, int(idx.numel()), out[k])
        return out

    def train_minibatch(self, batch: dict, idx: torch.Tensor, ent_coef: torch.Tensor, clip: float,
                        value_coef: float, l2_coef: float, loss_stats: torch.Tensor, all_reduce=None,
                        adv_stats: torch.Tensor | None = None) -> None:
        """Write the minibatch's PPO gradient into ``flat.grad`` (overwrites
        it). `adv_stats` supplies the minibatch's already reduced advantage
        statistics; otherwise they are computed (and all-reduced) here."""
        b = int(idx.numel())
        if adv_stats is not None:
            self.adv_stats.copy_(adv_stats)
        else:
            self.ext.policy_adv_stats(batch["adv"], idx, b, self.adv_stats)
            if all_reduce is not None:
                all_reduce(self.adv_stats)
        part = self.partials(b)
        self.ext.policy_train(batch["obs"], idx, self.action_dim, self.images, self.flat.flat, self.offsets,
                              batch["actions"], batch.get("mask"), batch["logp"], batch["adv"], batch["returns"],
                              self.adv_stats, ent_coef, float(clip), float(value_coef), part, loss_stats,
                              self.status)
        self.ext.policy_grad_reduce(part, math.ceil(b / self.rows), self.flat.flat, self.flat.grad,
                                    float(l2_coef), self.l2_ranges)
