"""Flat parameter storage and the fused clip + Adam optimizer.

All trainable parameters of a module are re-homed into one contiguous fp32
buffer and their gradients into a second one. The whole update is then two
kernel launches (partial squared norms, then norm -> clip scale -> Adam), and
a data-parallel gradient reduction is one collective over one buffer.
Reference behaviour: ``clip_grad_norm_(max_norm)`` followed by
``torch.optim.Adam(lr, eps=1e-5)`` (frc_defense/tensor_training_ppo.py:80,433-434).
"""
from __future__ import annotations

import torch
from torch import nn

from ..ops import require_extension
from ..utils import launches


class FlatParameters:
    def __init__(self, module: nn.Module):
        params = [p for p in module.parameters() if p.requires_grad]
        if not params:
            raise ValueError("module has no trainable parameters")
        device = params[0].device
        total = sum(p.numel() for p in params)
        self.params = params
        self.flat = torch.empty(total, device=device, dtype=torch.float32)
        self.grad = torch.zeros(total, device=device, dtype=torch.float32)
        offset = 0
        self.slices = []
        for p in params:
            n = p.numel()
            self.flat[offset:offset + n].copy_(p.detach().reshape(-1).float())
            p.data = self.flat[offset:offset + n].view_as(p)
            p.grad = self.grad[offset:offset + n].view_as(p)
            self.slices.append((offset, n))
            offset += n

    def rehome(self, flat: torch.Tensor, grad: torch.Tensor) -> None:
        """Move parameters and gradients into caller-provided flat buffers
        (already holding the parameter values), e.g. peer-visible memory."""
        if flat.numel() != self.flat.numel() or grad.numel() != self.grad.numel():
            raise ValueError("rehome buffers must match the flat parameter count")
        self.flat, self.grad = flat, grad
        for p, (o, n) in zip(self.params, self.slices):
            p.data = self.flat[o:o + n].view_as(p)
            p.grad = self.grad[o:o + n].view_as(p)

    def zero_grad(self) -> None:
        self.grad.zero_()
        # autograd may have replaced a .grad with a fresh tensor; re-bind views
        for p, (o, n) in zip(self.params, self.slices):
            if p.grad is None or p.grad.data_ptr() != self.grad[o:o + n].data_ptr():
                if p.grad is not None:
                    self.grad[o:o + n].copy_(p.grad.reshape(-1))
                p.grad = self.grad[o:o + n].view_as(p)

    def sync_grads(self) -> None:
        """Fold any gradient autograd stored outside the flat buffer back in."""
        for p, (o, n) in zip(self.params, self.slices):
            if p.grad is not None and p.grad.data_ptr() != self.grad[o:o + n].data_ptr():
                self.grad[o:o + n].copy_(p.grad.reshape(-1))
                p.grad = self.grad[o:o + n].view_as(p)


class FusedAdam:
    """Adam with global-norm clipping on a FlatParameters buffer."""

    def __init__(self, module: nn.Module, lr: float = 3e-4, betas=(.9, .999), eps: float = 1e-5,
                 weight_decay: float = 0., max_grad_norm: float = .5):
        self.ext = require_extension()
        self.flat = FlatParameters(module)
        self.lr, self.betas, self.eps = float(lr), betas, float(eps)
        self.weight_decay, self.max_grad_norm = float(weight_decay), float(max_grad_norm)
        dev = self.flat.flat.device
        self.m = torch.zeros_like(self.flat.flat)
        self.v = torch.zeros_like(self.flat.flat)
        self.partial = torch.zeros(int(self.ext.ADAM_NORM_BLOCKS), device=dev)
        self.last_norm = torch.zeros(1, device=dev)
        self.step_count = 0

    @property
    def grad(self) -> torch.Tensor:
        return self.flat.grad

    def zero_grad(self, set_to_none: bool = False) -> None:  # noqa: ARG002 - flat buffers persist
        self.flat.zero_grad()

    def step(self) -> torch.Tensor:
        self.flat.sync_grads()
        self.step_count += 1
        launches.add(2)   # partial sums of squares + clip / Adam
        self.ext.adam_fused(self.flat.flat, self.flat.grad, self.m, self.v, self.partial, self.last_norm,
                            self.step_count, self.lr, self.betas[0], self.betas[1], self.eps,
                            self.weight_decay, self.max_grad_norm)
        return self.last_norm

    def state_dict(self) -> dict:
        return {"m": self.m.detach().cpu(), "v": self.v.detach().cpu(), "step": self.step_count,
                "lr": self.lr, "betas": tuple(self.betas), "eps": self.eps}

    def load_state_dict(self, state: dict) -> None:
        self.m.copy_(state["m"])
        self.v.copy_(state["v"])
        self.step_count = int(state["step"])
