"""LayerNorm for bf16 activations on a fused sm_100a kernel
(``csrc/layernorm.cu``): fp32 statistics and affine parameters, a bf16
result, one read and one write of each element in the forward and one write
of the input gradient in the backward.

``FusedLayerNorm`` is a drop-in ``nn.LayerNorm`` (same parameters and
state-dict keys). On CUDA, for a bf16 input or inside a bf16 autocast region,
and a normalised width of 64, 128, 256 or 512, it runs the fused kernel and
returns bf16 (autocast's own policy would run LayerNorm in fp32 and return
fp32, which the next bf16 layer casts back). Everywhere else it is
``nn.LayerNorm``.
"""
from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from ..utils import launches
from .ext import require_extension

WIDTHS = (64, 128, 256, 512)


class _LayerNormBf16Fn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, bias, eps):
        d = x.shape[-1]
        x2 = x.reshape(-1, d).to(torch.bfloat16).contiguous()
        launches.add(1)
        y, mean, rstd = require_extension().layer_norm_bf16_fwd(x2, weight.detach().float().contiguous(),
                                                                bias.detach().float().contiguous(), float(eps))
        ctx.save_for_backward(x2, weight, mean, rstd)
        ctx.in_shape, ctx.in_dtype = x.shape, x.dtype
        return y.reshape(x.shape)

    @staticmethod
    def backward(ctx, gy):
        x2, weight, mean, rstd = ctx.saved_tensors
        d = x2.shape[-1]
        g = gy.reshape(-1, d).to(torch.bfloat16).contiguous()
        launches.add(1)
        dx, dw, db = require_extension().layer_norm_bf16_bwd(g, x2, weight.detach().float().contiguous(), mean, rstd)
        dx = dx.reshape(ctx.in_shape)
        return (dx if ctx.in_dtype == torch.bfloat16 else dx.to(ctx.in_dtype)), dw, db, None


def layer_norm_bf16(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    """LayerNorm over the last dimension of `x` on the fused kernel (bf16 result)."""
    return _LayerNormBf16Fn.apply(x, weight, bias, eps)


class FusedLayerNorm(nn.LayerNorm):
    def forward(self, x: torch.Tensor) -> torch.Tensor:
        bf16 = x.dtype == torch.bfloat16 or (torch.is_autocast_enabled("cuda")
                                             and torch.get_autocast_dtype("cuda") == torch.bfloat16)
        if (x.is_cuda and bf16 and self.elementwise_affine and self.bias is not None
                and len(self.normalized_shape) == 1 and self.normalized_shape[0] in WIDTHS):
            return _LayerNormBf16Fn.apply(x, self.weight, self.bias, self.eps)
        return F.layer_norm(x, self.normalized_shape, self.weight, self.bias, self.eps)
