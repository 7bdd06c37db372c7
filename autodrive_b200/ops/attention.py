"""Variable-length multi-head self-attention on the sm_100a tensor cores
(``csrc/attention.cu``), with autograd.

``varlen_attention(qkv, cu, max_len, heads)`` takes the packed projection
qkv [total, 3 * heads * 64] of the valid tokens of all samples back to back
(sample i at rows cu[i]:cu[i+1], last dimension [3][heads][64]) and returns
the attention output [total, heads * 64] in bf16: every token attends to the
tokens of its own sample, softmax scale 1/8. The backward returns d(qkv) in
one bf16 buffer of qkv's layout.

The kernels report timed-out waits through the same device status word as
the tcgen05 GEMM, so ``ops.tc_linear.check_gemm_status`` covers both.
``reference_attention`` is the same operation in plain fp32 PyTorch (the
oracle of the tests).
"""
from __future__ import annotations

import torch
from torch import Tensor

from ..utils import launches
from .ext import require_extension
from .tc_linear import _Status

HEAD_DIM = 64


def supported(qkv: Tensor, heads: int) -> bool:
    """Whether the tensor-core kernels take this projection (CUDA, head dim 64)."""
    return qkv.is_cuda and qkv.dim() == 2 and qkv.shape[1] == 3 * heads * HEAD_DIM


class _TcVarlenAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv: Tensor, cu: Tensor, max_len: int, heads: int) -> Tensor:
        ext = require_extension()
        x = qkv.to(torch.bfloat16).contiguous()
        if x.data_ptr() % 16:
            x = x.clone()
        cu32 = cu.to(device=x.device, dtype=torch.int32).contiguous()
        total = x.shape[0]
        out = torch.empty((total, heads * HEAD_DIM), dtype=torch.bfloat16, device=x.device)
        lse = torch.empty((heads, total), dtype=torch.float32, device=x.device)
        status = _Status.get(x.device)
        ext.attn_fwd(x, cu32, int(max_len), int(heads), out, lse, status)
        launches.add(1)
        _Status.after_launch(x.device)
        ctx.save_for_backward(x, cu32, out, lse)
        ctx.max_len, ctx.heads, ctx.in_dtype = int(max_len), int(heads), qkv.dtype
        return out

    @staticmethod
    def backward(ctx, grad: Tensor):
        x, cu32, out, lse = ctx.saved_tensors
        ext = require_extension()
        g = grad.to(torch.bfloat16).contiguous()
        dqkv = torch.empty_like(x)
        status = _Status.get(x.device)
        ext.attn_bwd(x, cu32, ctx.max_len, ctx.heads, out, g, lse, dqkv, status)
        launches.add(1)
        _Status.after_launch(x.device)
        return dqkv.to(ctx.in_dtype), None, None, None


def varlen_attention(qkv: Tensor, cu: Tensor, max_len: int, heads: int) -> Tensor:
    """Attention within each sample of the packed projection `qkv` (see the
    module docstring); `max_len` is at least the longest sample."""
    if not supported(qkv, heads):
        raise ValueError("varlen_attention needs a CUDA qkv [total, 3 * heads * 64]")
    return _TcVarlenAttention.apply(qkv, cu, max_len, heads)


def reference_attention(qkv: Tensor, cu: Tensor, heads: int) -> Tensor:
    """fp32 PyTorch attention of the same packed layout (test oracle)."""
    x = qkv.float()
    total, d3 = x.shape
    dh = d3 // (3 * heads)
    out = torch.zeros((total, heads * dh), dtype=torch.float32, device=x.device)
    bounds = cu.tolist()
    for i in range(len(bounds) - 1):
        a, b = bounds[i], bounds[i + 1]
        if b <= a:
            continue
        q, k, v = x[a:b].view(b - a, 3, heads, dh).permute(1, 2, 0, 3)   # [heads, L, dh] each
        w = torch.softmax(q @ k.transpose(-1, -2) / dh ** .5, dim=-1)
        out[a:b] = (w @ v).permute(1, 0, 2).reshape(b - a, heads * dh)
    return out
