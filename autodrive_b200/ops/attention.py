"""Variable-length multi-head self-attention on the sm_100a tensor cores
(``csrc/attention.cu``), with autograd.

``varlen_attention(qkv, cu, max_len, heads)`` takes the packed projection
qkv [total, 3 * heads * 64] of the valid tokens of all samples back to back
(sample i at rows cu[i]:cu[i+1], last dimension [3][heads][64]) and returns
the attention output [total, heads * 64] in bf16: every token attends to the
tokens of its own sample, softmax scale 1/8. The backward returns d(qkv) in
one bf16 buffer of qkv's layout.

``varlen_query_attention(q, kv, cu_q, cu_k, max_q, max_k, heads)`` is the
same operation with separate sources: sample i's queries are rows
cu_q[i]:cu_q[i+1] of q [total_q, heads * 64], its keys and values rows
cu_k[i]:cu_k[i+1] of kv [total_k, 2 * heads * 64] (keys, then values). The
entity encoder's last block uses it with one query (the context token) per
sample.

The kernels report timed-out waits through the same device status word as
the tcgen05 GEMM, so ``ops.tc_linear.check_gemm_status`` covers both.
``reference_attention`` and ``reference_query_attention`` are the same
operations in plain fp32 PyTorch (the oracles of the tests).
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


def _bf16_rows(x: Tensor) -> Tensor:
    y = x.to(torch.bfloat16).contiguous()
    return y if y.data_ptr() % 16 == 0 else y.clone()


def _launched(device) -> None:
    launches.add(1)
    _Status.after_launch(device)


class _TcVarlenAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv: Tensor, cu: Tensor, max_len: int, heads: int) -> Tensor:
        ext = require_extension()
        x = _bf16_rows(qkv)
        cu32 = cu.to(device=x.device, dtype=torch.int32).contiguous()
        total, d = x.shape[0], heads * HEAD_DIM
        out = torch.empty((total, d), dtype=torch.bfloat16, device=x.device)
        lse = torch.empty((heads, total), dtype=torch.float32, device=x.device)
        ext.attn_fwd(x, 0, x, d, 2 * d, cu32, cu32, int(max_len), int(heads), out, lse, _Status.get(x.device))
        _launched(x.device)
        ctx.save_for_backward(x, cu32, out, lse)
        ctx.max_len, ctx.heads, ctx.in_dtype = int(max_len), int(heads), qkv.dtype
        return out

    @staticmethod
    def backward(ctx, grad: Tensor):
        x, cu32, out, lse = ctx.saved_tensors
        ext = require_extension()
        d = ctx.heads * HEAD_DIM
        g = grad.to(torch.bfloat16).contiguous()
        dqkv = torch.empty_like(x)
        ext.attn_bwd(x, 0, x, d, 2 * d, cu32, cu32, ctx.max_len, ctx.heads, out, g, lse, dqkv, 0, dqkv, d, 2 * d,
                     _Status.get(x.device))
        _launched(x.device)
        return dqkv.to(ctx.in_dtype), None, None, None


class _TcQueryAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q: Tensor, kv: Tensor, cu_q: Tensor, cu_k: Tensor, max_q: int, max_k: int, heads: int) -> Tensor:
        ext = require_extension()
        qb, kvb = _bf16_rows(q), _bf16_rows(kv)
        cq = cu_q.to(device=qb.device, dtype=torch.int32).contiguous()
        ck = cu_k.to(device=qb.device, dtype=torch.int32).contiguous()
        d = heads * HEAD_DIM
        out = torch.empty((qb.shape[0], d), dtype=torch.bfloat16, device=qb.device)
        lse = torch.empty((heads, qb.shape[0]), dtype=torch.float32, device=qb.device)
        ext.attn_fwd(qb, 0, kvb, 0, d, cq, ck, int(max_q), int(heads), out, lse, _Status.get(qb.device))
        _launched(qb.device)
        ctx.save_for_backward(qb, kvb, cq, ck, out, lse)
        ctx.max_k, ctx.heads, ctx.dtypes = int(max_k), int(heads), (q.dtype, kv.dtype)
        return out

    @staticmethod
    def backward(ctx, grad: Tensor):
        qb, kvb, cq, ck, out, lse = ctx.saved_tensors
        ext = require_extension()
        d = ctx.heads * HEAD_DIM
        g = grad.to(torch.bfloat16).contiguous()
        dq, dkv = torch.empty_like(qb), torch.empty_like(kvb)
        ext.attn_bwd(qb, 0, kvb, 0, d, cq, ck, ctx.max_k, ctx.heads, out, g, lse, dq, 0, dkv, 0, d,
                     _Status.get(qb.device))
        _launched(qb.device)
        return dq.to(ctx.dtypes[0]), dkv.to(ctx.dtypes[1]), None, None, None, None, None


def varlen_attention(qkv: Tensor, cu: Tensor, max_len: int, heads: int) -> Tensor:
    """Attention within each sample of the packed projection `qkv` (see the
    module docstring); `max_len` is at least the longest sample."""
    if not supported(qkv, heads):
        raise ValueError("varlen_attention needs a CUDA qkv [total, 3 * heads * 64]")
    return _TcVarlenAttention.apply(qkv, cu, max_len, heads)


def varlen_query_attention(q: Tensor, kv: Tensor, cu_q: Tensor, cu_k: Tensor, max_q: int, max_k: int,
                           heads: int) -> Tensor:
    """Attention of the packed queries `q` over the packed keys / values `kv`
    of the same sample (see the module docstring); `max_q` and `max_k` are at
    least the most queries and keys of a sample."""
    d = heads * HEAD_DIM
    if not (q.is_cuda and kv.is_cuda and q.dim() == 2 and kv.dim() == 2 and q.shape[1] == d and kv.shape[1] == 2 * d):
        raise ValueError("varlen_query_attention needs CUDA q [total_q, heads * 64] and kv [total_k, 2 * heads * 64]")
    return _TcQueryAttention.apply(q, kv, cu_q, cu_k, max_q, max_k, heads)


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


def reference_query_attention(q: Tensor, kv: Tensor, cu_q: Tensor, cu_k: Tensor, heads: int) -> Tensor:
    """fp32 PyTorch attention of separate packed query and key / value sources."""
    qf, kvf = q.float(), kv.float()
    dh = qf.shape[1] // heads
    out = torch.zeros((qf.shape[0], heads * dh), dtype=torch.float32, device=qf.device)
    bq, bk = cu_q.tolist(), cu_k.tolist()
    for i in range(len(bq) - 1):
        a, b, c, e = bq[i], bq[i + 1], bk[i], bk[i + 1]
        if b <= a or e <= c:
            continue
        qq = qf[a:b].view(b - a, heads, dh).transpose(0, 1)
        k, v = kvf[c:e].view(e - c, 2, heads, dh).permute(1, 2, 0, 3)
        w = torch.softmax(qq @ k.transpose(-1, -2) / dh ** .5, dim=-1)
        out[a:b] = (w @ v).transpose(0, 1).reshape(b - a, heads * dh)
    return out
