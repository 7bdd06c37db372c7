"""Linear layers on the sm_100a tensor-core GEMM (``csrc/tc_gemm.cu``).

``TcLinear`` is a drop-in ``nn.Linear`` (same ``weight`` / ``bias`` parameters,
same state-dict keys) whose forward and backward run as bf16 tcgen05 GEMMs
with fp32 accumulation on CUDA:

    forward  Y  = X W^T + b        (bias and tanh/relu fused in the epilogue)
    dX       dY W                   (W read MN-major, no transpose)
    dW       dY^T X                 (both read MN-major, no transpose)

Inputs are rounded to bf16 and zero-padded to a multiple of 8 features (the
TMA row-stride rule); parameters stay fp32 masters. On CPU the layer is
``F.linear``. ``tensorize(module)`` swaps every ``nn.Linear`` of a module for
a ``TcLinear`` sharing its parameters.
"""
from __future__ import annotations

import torch
from torch import nn
from torch.nn import functional as F

from ..utils import launches
from .ext import require_extension

ACTS = {None: 0, "none": 0, "tanh": 1, "relu": 2, "gelu": 4, "gelu_grad": 5}


def _pad8(n: int) -> int:
    return (n + 7) // 8 * 8


def _bf16_padded(x: torch.Tensor, cols: int, rows: int | None = None) -> torch.Tensor:
    """`x` as a contiguous, 16-byte aligned bf16 [rows, cols] operand; zero
    padding only where the shape grows (no copy when `x` already qualifies)."""
    r = x.shape[0] if rows is None else rows
    if x.shape[1] == cols and r == x.shape[0]:
        y = x.to(torch.bfloat16).contiguous()
        if y.data_ptr() % 16 == 0:
            return y
        return y.clone()
    out = torch.zeros((r, cols), dtype=torch.bfloat16, device=x.device)
    out[:x.shape[0], :x.shape[1]] = x
    return out


def _result_dtype(x: torch.Tensor) -> torch.dtype:
    """Output dtype of a linear layer on `x`: the autocast dtype inside a CUDA
    autocast region (as for nn.Linear), else x's own dtype."""
    if x.is_cuda and torch.is_autocast_enabled("cuda"):
        return torch.get_autocast_dtype("cuda")
    return x.dtype


class TensorCoreTimeout(RuntimeError):
    """A bounded pipeline wait of the tcgen05 GEMM ran out; results of the
    GEMMs since the last check are not valid."""


_PHASES = ((1, "producer: stage free"), (2, "MMA: stage loaded"), (4, "epilogue: accumulator full"),
           (8, "MMA: accumulator free"), (16, "drain of in-flight loads"), (32, "drain of in-flight MMAs"),
           (64, "attention forward MMA"), (128, "attention backward MMA"), (256, "attention drain of in-flight MMAs"))


def _describe(word: int) -> str:
    return ", ".join(name for bit, name in _PHASES if word & bit) or f"status {word:#x}"


class _Status:
    """Per-device GEMM status word, read back without stalling the stream.

    Every GEMM ORs a bit into the word when one of its bounded waits runs
    out. Every `poll_every` launches (and at `check_gemm_status`) the word is
    copied into pinned host memory behind an event; a later call that finds
    the event complete reads it, clears the word and raises
    `TensorCoreTimeout` naming the failed phases.
    """
    poll_every = 64
    _state: dict = {}

    @classmethod
    def _entry(cls, device):
        key = str(device)
        e = cls._state.get(key)
        if e is None:
            word = torch.zeros(1, dtype=torch.int32, device=device)
            host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
            e = {"word": word, "host": host, "event": None, "launches": 0}
            cls._state[key] = e
        return e

    @classmethod
    def get(cls, device) -> torch.Tensor:
        return cls._entry(device)["word"]

    @classmethod
    def _consume(cls, e, block: bool) -> None:
        ev = e["event"]
        if ev is None:
            return
        if not block and not ev.query():
            return
        ev.synchronize()
        e["event"] = None
        value = int(e["host"][0])
        if value:
            e["word"].zero_()
            raise TensorCoreTimeout(f"tcgen05 GEMM wait ran out ({_describe(value)})")

    @classmethod
    def _post(cls, e) -> None:
        if torch.cuda.is_current_stream_capturing():
            return
        e["host"].copy_(e["word"], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        e["event"] = ev

    @classmethod
    def after_launch(cls, device) -> None:
        e = cls._entry(device)
        e["launches"] += 1
        if e["event"] is not None:
            cls._consume(e, block=False)
        if e["event"] is None and e["launches"] % cls.poll_every == 0:
            cls._post(e)

    @classmethod
    def check(cls, device, block: bool = True) -> None:
        e = cls._entry(device)
        cls._consume(e, block=True)
        if torch.cuda.is_current_stream_capturing():
            return
        cls._post(e)
        if block:
            cls._consume(e, block=True)


def check_gemm_status(device=None, block: bool = True) -> None:
    """Raise `TensorCoreTimeout` if a tcgen05 GEMM on `device` (default: the
    current CUDA device) reported a timed-out wait since the last check. With
    block=False only an already finished read-back is examined and a new one
    is queued."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    _Status.check(dev, block)


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn: bool = False, b_mn: bool = False, bias=None, act=None,
         out: torch.Tensor | None = None, accumulate: bool = False, out_dtype=torch.float32,
         wait_ns: int = 2_000_000_000, aux: torch.Tensor | None = None) -> torch.Tensor:
    """C = op(A) op(B)^T on the tensor cores; A is [M,K] (or [K,M] when a_mn),
    B is [N,K] (or [K,N] when b_mn); both bf16 with row strides % 8 == 0.
    `act` "gelu" (erf form) also writes the pre-activation into `aux` (bf16,
    C's layout) when given; "gelu_grad" multiplies the product by GELU' of
    the pre-activation `aux` (the backward of "gelu").
    `wait_ns` bounds every pipeline wait inside the kernel (tests shorten it
    to make a wait run out); timeouts surface through `check_gemm_status`."""
    ext = require_extension()
    m = a.shape[1] if a_mn else a.shape[0]
    n = b.shape[1] if b_mn else b.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    ext.tc_gemm(a, a_mn, b, b_mn, out, bias, ACTS[act], accumulate, _Status.get(a.device), int(wait_ns), aux)
    launches.add(1)
    _Status.after_launch(a.device)
    return out


class _TcLinearFn(torch.autograd.Function):
    """Forward and both gradients on the tensor-core GEMM. A bf16 result (bf16
    input, or a bf16 autocast region) comes straight out of the GEMM epilogue,
    as does a bf16 input gradient: no fp32 intermediate and no cast pass."""

    @staticmethod
    def forward(ctx, x, weight, bias, act):
        out_f, in_f = weight.shape
        lead = x.shape[:-1]
        x2 = x.reshape(-1, in_f)
        in_p, out_p = _pad8(in_f), _pad8(out_f)
        xb = _bf16_padded(x2, in_p)
        wb = _bf16_padded(weight.detach(), in_p, rows=out_p)
        target = _result_dtype(x)
        y_dtype = torch.bfloat16 if target == torch.bfloat16 else torch.float32
        # "gelu": the epilogue also keeps the pre-activation (bf16) for the backward
        z = torch.empty((xb.shape[0], out_f), dtype=torch.bfloat16, device=x.device) if act == "gelu" else None
        y = gemm(xb, wb[:out_f], bias=None if bias is None else bias.detach().float().contiguous(), act=act,
                 out_dtype=y_dtype, aux=z)
        ctx.act = act
        ctx.shapes = (in_f, out_f, in_p, out_p, lead)
        ctx.x_dtype = x.dtype
        ctx.has_bias = bias is not None
        keep = y if act in ("tanh", "relu") else (z if act == "gelu" else torch.empty(0, device=x.device))
        ctx.save_for_backward(xb, wb, keep)
        y = y.reshape(*lead, out_f)
        return y if y.dtype == target else y.to(target)

    @staticmethod
    def backward(ctx, gy):
        xb, wb, y = ctx.saved_tensors
        in_f, out_f, in_p, out_p, lead = ctx.shapes
        g = gy.reshape(-1, out_f)
        if ctx.act == "tanh":
            g = g.float() * (1 - y.float().square())
        elif ctx.act == "relu":
            g = g.float() * (y > 0)
        elif ctx.act == "gelu":   # y holds the pre-activation
            g = torch.ops.aten.gelu_backward(g.float(), y.float())
        gb = _bf16_padded(g, out_p)
        gx = gw = gbias = None
        if ctx.needs_input_grad[0]:
            gx_dtype = torch.bfloat16 if ctx.x_dtype == torch.bfloat16 else torch.float32
            gx = gemm(gb, wb, b_mn=True, out_dtype=gx_dtype)[:, :in_f].reshape(*lead, in_f)
        if ctx.needs_input_grad[1]:
            gw = gemm(gb, xb, a_mn=True, b_mn=True)[:out_f, :in_f]
        if ctx.has_bias and ctx.needs_input_grad[2]:
            gbias = g.sum(0, dtype=torch.float32)
        return gx, gw, gbias, None


class TcLinear(nn.Linear):
    """nn.Linear on the tensor-core GEMM (CUDA), optional fused activation
    ("tanh", "relu", or "gelu" in its exact erf form, like nn.GELU())."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, act: str | None = None,
                 device=None, dtype=None):
        super().__init__(in_features, out_features, bias, device=device, dtype=dtype)
        if act not in ACTS:
            raise ValueError(f"activation must be one of {sorted(k for k in ACTS if k)}")
        self.act = act

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.device.type != "cuda":
            y = F.linear(x, self.weight, self.bias)
            if self.act == "gelu":
                return F.gelu(y)
            return torch.tanh(y) if self.act == "tanh" else (F.relu(y) if self.act == "relu" else y)
        return _TcLinearFn.apply(x, self.weight, self.bias, self.act)


def _plain_gelu(m: nn.Module) -> bool:
    return type(m) is nn.GELU and m.approximate == "none"


def _as_tc_linear(child: nn.Linear, act=None) -> TcLinear:
    tl = TcLinear.__new__(TcLinear)
    nn.Module.__init__(tl)
    tl.in_features, tl.out_features, tl.act = child.in_features, child.out_features, act
    tl.weight = child.weight
    tl.bias = child.bias
    return tl


def tensorize(module: nn.Module) -> nn.Module:
    """Replace every nn.Linear in `module` (recursively) with a TcLinear that
    shares its parameters; a Linear -> GELU -> Linear sequence becomes a
    `TcFeedForward` (GELU fused into both GEMM epilogues) and a Linear
    followed by a GELU a TcLinear with the GELU in its epilogue (the GELU
    module becomes an Identity). Parameters and state-dict keys are kept.
    Returns the module."""
    if type(module) is nn.Sequential and len(module) == 3 and type(module[0]) is nn.Linear \
            and _plain_gelu(module[1]) and type(module[2]) is nn.Linear:
        module.__class__ = TcFeedForward
        module[0] = _as_tc_linear(module[0])
        module[2] = _as_tc_linear(module[2])
        return module
    children = list(module.named_children())
    for k, (name, child) in enumerate(children):
        if type(child) is nn.Linear:
            fuse = isinstance(module, nn.Sequential) and k + 1 < len(children) and _plain_gelu(children[k + 1][1])
            setattr(module, name, _as_tc_linear(child, "gelu" if fuse else None))
            if fuse:
                setattr(module, children[k + 1][0], nn.Identity())
        else:
            tensorize(child)
    return module


class _TcFeedForwardFn(torch.autograd.Function):
    """Linear -> GELU (erf) -> Linear on three tensor-core GEMMs forward and
    three backward. The first forward GEMM writes GELU(Z) and keeps Z (bf16);
    the backward's dH GEMM multiplies by GELU'(Z) in its epilogue, so dZ comes
    out of it directly: no GELU pass and no dH tensor."""

    @staticmethod
    def forward(ctx, x, w1, b1, w2, b2):
        hid, in_f = w1.shape
        out_f = w2.shape[0]
        lead = x.shape[:-1]
        xb = _bf16_padded(x.reshape(-1, in_f), in_f)
        w1b = _bf16_padded(w1.detach(), in_f)
        w2b = _bf16_padded(w2.detach(), hid)
        m = xb.shape[0]
        z = torch.empty((m, hid), dtype=torch.bfloat16, device=x.device)
        h = gemm(xb, w1b, bias=None if b1 is None else b1.detach().float().contiguous(), act="gelu",
                 out_dtype=torch.bfloat16, aux=z)
        target = _result_dtype(x)
        y = gemm(h, w2b, bias=None if b2 is None else b2.detach().float().contiguous(),
                 out_dtype=torch.bfloat16 if target == torch.bfloat16 else torch.float32)
        ctx.save_for_backward(xb, w1b, w2b, z, h)
        ctx.lead, ctx.x_dtype, ctx.biases = lead, x.dtype, (b1 is not None, b2 is not None)
        y = y.reshape(*lead, out_f)
        return y if y.dtype == target else y.to(target)

    @staticmethod
    def backward(ctx, gy):
        xb, w1b, w2b, z, h = ctx.saved_tensors
        out_f, hid = w2b.shape
        in_f = w1b.shape[1]
        g = _bf16_padded(gy.reshape(-1, out_f), out_f)
        dz = gemm(g, w2b, b_mn=True, act="gelu_grad", aux=z, out_dtype=torch.bfloat16)
        gx = gw1 = gb1 = gw2 = gb2 = None
        if ctx.needs_input_grad[0]:
            gx_dtype = torch.bfloat16 if ctx.x_dtype == torch.bfloat16 else torch.float32
            gx = gemm(dz, w1b, b_mn=True, out_dtype=gx_dtype).reshape(*ctx.lead, in_f)
        if ctx.needs_input_grad[1]:
            gw1 = gemm(dz, xb, a_mn=True, b_mn=True)
        if ctx.biases[0] and ctx.needs_input_grad[2]:
            gb1 = dz.sum(0, dtype=torch.float32)
        if ctx.needs_input_grad[3]:
            gw2 = gemm(g, h, a_mn=True, b_mn=True)
        if ctx.biases[1] and ctx.needs_input_grad[4]:
            gb2 = g.sum(0, dtype=torch.float32)
        return gx, gw1, gb1, gw2, gb2


class TcFeedForward(nn.Sequential):
    """Linear -> GELU -> Linear (children 0, 1, 2, as the nn.Sequential it
    replaces) whose CUDA forward and backward run as `_TcFeedForwardFn`; on
    CPU it is the plain sequence."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        l1, l2 = self[0], self[2]
        if x.device.type != "cuda" or l1.in_features % 8 or l1.out_features % 8 or l2.out_features % 8:
            return super().forward(x)
        return _TcFeedForwardFn.apply(x, l1.weight, l1.bias, l2.weight, l2.bias)
