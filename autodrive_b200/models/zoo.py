"""Policy architecture zoo over perception inputs.

Every network maps the perception dictionary of
``autodrive_b200.models.perception.PerceptionInputs``

    scalars      [B, 137]              the strategic observation
    field        [B, 12, H, W]         world-aligned semantic raster
    entities     [B, E, 12]            FUEL tracks + self + 2 allies + opponent
    entity_mask  [B, E]                valid entity slots

to ``(logits [B, A], value [B])``. Architectures (frc_defense/architecture_*.py):

* ``residual_mlp``       scalar-only pre-LN residual GELU MLP (3 blocks, 128)
* ``field_fno``          Fourier-layer field encoder (spectral mixing of the
                         lowest modes, Li et al., arXiv:2010.08895) + scalars
* ``full_field_cnn``     strided 3x3 conv stack with spatial flatten (after
                         the DQN encoder, Mnih et al. 2015) + scalar late fusion
* ``full_field_resnet``  IMPALA-style pooled residual stages (Espeholt et al.
                         2018) + scalar late fusion
* ``deep_sets``          per-entity encoder with mean / max / count pooling
                         (Zaheer et al. 2017)
* ``entity_attention``   pre-LN self-attention blocks over entity tokens with a
                         scalar context token (d=64, 4 heads, 2 blocks)
* ``entity_attention_256``  the same at d=256 with a wide MLP head (~3.8M
                         parameters): the strategic entity encoder
* ``raster_cnn_large``   six 128-channel 3x3 conv layers on a 12 x 64 x 128
                         raster and a wide MLP head (~25M parameters)

Module attribute names follow the reference networks (``trunk``, ``actor``,
``critic``, ``field_encoder``, ``scalar_encoder``, ``fusion``, ``blocks``;
attention keeps ``in_proj_weight`` / ``out_proj``), so their state dicts line
up. On CUDA every ``nn.Linear`` and the attention projections run on the
tcgen05 GEMM (``ops.tc_linear``) when ``tensor_cores=True``, and so does the
variable-length self-attention of the packed entity tokens
(``ops.attention``, head dim 64).
"""
from __future__ import annotations

import torch
from torch import Tensor, nn
from torch.nn import functional as F

from torch.nn.attention import SDPBackend, sdpa_kernel

from ..ops.attention import supported as _tc_attention_supported, varlen_attention, varlen_query_attention
from ..ops.layernorm import FusedLayerNorm
from ..ops.tc_linear import _TcLinearFn, tensorize

_SDPA_BACKENDS = [SDPBackend.EFFICIENT_ATTENTION, SDPBackend.FLASH_ATTENTION, SDPBackend.MATH]


def _linear(x: Tensor, weight: Tensor, bias: Tensor | None, tensor_cores: bool) -> Tensor:
    if tensor_cores and x.is_cuda:
        return _TcLinearFn.apply(x, weight, bias, None)
    return F.linear(x, weight, bias)


# --------------------------------------------------------------------------- dense
class ResidualBlock(nn.Module):
    """x + 0.5 * MLP(LN(x)) with a GELU hidden layer."""

    def __init__(self, width: int):
        super().__init__()
        self.layers = nn.Sequential(nn.LayerNorm(width), nn.Linear(width, width), nn.GELU(),
                                    nn.Linear(width, width))

    def forward(self, x: Tensor) -> Tensor:
        return x + .5 * self.layers(x)


class ResidualMLP(nn.Module):
    def __init__(self, scalar_dim: int = 137, action_dim: int = 8, width: int = 128, blocks: int = 3):
        super().__init__()
        self.trunk = nn.Sequential(nn.Linear(scalar_dim, width), nn.GELU(),
                                   *(ResidualBlock(width) for _ in range(blocks)), nn.LayerNorm(width))
        self.actor = nn.Linear(width, action_dim)
        self.critic = nn.Linear(width, 1)

    def forward(self, inputs: dict) -> tuple[Tensor, Tensor]:
        h = self.trunk(inputs["scalars"])
        return self.actor(h), self.critic(h).squeeze(-1)


class BaselineMLP(nn.Module):
    """The 2 x 128 tanh trunk over scalars, in the perception interface."""

    def __init__(self, scalar_dim: int = 137, action_dim: int = 8):
        super().__init__()
        self.trunk = nn.Sequential(nn.Linear(scalar_dim, 128), nn.Tanh(), nn.Linear(128, 128), nn.Tanh())
        self.actor = nn.Linear(128, action_dim)
        self.critic = nn.Linear(128, 1)

    def forward(self, inputs: dict) -> tuple[Tensor, Tensor]:
        h = self.trunk(inputs["scalars"])
        return self.actor(h), self.critic(h).squeeze(-1)


# --------------------------------------------------------------------------- Fourier field
class SpectralMix(nn.Module):
    """Learned complex channel mixing of the lowest (modes_y, modes_x) rFFT
    modes of a real 2-D field; positive and negative vertical frequencies have
    separate weights. Weights are stored as real pairs."""

    def __init__(self, width: int, modes_y: int = 4, modes_x: int = 6):
        super().__init__()
        self.modes_y, self.modes_x = modes_y, modes_x
        self.weights = nn.Parameter(torch.randn(2, width, width, modes_y, modes_x, 2) / width)

    def forward(self, x: Tensor) -> Tensor:
        spec = torch.fft.rfft2(x, norm="ortho")
        my = min(self.modes_y, x.shape[-2] // 2)
        mx = min(self.modes_x, spec.shape[-1])
        w = torch.view_as_complex(self.weights.contiguous())
        out = torch.zeros_like(spec)
        out[:, :, :my, :mx] = torch.einsum("bchw,cohw->bohw", spec[:, :, :my, :mx], w[0, :, :, :my, :mx])
        out[:, :, -my:, :mx] = torch.einsum("bchw,cohw->bohw", spec[:, :, -my:, :mx], w[1, :, :, :my, :mx])
        return torch.fft.irfft2(out, s=x.shape[-2:], norm="ortho")


class FieldFNOPolicy(nn.Module):
    def __init__(self, scalar_dim: int = 137, action_dim: int = 8, width: int = 16, layers: int = 3):
        super().__init__()
        self.lift = nn.Conv2d(12 + 2, width, 1)
        self.spectral = nn.ModuleList(SpectralMix(width) for _ in range(layers))
        self.local = nn.ModuleList(nn.Conv2d(width, width, 1) for _ in range(layers))
        self.scalar_branch = nn.Sequential(nn.Linear(scalar_dim, 64), nn.Tanh())
        self.trunk = nn.Sequential(nn.Linear(width * 4 * 8 + 64, 128), nn.GELU())
        self.actor = nn.Linear(128, action_dim)
        self.critic = nn.Linear(128, 1)

    def forward(self, inputs: dict) -> tuple[Tensor, Tensor]:
        field = inputs["field"]
        b, _, hgt, wid = field.shape
        ys = torch.linspace(-1, 1, hgt, device=field.device, dtype=field.dtype)
        xs = torch.linspace(-1, 1, wid, device=field.device, dtype=field.dtype)
        gy, gx = torch.meshgrid(ys, xs, indexing="ij")
        coords = torch.stack((gx, gy))[None].expand(b, -1, -1, -1)
        z = self.lift(torch.cat((field, coords), 1))
        z = F.pad(z, (0, 4, 0, 4))  # damp the FFT's periodic wrap
        for spec, loc in zip(self.spectral, self.local):
            z = F.gelu(spec(z) + loc(z))
        z = F.adaptive_avg_pool2d(z[:, :, :hgt, :wid], (4, 8)).flatten(1)
        h = self.trunk(torch.cat((z, self.scalar_branch(inputs["scalars"])), 1))
        return self.actor(h), self.critic(h).squeeze(-1)


# --------------------------------------------------------------------------- rasters
class FullFieldCNN(nn.Module):
    def __init__(self, scalar_dim: int = 137, action_dim: int = 8):
        super().__init__()
        chans = (12, 16, 32, 32)
        convs = []
        for cin, cout in zip(chans[:-1], chans[1:]):
            convs += [nn.Conv2d(cin, cout, 3, stride=2, padding=1), nn.ReLU()]
        self.field_encoder = nn.Sequential(*convs, nn.Flatten(), nn.Linear(32 * 4 * 8, 128), nn.ReLU())
        self.scalar_encoder = nn.Sequential(nn.Linear(scalar_dim, 128), nn.Tanh())
        self.fusion = nn.Sequential(nn.Linear(256, 128), nn.Tanh())
        self.actor = nn.Linear(128, action_dim)
        self.critic = nn.Linear(128, 1)

    def forward(self, inputs: dict) -> tuple[Tensor, Tensor]:
        h = self.fusion(torch.cat((self.field_encoder(inputs["field"]), self.scalar_encoder(inputs["scalars"])), -1))
        return self.actor(h), self.critic(h).squeeze(-1)


class ConvResidual(nn.Module):
    def __init__(self, channels: int):
        super().__init__()
        self.layers = nn.Sequential(nn.ReLU(), nn.Conv2d(channels, channels, 3, padding=1),
                                    nn.ReLU(), nn.Conv2d(channels, channels, 3, padding=1))

    def forward(self, x: Tensor) -> Tensor:
        return x + self.layers(x)


class FullFieldResNet(nn.Module):
    def __init__(self, scalar_dim: int = 137, action_dim: int = 8):
        super().__init__()
        stages, cin = [], 12
        for cout in (16, 32, 32):
            stages += [nn.Conv2d(cin, cout, 3, padding=1), nn.MaxPool2d(3, stride=2, padding=1),
                       ConvResidual(cout), ConvResidual(cout)]
            cin = cout
        self.field_encoder = nn.Sequential(*stages, nn.ReLU(), nn.Flatten(), nn.Linear(32 * 4 * 8, 128), nn.ReLU())
        self.scalar_encoder = nn.Sequential(nn.Linear(scalar_dim, 128), nn.Tanh())
        self.fusion = nn.Sequential(nn.Linear(256, 128), nn.Tanh())
        self.actor = nn.Linear(128, action_dim)
        self.critic = nn.Linear(128, 1)

    def forward(self, inputs: dict) -> tuple[Tensor, Tensor]:
        h = self.fusion(torch.cat((self.field_encoder(inputs["field"]), self.scalar_encoder(inputs["scalars"])), -1))
        return self.actor(h), self.critic(h).squeeze(-1)


class RasterCNNLarge(nn.Module):
    """Six 128-channel 3x3 convs (strides 2,1,2,1,2,1) on a 12 x 64 x 128
    raster -> 128 x 8 x 16 -> wide MLP head; ~25M parameters."""

    def __init__(self, scalar_dim: int = 137, action_dim: int = 8, channels: int = 128, hidden: int = 1408):
        super().__init__()
        layers, cin = [], 12
        for stride in (2, 1, 2, 1, 2, 1):
            layers += [nn.Conv2d(cin, channels, 3, stride=stride, padding=1), nn.ReLU()]
            cin = channels
        self.field_encoder = nn.Sequential(*layers, nn.Flatten())
        self.scalar_encoder = nn.Sequential(nn.Linear(scalar_dim, 256), nn.Tanh())
        self.fusion = nn.Sequential(nn.Linear(channels * 8 * 16 + 256, hidden), nn.ReLU(),
                                    nn.Linear(hidden, 256), nn.Tanh())
        self.actor = nn.Linear(256, action_dim)
        self.critic = nn.Linear(256, 1)

    def forward(self, inputs: dict) -> tuple[Tensor, Tensor]:
        h = self.fusion(torch.cat((self.field_encoder(inputs["field"]), self.scalar_encoder(inputs["scalars"])), -1))
        return self.actor(h), self.critic(h).squeeze(-1)


# --------------------------------------------------------------------------- entity sets
class DeepSetsPolicy(nn.Module):
    def __init__(self, scalar_dim: int = 137, action_dim: int = 8, width: int = 64):
        super().__init__()
        self.width = width
        self.scalar_encoder = nn.Sequential(nn.Linear(scalar_dim, width), nn.Tanh())
        self.entity_encoder = nn.Sequential(nn.Linear(12, width), nn.ReLU(), nn.Linear(width, width), nn.ReLU())
        self.fusion = nn.Sequential(nn.Linear(3 * width + 1, 128), nn.Tanh())
        self.actor = nn.Linear(128, action_dim)
        self.critic = nn.Linear(128, 1)

    def forward(self, inputs: dict) -> tuple[Tensor, Tensor]:
        mask = inputs["entity_mask"].bool()
        m = mask[..., None]
        enc = self.entity_encoder(inputs["entities"].masked_fill(~m, 0.))
        count = mask.sum(1, keepdim=True)
        mean = enc.masked_fill(~m, 0.).sum(1) / count.clamp_min(1)
        mx = enc.masked_fill(~m, -torch.inf).amax(1)
        mx = torch.where(count > 0, mx, torch.zeros_like(mx))
        h = self.fusion(torch.cat((self.scalar_encoder(inputs["scalars"]), mean, mx, count.float().log1p()), -1))
        return self.actor(h), self.critic(h).squeeze(-1)


def _key_padding_bias(padding: Tensor, heads: int, dtype: torch.dtype) -> Tensor:
    """Additive key-padding bias [b, heads, t, t] (a broadcast view) whose row
    storage is padded to 16 elements, the alignment the attention kernel
    needs for its bias rows."""
    b, t = padding.shape
    tp = (t + 15) // 16 * 16
    full = torch.zeros((b, 1, 1, tp), device=padding.device, dtype=dtype)
    bias = full[..., :t]
    bias.masked_fill_(padding[:, None, None, :], -torch.inf)
    return bias.expand(b, heads, t, t)


def _has_efficient_attention_ops() -> bool:
    """PyTorch's memory-efficient attention entry points (private aten ops
    that the packed and variable-length paths call directly)."""
    return hasattr(torch.ops.aten, "_efficient_attention_forward") and \
        hasattr(torch.ops.aten, "_efficient_attention_backward")


_EFFICIENT_OPS = _has_efficient_attention_ops()


class _PackedAttention(torch.autograd.Function):
    """Multi-head self-attention over a packed projection qkv (= [..., 3,
    heads, dh]) on PyTorch's memory-efficient attention kernel, called in its
    native [b, t, heads, dh] layout. Two forms:

    * padded: qkv [b, t, 3d] with an additive key-padding bias;
    * variable length: qkv [total, 3d] holding the valid tokens of all
      samples back to back, sample i at rows cu[i]:cu[i+1] (no bias).

    Queries, keys and values are strided views of qkv, the output comes back
    without a transpose, and the backward asks for dq, dk, dv in one shared
    [..., 3, heads, dh] buffer, which is returned as d(qkv) without a
    stacking copy."""

    @staticmethod
    def forward(ctx, qkv: Tensor, bias, heads: int, cu=None, max_len: int = 0) -> Tensor:
        shape = qkv.shape
        x = qkv.view(*((1,) if cu is not None else ()), *shape[:-1], 3, heads, shape[-1] // (3 * heads))
        q, k, v = x.select(-3, 0), x.select(-3, 1), x.select(-3, 2)
        out, lse, seed, offset, _, _ = torch.ops.aten._efficient_attention_forward(
            q, k, v, bias, cu, cu, max_len if cu is not None else None, max_len if cu is not None else None,
            0.0, 0, True)
        ctx.heads, ctx.max_len = heads, max_len
        ctx.save_for_backward(qkv, bias, out, lse, seed, offset, cu)
        return out.reshape(*shape[:-1], shape[-1] // 3)

    @staticmethod
    def backward(ctx, grad: Tensor):
        qkv, bias, out, lse, seed, offset, cu = ctx.saved_tensors
        shape, h = qkv.shape, ctx.heads
        d3 = shape[-1]
        x = qkv.view(*((1,) if cu is not None else ()), *shape[:-1], 3, h, d3 // (3 * h))
        q, k, v = x.select(-3, 0), x.select(-3, 1), x.select(-3, 2)
        t = q.shape[1]
        ml = ctx.max_len if cu is not None else t
        gq, gk, gv, _ = torch.ops.aten._efficient_attention_backward(
            grad.reshape(out.shape).contiguous().to(out.dtype), q, k, v, bias, out, cu, cu, ml, ml, lse,
            0.0, seed, offset, 0, False, shared_storage_dqdkdv=True)
        d, es = d3 // 3, gq.element_size()
        packed = (gq.stride()[1:] == (d3, d3 // (3 * h), 1) and gk.stride() == gq.stride()
                  and gv.stride() == gq.stride() and (gq.shape[0] == 1 or gq.stride(0) == t * d3)
                  and gk.data_ptr() == gq.data_ptr() + d * es and gv.data_ptr() == gq.data_ptr() + 2 * d * es)
        if packed:
            gqkv = gq.as_strided(shape, qkv.stride())
        else:
            gqkv = torch.stack((gq, gk, gv), -3).reshape(shape)
        return gqkv, None, None, None, None


class _VarlenQueryAttention(torch.autograd.Function):
    """One query per sample attending over that sample's packed keys and
    values: q [b, d], kv [total, 2d] (keys then values, sample i at rows
    cu_k[i]:cu_k[i+1]) on the memory-efficient attention kernel with
    variable-length keys. Used for the last entity block, whose only consumed
    output is the context token's."""

    @staticmethod
    def forward(ctx, q: Tensor, kv: Tensor, heads: int, cu_q: Tensor, cu_k: Tensor, max_k: int) -> Tensor:
        b, d = q.shape
        dh = d // heads
        x = kv.view(1, kv.shape[0], 2, heads, dh)
        out, lse, seed, offset, _, _ = torch.ops.aten._efficient_attention_forward(
            q.view(1, b, heads, dh), x.select(2, 0), x.select(2, 1), None, cu_q, cu_k, 1, max_k, 0.0, 0, True)
        ctx.heads, ctx.max_k = heads, max_k
        ctx.save_for_backward(q, kv, out, lse, seed, offset, cu_q, cu_k)
        return out.reshape(b, d)

    @staticmethod
    def backward(ctx, grad: Tensor):
        q, kv, out, lse, seed, offset, cu_q, cu_k = ctx.saved_tensors
        b, d = q.shape
        h = ctx.heads
        x = kv.view(1, kv.shape[0], 2, h, d // h)
        gq, gk, gv, _ = torch.ops.aten._efficient_attention_backward(
            grad.reshape(out.shape).contiguous().to(out.dtype), q.view(1, b, h, d // h), x.select(2, 0),
            x.select(2, 1), None, out, cu_q, cu_k, 1, ctx.max_k, lse, 0.0, seed, offset, 0, False)
        gkv = torch.stack((gk, gv), 2).reshape(kv.shape)
        return gq.reshape(b, d), gkv, None, None, None, None


class SelfAttention(nn.Module):
    """Multi-head self-attention with key padding; projections packed as
    ``in_proj_weight`` [3d, d] and ``out_proj`` like nn.MultiheadAttention."""

    def __init__(self, dim: int, heads: int, tensor_cores: bool = False):
        super().__init__()
        self.dim, self.heads, self.tensor_cores = dim, heads, tensor_cores
        self.in_proj_weight = nn.Parameter(torch.empty(3 * dim, dim))
        self.in_proj_bias = nn.Parameter(torch.zeros(3 * dim))
        self.out_proj = nn.Linear(dim, dim)
        nn.init.xavier_uniform_(self.in_proj_weight)
        nn.init.zeros_(self.out_proj.bias)

    def forward_packed(self, x: Tensor, cu: Tensor, max_len: int) -> Tensor:
        """Attention within each sample of packed valid tokens x [total, d]
        (sample i at rows cu[i]:cu[i+1]); CUDA, bf16 / fp16 projections."""
        qkv = _linear(x, self.in_proj_weight, self.in_proj_bias, self.tensor_cores)
        if self.tensor_cores and _tc_attention_supported(qkv, self.heads):
            return self.out_proj(varlen_attention(qkv, cu, max_len, self.heads))
        return self.out_proj(_PackedAttention.apply(qkv, None, self.heads, cu, max_len))

    def forward_packed_query(self, x: Tensor, cu: Tensor, max_len: int, rows: Tensor) -> Tensor:
        """Attention output of the packed tokens `rows` only (one per sample,
        e.g. each context token) over all valid tokens of their sample: the
        key / value projection covers every token, the query projection only
        those rows."""
        d = self.dim
        kv = _linear(x, self.in_proj_weight[d:], self.in_proj_bias[d:], self.tensor_cores)
        q = _linear(x[rows], self.in_proj_weight[:d], self.in_proj_bias[:d], self.tensor_cores)
        cu_q = torch.arange(rows.numel() + 1, device=x.device, dtype=torch.int32)
        if self.tensor_cores and kv.is_cuda and self.dim == self.heads * 64:
            return self.out_proj(varlen_query_attention(q, kv, cu_q, cu, 1, max_len, self.heads))
        return self.out_proj(_VarlenQueryAttention.apply(q, kv, self.heads, cu_q, cu, max_len))

    def forward(self, x: Tensor, padding: Tensor) -> Tensor:
        b, t, d = x.shape
        qkv = _linear(x, self.in_proj_weight, self.in_proj_bias, self.tensor_cores)
        if _EFFICIENT_OPS and qkv.is_cuda and qkv.dtype in (torch.bfloat16, torch.float16) and (d // self.heads) % 8 == 0:
            o = _PackedAttention.apply(qkv, _key_padding_bias(padding, self.heads, qkv.dtype), self.heads)
            return self.out_proj(o)
        q, k, v = qkv.view(b, t, 3, self.heads, d // self.heads).permute(2, 0, 3, 1, 4)
        bias = torch.zeros((b, 1, 1, t), device=x.device, dtype=q.dtype).masked_fill(padding[:, None, None, :], -torch.inf)
        # the memory-efficient kernel takes the padding bias directly; the cuDNN
        # backend rebuilds its execution plan on the host for such masks
        with sdpa_kernel(_SDPA_BACKENDS):
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=bias)
        return self.out_proj(o.transpose(1, 2).reshape(b, t, d))


class EntityAttentionBlock(nn.Module):
    def __init__(self, dim: int = 64, heads: int = 4, ff: int = 128, tensor_cores: bool = False):
        super().__init__()
        self.norm_attention = FusedLayerNorm(dim)
        self.attention = SelfAttention(dim, heads, tensor_cores)
        self.norm_feedforward = FusedLayerNorm(dim)
        self.feedforward = nn.Sequential(nn.Linear(dim, ff), nn.GELU(), nn.Linear(ff, dim))

    def forward_packed(self, tokens: Tensor, cu: Tensor, max_len: int) -> Tensor:
        tokens = tokens + self.attention.forward_packed(self.norm_attention(tokens), cu, max_len)
        return tokens + self.feedforward(self.norm_feedforward(tokens))

    def forward_packed_rows(self, tokens: Tensor, cu: Tensor, max_len: int, rows: Tensor) -> Tensor:
        """This block's outputs for the packed tokens `rows` only (one per
        sample): the same values `forward_packed(...)[rows]` gives, without
        the queries, projections and feed-forward of the other tokens."""
        out = tokens[rows] + self.attention.forward_packed_query(self.norm_attention(tokens), cu, max_len, rows)
        return out + self.feedforward(self.norm_feedforward(out))

    def forward(self, tokens: Tensor, padding: Tensor) -> Tensor:
        tokens = tokens + self.attention(self.norm_attention(tokens), padding)
        tokens = tokens + self.feedforward(self.norm_feedforward(tokens))
        return tokens.masked_fill(padding[..., None], 0.)


class EntityAttentionPolicy(nn.Module):
    """Entity tokens plus an always-valid scalar context token; the context
    token's final state feeds the heads (no positional encoding: entity order
    carries no meaning)."""

    def __init__(self, scalar_dim: int = 137, action_dim: int = 8, dim: int = 64, heads: int = 4,
                 blocks: int = 2, ff: int | None = None, head_hidden: tuple[int, ...] = (128,),
                 tensor_cores: bool = False):
        super().__init__()
        ff = ff or 2 * dim
        self.scalar_encoder = nn.Sequential(nn.Linear(scalar_dim, dim), nn.Tanh())
        self.entity_encoder = nn.Sequential(nn.Linear(12, dim), nn.GELU())
        self.blocks = nn.ModuleList(EntityAttentionBlock(dim, heads, ff, tensor_cores) for _ in range(blocks))
        head, width = [FusedLayerNorm(dim)], dim
        for i, hid in enumerate(head_hidden):
            head += [nn.Linear(width, hid), nn.Tanh() if i == len(head_hidden) - 1 else nn.GELU()]
            width = hid
        self.fusion = nn.Sequential(*head)
        self.actor = nn.Linear(width, action_dim)
        self.critic = nn.Linear(width, 1)

    def _packed_ok(self, inputs: dict) -> bool:
        x = inputs["entities"]
        dh = self.blocks[0].attention.dim // self.blocks[0].attention.heads if len(self.blocks) else 0
        return (_EFFICIENT_OPS and x.is_cuda and len(self.blocks) > 0 and dh % 8 == 0
                and torch.is_autocast_enabled("cuda")
                and torch.get_autocast_dtype("cuda") in (torch.bfloat16, torch.float16))

    def _forward_packed(self, inputs: dict) -> tuple[Tensor, Tensor]:
        """The same network on the valid tokens only, packed back to back
        (context token first in each sample). Padding tokens never act as
        keys and their outputs are discarded, so the valid tokens' results
        are those of the padded form; the linear layers and the attention
        then cost what the held tracks cost, not what the slot count does."""
        mask = inputs["entity_mask"].bool()
        b, e = mask.shape
        t = e + 1
        valid = torch.cat((mask.new_ones((b, 1)), mask), 1)
        counts = valid.sum(1, dtype=torch.int32)
        cu = F.pad(counts.cumsum(0, dtype=torch.int32), (1, 0))
        max_len = int(counts.max())
        rows = valid.reshape(-1).nonzero().squeeze(1)
        ents = torch.cat((inputs["entities"].new_zeros((b, 1, inputs["entities"].shape[-1])), inputs["entities"]), 1)
        tokens = self.entity_encoder(ents.reshape(b * t, -1)[rows])
        first = cu[:-1].long()
        ctx = self.scalar_encoder(inputs["scalars"])
        tokens = tokens.index_put((first,), ctx.to(tokens.dtype))
        for blk in self.blocks[:-1]:
            tokens = blk.forward_packed(tokens, cu, max_len)
        # only the context token's final state is read, so the last block
        # computes its output for those rows alone
        h = self.fusion(self.blocks[-1].forward_packed_rows(tokens, cu, max_len, first))
        return self.actor(h), self.critic(h).squeeze(-1)

    def forward(self, inputs: dict) -> tuple[Tensor, Tensor]:
        if self._packed_ok(inputs):
            return self._forward_packed(inputs)
        mask = inputs["entity_mask"].bool()
        ents = inputs["entities"].masked_fill(~mask[..., None], 0.)
        ctx = self.scalar_encoder(inputs["scalars"])[:, None]
        tokens = torch.cat((ctx, self.entity_encoder(ents)), 1)
        padding = torch.cat((mask.new_zeros((mask.shape[0], 1)), ~mask), 1)
        for blk in self.blocks:
            tokens = blk(tokens, padding)
        h = self.fusion(tokens[:, 0])
        return self.actor(h), self.critic(h).squeeze(-1)


def entity_attention_256(scalar_dim: int = 137, action_dim: int = 8, tensor_cores: bool = False):
    return EntityAttentionPolicy(scalar_dim, action_dim, dim=256, heads=4, blocks=2, ff=1024,
                                 head_hidden=(1536, 1024), tensor_cores=tensor_cores)


ARCHITECTURES = {
    "baseline_mlp": BaselineMLP,
    "residual_mlp": ResidualMLP,
    "deep_sets": DeepSetsPolicy,
    "entity_attention": EntityAttentionPolicy,
    "entity_attention_256": entity_attention_256,
    "full_field_cnn": FullFieldCNN,
    "full_field_resnet": FullFieldResNet,
    "field_fno": FieldFNOPolicy,
    "raster_cnn_large": RasterCNNLarge,
}

# raster resolution (rows, cols) each architecture expects
FIELD_SHAPE = {"raster_cnn_large": (64, 128)}
# perception-dictionary entries each architecture reads (a rollout stores only these)
INPUT_KEYS = {
    "baseline_mlp": ("scalars",), "residual_mlp": ("scalars",),
    "deep_sets": ("scalars", "entities", "entity_mask"),
    "entity_attention": ("scalars", "entities", "entity_mask"),
    "entity_attention_256": ("scalars", "entities", "entity_mask"),
    "full_field_cnn": ("scalars", "field"), "full_field_resnet": ("scalars", "field"),
    "field_fno": ("scalars", "field"), "raster_cnn_large": ("scalars", "field"),
}


class PerceptionActorCritic(nn.Module):
    """ActorCritic interface (forward -> (logits, None, value), sample, score)
    over perception dictionaries, with the action mask taken from the last
    `action_dim` scalar features when none is given."""

    def __init__(self, architecture: str, scalar_dim: int = 137, action_dim: int = 8, tensor_cores: bool = True):
        super().__init__()
        if architecture not in ARCHITECTURES:
            raise ValueError(f"unknown architecture {architecture!r}; choose from {sorted(ARCHITECTURES)}")
        self.architecture = architecture
        self.action_kind = "categorical"
        self.obs_dim, self.action_dim = scalar_dim, action_dim
        fn = ARCHITECTURES[architecture]
        kwargs = {"tensor_cores": tensor_cores} if architecture in ("entity_attention", "entity_attention_256") else {}
        self.network = fn(scalar_dim, action_dim, **kwargs)
        if tensor_cores:
            tensorize(self.network)
        self.field_shape = FIELD_SHAPE.get(architecture, (32, 64))
        self.input_keys = INPUT_KEYS[architecture]

    def forward(self, inputs: dict):
        logits, value = self.network(inputs)
        return logits, None, value

    def _masked(self, logits: Tensor, inputs: dict, mask):
        if mask is None:
            mask = inputs["scalars"][:, -self.action_dim:] > .5
        mask = mask.bool()
        mask = torch.where(mask.any(-1, keepdim=True), mask, torch.ones_like(mask))
        return logits.masked_fill(~mask, torch.finfo(logits.dtype).min)

    def sample(self, inputs: dict, deterministic: bool = False, action_mask=None):
        logits, _, value = self(inputs)
        logits = self._masked(logits.float(), inputs, action_mask)
        dist = torch.distributions.Categorical(logits=logits)
        action = logits.argmax(-1) if deterministic else dist.sample()
        return action, dist.log_prob(action), value

    def score(self, inputs: dict, actions: Tensor, action_mask=None):
        logits, _, value = self(inputs)
        logits = self._masked(logits.float(), inputs, action_mask)
        dist = torch.distributions.Categorical(logits=logits)
        actions = actions.long().reshape(-1)
        return dist.log_prob(actions), dist.entropy(), value, logits


def make_policy(architecture: str = "baseline_mlp", tensor_cores: bool = True):
    """The scalar MLP returns the plain ActorCritic; every other architecture
    a PerceptionActorCritic over perception dictionaries."""
    if architecture == "baseline_mlp":
        from .actor_critic import ActorCritic
        return ActorCritic(137, 8, "categorical")
    return PerceptionActorCritic(architecture, tensor_cores=tensor_cores)


def parameter_count(module: nn.Module) -> int:
    return sum(p.numel() for p in module.parameters())


def _register():
    from . import register
    for name in ARCHITECTURES:
        if name == "baseline_mlp":
            continue

        def build(obs_dim, action_dim, action_kind, _name=name):
            if action_kind != "categorical":
                raise ValueError(f"{_name} is a categorical perception policy")
            return PerceptionActorCritic(_name, obs_dim, action_dim)

        register(name)(build)


_register()
__all__ = ["ARCHITECTURES", "PerceptionActorCritic", "make_policy", "parameter_count"]
