"""Fused bf16 LayerNorm kernel against a plain PyTorch fp32 LayerNorm."""
import pytest
import torch
from torch import nn

from autodrive_b200.ops.layernorm import FusedLayerNorm


def test_fused_layer_norm_is_layer_norm_on_cpu():
    torch.manual_seed(0)
    ref = nn.LayerNorm(256)
    fused = FusedLayerNorm(256)
    fused.load_state_dict(ref.state_dict())
    x = torch.randn(7, 5, 256)
    assert torch.allclose(fused(x), ref(x))
    assert set(fused.state_dict()) == {"weight", "bias"}


@pytest.mark.gpu
@pytest.mark.parametrize("d", [64, 128, 256, 512])
@pytest.mark.parametrize("rows", [1, 37, 20000])
def test_fused_layer_norm_matches_fp32(d, rows):
    torch.manual_seed(d + rows)
    ref = nn.LayerNorm(d).cuda()
    with torch.no_grad():
        ref.weight.uniform_(.5, 1.5)
        ref.bias.uniform_(-.2, .2)
    fused = FusedLayerNorm(d).cuda()
    fused.load_state_dict(ref.state_dict())
    x = (torch.randn(rows, d, device="cuda") * 2 + .7).bfloat16().requires_grad_(True)
    xr = x.detach().float().requires_grad_(True)
    y = fused(x)
    y_ref = ref(xr)
    assert y.dtype == torch.bfloat16
    assert (y.float() - y_ref).abs().max().item() < 4e-2
    w = torch.randn_like(y_ref)
    (y.float() * w).sum().backward()
    (y_ref * w).sum().backward()
    assert x.grad.dtype == torch.bfloat16
    for got, want in ((x.grad.float(), xr.grad), (fused.weight.grad, ref.weight.grad), (fused.bias.grad, ref.bias.grad)):
        rel = (got - want).norm().item() / max(want.norm().item(), 1e-12)
        assert rel < 1e-2, rel


@pytest.mark.gpu
def test_fused_layer_norm_under_autocast_takes_fp32_input():
    ln = FusedLayerNorm(256).cuda()
    x = torch.randn(3, 10, 256, device="cuda", requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = ln(x)
    assert y.dtype == torch.bfloat16 and y.shape == x.shape
    y.float().sum().backward()
    assert x.grad.dtype == torch.float32 and torch.isfinite(x.grad).all()
