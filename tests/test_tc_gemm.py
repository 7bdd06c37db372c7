"""tcgen05 GEMM and TcLinear against plain PyTorch fp32 references."""
import pytest
import torch
from torch import nn

from autodrive_b200.ops.tc_linear import TcLinear, gemm, tensorize


def _store(t: torch.Tensor) -> torch.Tensor:
    """bf16 copy of a 2-D tensor in storage whose row stride is a multiple of 8."""
    r, c = t.shape
    buf = torch.zeros((r, (c + 7) // 8 * 8), dtype=torch.bfloat16, device=t.device)
    buf[:, :c] = t
    return buf[:, :c]


def test_tc_linear_cpu_matches_linear():
    torch.manual_seed(0)
    lin = nn.Linear(13, 7)
    tl = tensorize(nn.Sequential(lin))[0]
    assert isinstance(tl, TcLinear) and tl.weight is lin.weight
    x = torch.randn(5, 13)
    assert torch.allclose(tl(x), x @ lin.weight.T + lin.bias)


@pytest.mark.gpu
@pytest.mark.parametrize("a_mn", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("mnk", [(128, 128, 64), (300, 200, 152), (1000, 72, 1024), (64, 520, 40),
                                 (256, 136, 40000),    # split-K
                                 (4096, 1024, 256),    # 256 tiles: two per persistent CTA
                                 (20000, 384, 136),    # 471 tiles: both accumulators reused
                                 (3000, 520, 1024),    # 256-wide tiles (K >= 512), ragged N
                                 (700, 256, 600)])     # 256-wide tiles, ragged K
def test_gemm_majors_match_fp32(a_mn, b_mn, mnk):
    m, n, k = mnk
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g)
    b = torch.randn(n, k, device="cuda", generator=g)
    ab, bb = a.bfloat16(), b.bfloat16()
    ref = ab.float() @ bb.float().T
    a_arg = _store(ab.T.contiguous()) if a_mn else _store(ab)
    b_arg = _store(bb.T.contiguous()) if b_mn else _store(bb)
    out = gemm(a_arg, b_arg, a_mn=a_mn, b_mn=b_mn)
    torch.cuda.synchronize()
    err = (out - ref).abs().max().item()
    assert err < 1e-3 * max(1., ref.abs().max().item()), err


@pytest.mark.gpu
def test_gemm_epilogues():
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(257, 96, device="cuda", generator=g).bfloat16()
    b = torch.randn(130, 96, device="cuda", generator=g).bfloat16()
    bias = torch.randn(130, device="cuda", generator=g)
    ref = a.float() @ b.float().T + bias
    assert torch.allclose(gemm(a, b, bias=bias, act="tanh"), ref.tanh(), atol=2e-3)
    assert torch.allclose(gemm(a, b, bias=bias, act="relu"), ref.relu(), atol=2e-3)
    out16 = gemm(a, b, bias=bias, out_dtype=torch.bfloat16)
    assert out16.dtype == torch.bfloat16 and torch.allclose(out16.float(), ref, atol=5e-2, rtol=1e-2)
    acc = torch.ones(257, 130, device="cuda")
    gemm(a, b, out=acc, accumulate=True)
    assert torch.allclose(acc, 1 + a.float() @ b.float().T, atol=2e-3)


@pytest.mark.gpu
def test_gelu_epilogues_keep_and_use_the_pre_activation():
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(300, 64, device="cuda", generator=g).bfloat16()
    b = torch.randn(136, 64, device="cuda", generator=g).bfloat16()
    bias = torch.randn(136, device="cuda", generator=g)
    z_ref = a.float() @ b.float().T + bias
    z = torch.empty(300, 136, device="cuda", dtype=torch.bfloat16)
    y = gemm(a, b, bias=bias, act="gelu", aux=z, out_dtype=torch.bfloat16)
    torch.testing.assert_close(z.float(), z_ref, rtol=1e-2, atol=5e-2)
    torch.testing.assert_close(y.float(), torch.nn.functional.gelu(z_ref), rtol=1e-2, atol=5e-2)
    # backward epilogue: (A B^T) * GELU'(z)
    dy = torch.randn(300, 96, device="cuda", generator=g).bfloat16()
    w = torch.randn(96, 136, device="cuda", generator=g).bfloat16()
    dz = gemm(dy, w, b_mn=True, act="gelu_grad", aux=z)
    zf = z.float().requires_grad_(True)
    torch.nn.functional.gelu(zf).backward(dy.float() @ w.float())
    torch.testing.assert_close(dz, zf.grad, rtol=2e-2, atol=2e-2)


@pytest.mark.gpu
def test_gelu_epilogue_precision_in_fp32():
    """fp32 outputs expose the epilogue's own error: the GELU and GELU' values
    agree with PyTorch's exact (erf) forms to ~1e-6 over [-8, 8]."""
    g = torch.Generator(device="cuda").manual_seed(8)
    a = (torch.rand(512, 16, device="cuda", generator=g) * 2 - 1).bfloat16()
    b = (torch.rand(64, 16, device="cuda", generator=g) * 2 - 1).bfloat16()
    bias = torch.linspace(-6, 6, 64, device="cuda")
    z_ref = a.float() @ b.float().T + bias
    z = torch.empty(512, 64, device="cuda", dtype=torch.bfloat16)
    y = gemm(a, b, bias=bias, act="gelu", aux=z)
    assert float(z_ref.abs().max()) > 6
    torch.testing.assert_close(y, torch.nn.functional.gelu(z_ref), rtol=0, atol=2e-6)
    one = torch.ones(512, 16, device="cuda").bfloat16()
    w = (torch.rand(16, 64, device="cuda", generator=g) * 2 - 1).bfloat16()
    dz = gemm(one, w, b_mn=True, act="gelu_grad", aux=z)
    zf = z.float().requires_grad_(True)
    torch.nn.functional.gelu(zf).backward((one.float() @ w.float()))
    torch.testing.assert_close(dz, zf.grad, rtol=0, atol=2e-5)


@pytest.mark.gpu
def test_fused_feed_forward_matches_the_plain_sequence():
    from autodrive_b200.ops.tc_linear import TcFeedForward
    torch.manual_seed(4)
    ref = nn.Sequential(nn.Linear(256, 1024), nn.GELU(), nn.Linear(1024, 256)).cuda()
    fused = nn.Sequential(nn.Linear(256, 1024), nn.GELU(), nn.Linear(1024, 256)).cuda()
    fused.load_state_dict(ref.state_dict())
    tensorize(fused)
    assert type(fused) is TcFeedForward and set(fused.state_dict()) == set(ref.state_dict())
    x = torch.randn(3000, 256, device="cuda", requires_grad=True)
    x2 = x.detach().clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = fused(x)
    y_ref = ref(x2)
    assert y.dtype == torch.bfloat16
    torch.testing.assert_close(y.float(), y_ref, rtol=3e-2, atol=3e-2)
    w = torch.randn_like(y_ref)
    (y.float() * w).sum().backward()
    (y_ref * w).sum().backward()
    pairs = [(x.grad, x2.grad)] + [(p.grad, q.grad) for p, q in zip(fused.parameters(), ref.parameters())]
    for got, want in pairs:
        rel = (got.float() - want).norm().item() / max(want.norm().item(), 1e-12)
        assert rel < 3e-2, rel


@pytest.mark.gpu
def test_linear_gelu_pairs_fuse():
    torch.manual_seed(6)
    ref = nn.Sequential(nn.Linear(40, 136), nn.GELU(), nn.Linear(136, 64), nn.GELU(), nn.Linear(64, 8), nn.Tanh()).cuda()
    import copy
    net = copy.deepcopy(ref)
    tensorize(net)
    assert isinstance(net[1], nn.Identity) and net[0].act == "gelu" and net[2].act == "gelu"
    x = torch.randn(500, 40, device="cuda")
    torch.testing.assert_close(net(x), ref(x), rtol=3e-2, atol=3e-2)
    net(x).square().sum().backward()
    ref(x).square().sum().backward()
    rel = (net[0].weight.grad - ref[0].weight.grad).norm() / ref[0].weight.grad.norm()
    assert float(rel) < 3e-2, float(rel)


@pytest.mark.gpu
@pytest.mark.parametrize("act", [None, "tanh", "relu"])
def test_tc_linear_forward_backward(act):
    torch.manual_seed(1)
    ref = nn.Linear(137, 130).cuda()
    tl = TcLinear(137, 130, act=act).cuda()
    tl.load_state_dict(ref.state_dict())
    x = torch.randn(777, 137, device="cuda", requires_grad=True)
    x2 = x.detach().clone().requires_grad_(True)
    y_ref = ref(x2)
    y_ref = y_ref.tanh() if act == "tanh" else (y_ref.relu() if act == "relu" else y_ref)
    y = tl(x)
    assert (y - y_ref).abs().max().item() < 3e-2
    w = torch.randn_like(y)
    if act == "relu":
        # bf16 inputs flip the gate of pre-activations within rounding of 0:
        # compare gradients under the kernel's own gate
        w = w * ((y > 0) == (y_ref > 0)).float()
    (y * w).sum().backward()
    (y_ref * w).sum().backward()
    for got, want in ((x.grad, x2.grad), (tl.weight.grad, ref.weight.grad), (tl.bias.grad, ref.bias.grad)):
        rel = (got - want).norm().item() / max(want.norm().item(), 1e-12)
        assert rel < 2e-2, rel


@pytest.mark.gpu
def test_tensorized_mlp_trains():
    torch.manual_seed(2)
    net = nn.Sequential(nn.Linear(64, 256), nn.Tanh(), nn.Linear(256, 256), nn.Tanh(), nn.Linear(256, 1)).cuda()
    tensorize(net)
    opt = torch.optim.Adam(net.parameters(), lr=3e-3)
    x = torch.randn(4096, 64, device="cuda")
    target = (x[:, :4].sum(-1, keepdim=True)).tanh()
    first = None
    for _ in range(150):
        loss = (net(x) - target).square().mean()
        opt.zero_grad()
        loss.backward()
        opt.step()
        first = first if first is not None else loss.item()
    assert loss.item() < .2 * first


@pytest.mark.gpu
def test_tc_linear_bf16_autocast_outputs_and_grads():
    """Inside a bf16 autocast region the layer returns bf16 straight from the
    GEMM epilogue and a bf16 input receives a bf16 gradient."""
    torch.manual_seed(5)
    ref = nn.Linear(256, 520).cuda()
    tl = TcLinear(256, 520).cuda()
    tl.load_state_dict(ref.state_dict())
    x = torch.randn(3000, 256, device="cuda").bfloat16().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = tl(x)
    assert y.dtype == torch.bfloat16
    y_ref = x.detach().float() @ ref.weight.T + ref.bias
    assert (y.float() - y_ref).abs().max().item() < 5e-2 * max(1., y_ref.abs().max().item())
    w = torch.randn_like(y_ref)
    (y.float() * w).sum().backward()
    assert x.grad.dtype == torch.bfloat16
    gx_ref = w @ ref.weight
    gw_ref = w.T @ x.detach().float()
    for got, want in ((x.grad.float(), gx_ref), (tl.weight.grad, gw_ref), (tl.bias.grad, w.sum(0))):
        rel = (got - want).norm().item() / max(want.norm().item(), 1e-12)
        assert rel < 2e-2, rel


@pytest.mark.gpu
def test_gemm_wait_expiry_is_reported_and_context_survives():
    """With a zero wait limit the kernel's bounded waits run out: the CTAs
    drain their issued loads and MMAs, the status word records the phase, the
    host raises TensorCoreTimeout (and clears the word), and the next GEMM
    with the normal limit is correct."""
    from autodrive_b200.ops.tc_linear import TensorCoreTimeout, check_gemm_status
    g = torch.Generator(device="cuda").manual_seed(11)
    a = torch.randn(4096, 1024, device="cuda", generator=g).bfloat16()
    b = torch.randn(1024, 1024, device="cuda", generator=g).bfloat16()
    check_gemm_status()
    gemm(a, b, wait_ns=0)
    with pytest.raises(TensorCoreTimeout, match="wait ran out"):
        check_gemm_status()
    check_gemm_status()   # cleared
    out = gemm(a, b)
    check_gemm_status()
    ref = a.float() @ b.float().T
    assert (out - ref).abs().max().item() < 1e-3 * ref.abs().max().item()
