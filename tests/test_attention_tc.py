"""Variable-length attention on the tcgen05 kernels against a plain fp32
PyTorch reference of the same packed layout (forward and backward)."""
import pytest
import torch

from autodrive_b200.ops.attention import reference_attention, supported, varlen_attention

HEADS = 4


def _packed(lengths, seed=0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    total = sum(lengths)
    qkv = torch.randn((total, 3 * HEADS * 64), generator=g) * 1.5
    cu = torch.tensor([0] + list(torch.tensor(lengths).cumsum(0).tolist()), dtype=torch.int32)
    return qkv.to(device), cu.to(device)


def test_reference_matches_padded_sdpa():
    lengths = [3, 7, 1]
    qkv, cu = _packed(lengths)
    out = reference_attention(qkv, cu, HEADS)
    for i, n in enumerate(lengths):
        a = int(cu[i])
        q, k, v = qkv[a:a + n].view(n, 3, HEADS, 64).permute(1, 2, 0, 3)
        o = torch.nn.functional.scaled_dot_product_attention(q[None], k[None], v[None])[0]
        torch.testing.assert_close(out[a:a + n], o.permute(1, 0, 2).reshape(n, HEADS * 64), rtol=1e-5, atol=1e-5)


def test_cpu_tensors_are_not_supported():
    qkv, _ = _packed([4])
    assert not supported(qkv, HEADS)
    with pytest.raises(ValueError):
        varlen_attention(qkv, torch.tensor([0, 4]), 4, HEADS)


LENGTHS = [1, 5, 127, 128, 129, 200, 255, 256, 257, 405, 64, 2]


@pytest.mark.gpu
def test_forward_matches_fp32_reference():
    qkv, cu = _packed(LENGTHS, device="cuda")
    x = qkv.to(torch.bfloat16)
    out = varlen_attention(x, cu, max(LENGTHS), HEADS)
    ref = reference_attention(x.float(), cu, HEADS)
    torch.cuda.synchronize()
    assert out.dtype == torch.bfloat16 and out.shape == ref.shape
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    from autodrive_b200.ops.tc_linear import check_gemm_status
    check_gemm_status()


@pytest.mark.gpu
def test_backward_matches_fp32_reference():
    qkv, cu = _packed(LENGTHS, seed=1, device="cuda")
    x = qkv.to(torch.bfloat16).requires_grad_(True)
    out = varlen_attention(x, cu, max(LENGTHS), HEADS)
    g = torch.randn(out.shape, generator=torch.Generator().manual_seed(2)).to("cuda")
    out.backward(g.to(out.dtype))
    xr = x.detach().float().requires_grad_(True)
    reference_attention(xr, cu, HEADS).backward(g)
    got, want = x.grad.float(), xr.grad
    assert got.dtype == torch.float32 and torch.isfinite(got).all()
    scale = want.abs().amax(dim=0, keepdim=True).clamp_min(1e-3)
    err = ((got - want).abs() / scale).amax()
    assert float(err) < 3e-2, float(err)
    # relative Frobenius error of each of dq, dk, dv
    for part in range(3):
        sl = slice(part * HEADS * 64, (part + 1) * HEADS * 64)
        rel = (got[:, sl] - want[:, sl]).norm() / want[:, sl].norm()
        assert float(rel) < 2e-2, (part, float(rel))


@pytest.mark.gpu
def test_entity_network_uses_the_tensor_core_attention():
    from autodrive_b200.models.zoo import SelfAttention
    from autodrive_b200.utils import launches
    att = SelfAttention(256, HEADS, tensor_cores=True).cuda()
    lengths = [17, 140, 3]
    x = torch.randn((sum(lengths), 256), device="cuda")
    cu = torch.tensor([0, 17, 157, 160], dtype=torch.int32, device="cuda")
    before = launches.read()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = att.forward_packed(x, cu, 140)
    y.float().sum().backward()
    torch.cuda.synchronize()
    assert launches.read() >= before + 2          # the attention forward and backward kernels ran
    assert torch.isfinite(y.float()).all() and torch.isfinite(att.in_proj_weight.grad).all()
    # same result as the padded PyTorch path of the module
    pad = torch.zeros((3, 140, 256), device="cuda")
    mask = torch.ones((3, 140), dtype=torch.bool, device="cuda")
    for i, (a, n) in enumerate(zip([0, 17, 157], lengths)):
        pad[i, :n] = x[a:a + n]
        mask[i, :n] = False
    att.tensor_cores = False
    with torch.autocast("cuda", dtype=torch.bfloat16):
        ref = att(pad, mask)
    for i, (a, n) in enumerate(zip([0, 17, 157], lengths)):
        torch.testing.assert_close(y[a:a + n].float(), ref[i, :n].float(), rtol=3e-2, atol=3e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("queries", [[1] * 12, [3, 1, 0, 130, 2, 1, 1, 5, 1, 1, 1, 1]])
def test_query_attention_matches_fp32_reference(queries):
    from autodrive_b200.ops.attention import reference_query_attention, varlen_query_attention
    g = torch.Generator().manual_seed(3)
    keys = LENGTHS
    q = (torch.randn((sum(queries), HEADS * 64), generator=g) * 1.5).cuda().to(torch.bfloat16).requires_grad_(True)
    kv = (torch.randn((sum(keys), 2 * HEADS * 64), generator=g) * 1.5).cuda().to(torch.bfloat16).requires_grad_(True)
    cu_q = torch.tensor([0] + torch.tensor(queries).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    cu_k = torch.tensor([0] + torch.tensor(keys).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    out = varlen_query_attention(q, kv, cu_q, cu_k, max(queries), max(keys), HEADS)
    qr, kvr = q.detach().float().requires_grad_(True), kv.detach().float().requires_grad_(True)
    ref = reference_query_attention(qr, kvr, cu_q, cu_k, HEADS)
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    dout = torch.randn(out.shape, generator=torch.Generator().manual_seed(4)).cuda()
    out.backward(dout.to(out.dtype))
    ref.backward(dout)
    for got, want in ((q.grad.float(), qr.grad), (kv.grad.float(), kvr.grad)):
        rel = (got - want).norm() / want.norm().clamp_min(1e-6)
        assert float(rel) < 2e-2, float(rel)
