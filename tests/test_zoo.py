"""Architecture zoo and perception inputs (CPU; tensor-core path on GPU)."""
import pytest
import torch

from autodrive_b200.models import available_networks, build_policy
from autodrive_b200.models.perception import PerceptionInputs
from autodrive_b200.models.zoo import ARCHITECTURES, PerceptionActorCritic, make_policy, parameter_count


@pytest.fixture(scope="module")
def env_inputs():
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    env = TensorThreeVsThreeEnv(num_envs=2, device="cpu", seed=3, fuel_physics=False,
                                control_modes=("deterministic",) * 3 + ("nn",) * 3)
    env.step_held(None, 30)
    return env


def test_perception_inputs_shapes_and_content(env_inputs):
    env = env_inputs
    pin = PerceptionInputs(env, (3, 4, 5))
    d = pin()
    b, p = env.n * 3, env.fuel_count
    assert d["scalars"].shape == (b, 137)
    assert d["field"].shape == (b, 12, 32, 64)
    assert d["entities"].shape == (b, p + 4, 12) and d["entity_mask"].shape == (b, p + 4)
    assert torch.isfinite(d["field"]).all() and torch.isfinite(d["entities"]).all()
    # self token: type flag, zero relative position; exactly one self cell marked
    assert torch.all(d["entities"][:, p, 6] == 1.) and torch.allclose(d["entities"][:, p, :2], torch.zeros(b, 2))
    assert torch.all(d["field"][:, 6].flatten(1).sum(-1) == 1.)
    assert torch.all(d["field"][:, 9].flatten(1).sum(-1) >= 1.) and d["field"][:, 0].sum() > 0
    assert torch.all(d["entity_mask"][:, p:p + 3])
    big = PerceptionInputs(env, (3,), field_shape=(64, 128))()
    assert big["field"].shape == (env.n, 12, 64, 128)


@pytest.mark.parametrize("arch", sorted(ARCHITECTURES))
def test_every_architecture_samples_and_scores(env_inputs, arch):
    torch.manual_seed(0)
    pol = make_policy(arch, tensor_cores=False)
    if arch == "baseline_mlp":
        obs = env_inputs.ws["obs"][:, 3:6].reshape(-1, 137)
        a, lp, v = pol.sample(obs, action_mask=obs[:, -8:] > .5)
        assert a.shape == (6,)
        return
    pin = PerceptionInputs(env_inputs, (3, 4, 5), field_shape=pol.field_shape)
    d = pin()
    a, lp, v = pol.sample(d)
    assert a.shape == lp.shape == v.shape == (6,)
    mask = d["scalars"][:, -8:] > .5
    assert bool(mask.gather(1, a[:, None]).all() | ~mask.any(-1).all())
    logp, ent, val, logits = pol.score(d, a)
    assert torch.allclose(logp, lp, atol=1e-5) and torch.isfinite(ent).all()
    (logp.sum() + val.sum()).backward()
    assert all(p.grad is not None for p in pol.parameters() if p.requires_grad)


def test_parameter_counts_of_the_large_configs():
    n256 = parameter_count(PerceptionActorCritic("entity_attention_256", tensor_cores=False))
    ncnn = parameter_count(PerceptionActorCritic("raster_cnn_large", tensor_cores=False))
    assert 3.0e6 < n256 < 4.5e6, n256
    assert 2.2e7 < ncnn < 2.8e7, ncnn


def test_registry_builds_zoo_networks():
    assert {"entity_attention", "full_field_cnn", "deep_sets"} <= set(available_networks())
    pol = build_policy("deep_sets", 137, 8, "categorical")
    assert isinstance(pol, PerceptionActorCritic)


@pytest.mark.gpu
@pytest.mark.parametrize("arch", ["entity_attention_256", "full_field_cnn", "residual_mlp"])
def test_tensor_core_zoo_matches_fp32(arch):
    torch.manual_seed(4)
    ref = PerceptionActorCritic(arch, tensor_cores=False).cuda()
    tcp = PerceptionActorCritic(arch, tensor_cores=True).cuda()
    tcp.load_state_dict(ref.state_dict())
    b, e = 96, 40
    g = torch.Generator(device="cuda").manual_seed(1)
    d = {"scalars": torch.randn(b, 137, device="cuda", generator=g) * .5,
         "field": torch.rand(b, 12, *ref.field_shape, device="cuda", generator=g),
         "entities": torch.randn(b, e, 12, device="cuda", generator=g) * .3,
         "entity_mask": torch.rand(b, e, device="cuda", generator=g) > .3}
    l1, _, v1 = ref(d)
    l2, _, v2 = tcp(d)
    scale = max(1., l1.abs().max().item())
    assert (l1 - l2).abs().max().item() < 5e-2 * scale
    assert (v1 - v2).abs().max().item() < 5e-2 * max(1., v1.abs().max().item())
    (l2.square().mean() + v2.square().mean()).backward()
    assert all(torch.isfinite(p.grad).all() for p in tcp.parameters() if p.grad is not None)


@pytest.mark.gpu
@pytest.mark.parametrize("heads,dh", [(4, 64), (4, 16)])
def test_packed_attention_matches_fp32(heads, dh):
    """The packed-projection attention (forward and d(qkv)) against fp32
    softmax attention with the same key padding."""
    from autodrive_b200.models.zoo import _PackedAttention, _key_padding_bias
    torch.manual_seed(6)
    b, t = 24, 101
    d = heads * dh
    qkv = (torch.randn(b, t, 3 * d, device="cuda") * .5).bfloat16().requires_grad_(True)
    padding = torch.rand(b, t, device="cuda") > .6
    padding[:, 0] = False                      # the context token is always valid
    out = _PackedAttention.apply(qkv, _key_padding_bias(padding, heads, qkv.dtype), heads)
    x = qkv.detach().float().requires_grad_(True)
    q, k, v = x.view(b, t, 3, heads, dh).permute(2, 0, 3, 1, 4)
    s = (q @ k.transpose(-1, -2)) / dh ** .5
    s = s.masked_fill(padding[:, None, None, :], -torch.inf)
    ref = (s.softmax(-1) @ v).transpose(1, 2).reshape(b, t, d)
    assert out.shape == (b, t, d)
    assert (out.float() - ref).abs().max().item() < 3e-2
    w = torch.randn_like(ref)
    (out.float() * w).sum().backward()
    (ref * w).sum().backward()
    rel = (qkv.grad.float() - x.grad).norm().item() / x.grad.norm().item()
    assert rel < 3e-2, rel


@pytest.mark.gpu
def test_entity_attention_bf16_autocast_matches_fp32():
    torch.manual_seed(7)
    ref = PerceptionActorCritic("entity_attention_256", tensor_cores=False).cuda()
    tcp = PerceptionActorCritic("entity_attention_256", tensor_cores=True).cuda()
    tcp.load_state_dict(ref.state_dict())
    b, e = 64, 120
    g = torch.Generator(device="cuda").manual_seed(2)
    d = {"scalars": torch.randn(b, 137, device="cuda", generator=g) * .5,
         "entities": torch.randn(b, e, 12, device="cuda", generator=g) * .3,
         "entity_mask": torch.rand(b, e, device="cuda", generator=g) > .3}
    l1, _, v1 = ref(d)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        l2, _, v2 = tcp(d)
    assert (l1 - l2.float()).abs().max().item() < 8e-2 * max(1., l1.abs().max().item())
    assert (v1 - v2.float()).abs().max().item() < 8e-2 * max(1., v1.abs().max().item())
    (l1.square().mean() + v1.square().mean()).backward()
    (l2.float().square().mean() + v2.float().square().mean()).backward()
    num = sum((p.grad - q.grad).square().sum() for p, q in zip(ref.parameters(), tcp.parameters()) if p.grad is not None)
    den = sum(p.grad.square().sum() for p in ref.parameters() if p.grad is not None)
    assert (num / den).sqrt().item() < 8e-2


@pytest.mark.gpu
def test_entity_attention_packed_tokens_match_padded():
    """The variable-length form over valid tokens only gives the padded
    form's outputs and gradients (both in bf16 autocast)."""
    torch.manual_seed(8)
    net = PerceptionActorCritic("entity_attention_256", tensor_cores=True).cuda()
    b, e = 48, 150
    g = torch.Generator(device="cuda").manual_seed(3)
    mask = torch.rand(b, e, device="cuda", generator=g) < torch.rand(b, 1, device="cuda", generator=g)
    mask[0] = False                            # a sample with no valid entity
    d = {"scalars": torch.randn(b, 137, device="cuda", generator=g) * .5,
         "entities": torch.randn(b, e, 12, device="cuda", generator=g) * .3, "entity_mask": mask}
    pol = net.network
    assert pol._packed_ok.__func__ is not None
    outs, grads = [], []
    for packed in (True, False):
        net.zero_grad()
        pol._packed_ok = (lambda _inputs, p=packed: p)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits, _, value = net(d)
        (logits.float().square().mean() + value.float().square().mean()).backward()
        outs.append((logits.float(), value.float()))
        grads.append(torch.cat([p.grad.flatten() for p in net.parameters() if p.grad is not None]))
    del pol._packed_ok
    for a, b_ in zip(*outs):
        assert (a - b_).abs().max().item() < 3e-2 * max(1., b_.abs().max().item())
    rel = (grads[0] - grads[1]).norm().item() / grads[1].norm().item()
    assert rel < 3e-2, rel


@pytest.mark.gpu
def test_varlen_query_attention_matches_fp32():
    """One query per sample over variable-length packed keys / values
    (forward and gradients) against fp32 softmax attention."""
    from autodrive_b200.models.zoo import _VarlenQueryAttention
    torch.manual_seed(9)
    heads, dh = 4, 64
    d = heads * dh
    lens = torch.tensor([1, 7, 64, 130, 33, 250, 2, 90])
    cu = torch.nn.functional.pad(lens.cumsum(0), (1, 0)).to(torch.int32).cuda()
    total, b = int(lens.sum()), lens.numel()
    q = (torch.randn(b, d, device="cuda") * .5).bfloat16().requires_grad_(True)
    kv = (torch.randn(total, 2 * d, device="cuda") * .5).bfloat16().requires_grad_(True)
    cu_q = torch.arange(b + 1, device="cuda", dtype=torch.int32)
    out = _VarlenQueryAttention.apply(q, kv, heads, cu_q, cu, int(lens.max()))
    qf, kvf = q.detach().float().requires_grad_(True), kv.detach().float().requires_grad_(True)
    refs = []
    for i in range(b):
        s, e = int(cu[i]), int(cu[i + 1])
        k = kvf[s:e, :d].view(-1, heads, dh).transpose(0, 1)
        v = kvf[s:e, d:].view(-1, heads, dh).transpose(0, 1)
        qq = qf[i].view(heads, 1, dh)
        att = ((qq @ k.transpose(-1, -2)) / dh ** .5).softmax(-1)
        refs.append((att @ v).reshape(d))
    ref = torch.stack(refs)
    assert (out.float() - ref).abs().max().item() < 3e-2
    w = torch.randn_like(ref)
    (out.float() * w).sum().backward()
    (ref * w).sum().backward()
    for a, r in ((q.grad, qf.grad), (kv.grad, kvf.grad)):
        assert (a.float() - r).norm().item() / r.norm().item() < 3e-2
