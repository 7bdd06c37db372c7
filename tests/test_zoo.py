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
