"""GAE scan and fused clip+Adam (host twins here, sm_100a kernels in the gpu tests)
against plain PyTorch fp32 references."""
import pytest
import torch

from autodrive_b200.train.optim import FusedAdam
from autodrive_b200.train.rollout import gae_advantages, gae_reference


def _rollout(T=17, B=33, device="cpu", seed=0):
    g = torch.Generator().manual_seed(seed)
    rew = torch.randn(T, B, generator=g)
    done = torch.rand(T, B, generator=g) < .05
    trunc = torch.rand(T, B, generator=g) < .05
    val = torch.randn(T, B, generator=g)
    nval = torch.randn(T, B, generator=g)
    return [t.to(device) for t in (rew, done, trunc, val, nval)]


def _check_gae(device):
    rew, done, trunc, val, nval = _rollout(device=device)
    stats = torch.zeros(3, dtype=torch.float64, device=device)
    adv = gae_advantages(rew, done, trunc, val, nval, .993, .95, stats)
    ref = gae_reference(rew.cpu(), done.cpu(), trunc.cpu(), val.cpu(), nval.cpu(), .993, .95)
    assert torch.allclose(adv.cpu(), ref, atol=1e-5, rtol=1e-5)
    s = stats.cpu()
    assert s[0].item() == pytest.approx(ref.double().sum().item(), rel=1e-5, abs=1e-6)
    assert s[1].item() == pytest.approx(ref.double().square().sum().item(), rel=1e-5)
    assert s[2].item() == ref.numel()


def _check_adam(device):
    torch.manual_seed(0)
    a = torch.nn.Sequential(torch.nn.Linear(7, 16), torch.nn.Tanh(), torch.nn.Linear(16, 3)).to(device)
    b = torch.nn.Sequential(torch.nn.Linear(7, 16), torch.nn.Tanh(), torch.nn.Linear(16, 3)).to(device)
    b.load_state_dict(a.state_dict())
    fused = FusedAdam(a, lr=1e-2, eps=1e-5, max_grad_norm=.5)
    ref = torch.optim.Adam(b.parameters(), lr=1e-2, eps=1e-5)
    x = torch.randn(64, 7, device=device)
    for _ in range(5):
        fused.zero_grad()
        a(x).square().sum().backward()
        fused.step()
        ref.zero_grad()
        b(x).square().sum().backward()
        torch.nn.utils.clip_grad_norm_(b.parameters(), .5)
        ref.step()
    for pa, pb in zip(a.parameters(), b.parameters()):
        assert torch.allclose(pa, pb, atol=1e-5, rtol=1e-4)


def test_gae_host_matches_reference():
    _check_gae("cpu")


def test_fused_adam_host_matches_torch():
    _check_adam("cpu")


@pytest.mark.gpu
def test_gae_kernel_matches_reference():
    _check_gae("cuda")


@pytest.mark.gpu
def test_fused_adam_kernel_matches_torch():
    _check_adam("cuda")
