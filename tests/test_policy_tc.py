"""tcgen05 policy kernels against a plain PyTorch fp32 reference of the same ops."""
import pytest
import torch

from autodrive_b200.models.actor_critic import ActorCritic
from autodrive_b200.ops import policy_tc
from autodrive_b200.train.optim import FlatParameters


def test_supported_models_cpu():
    assert policy_tc.supported(ActorCritic(137, 8, "categorical"))
    assert not policy_tc.supported(ActorCritic(137, 8, "categorical", hidden=256))
    assert not policy_tc.supported(ActorCritic(35, 3, "continuous"))
    assert not policy_tc.supported(ActorCritic(137, 8, "categorical", layers=3))


def _policy(seed=0, obs_dim=137, act_dim=8):
    torch.manual_seed(seed)
    model = ActorCritic(obs_dim, act_dim, "categorical").cuda()
    flat = FlatParameters(model)
    tc = policy_tc.TensorCorePolicy(model, flat, seed=1234)
    tc.pack()
    return model, flat, tc


def _obs(n, obs_dim=137, act_dim=8, seed=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    obs = torch.randn(n, obs_dim, device="cuda", generator=g) * .7
    obs[:, -act_dim:] = (torch.rand(n, act_dim, device="cuda", generator=g) > .35).float()
    return obs


def _masked_logits(model, obs, act_dim):
    logits, _, value = model(obs)
    mask = obs[:, -act_dim:] > .5
    return logits.masked_fill(~mask, torch.finfo(logits.dtype).min), value, mask


@pytest.mark.gpu
def test_act_greedy_matches_fp32():
    model, flat, tc = _policy()
    obs = _obs(1000)
    obs[5, -8:] = 0.  # a fully masked row
    action, logp, value, mask = tc.act(obs, deterministic=True)
    torch.cuda.synchronize()
    tc._post_status()
    tc.check()
    with torch.no_grad():
        logits, v_ref, m_ref = _masked_logits(model, obs, 8)
        logp_ref = torch.log_softmax(logits, -1)
    keep = torch.ones(1000, dtype=torch.bool, device="cuda")
    keep[5] = False
    assert torch.equal(mask[keep], m_ref[keep])
    assert not mask[5].any()
    assert (value - v_ref).abs().max().item() < 3e-2
    agree = (action[keep] == logits[keep].argmax(-1)).float().mean().item()
    assert agree > .97
    chosen = logp_ref.gather(1, action[:, None]).squeeze(1)
    assert (logp[keep] - chosen[keep]).abs().max().item() < 5e-2
    assert abs(logp[5].item() + torch.log(torch.tensor(8.)).item()) < 1e-4
    assert bool(m_ref[keep].gather(1, action[keep, None]).all())


@pytest.mark.gpu
def test_act_sampling_distribution():
    model, flat, tc = _policy(seed=3)
    row = _obs(1, seed=7)
    row[0, -8:] = torch.tensor([1., 1., 0., 1., 1., 1., 0., 1.], device="cuda")
    obs = row.expand(200_000, -1).contiguous()
    action, logp, value, mask = tc.act(obs)
    with torch.no_grad():
        logits, _, _ = _masked_logits(model, row, 8)
        probs = torch.softmax(logits, -1)[0]
    freq = torch.bincount(action, minlength=8).float() / action.numel()
    assert freq[2].item() == 0. and freq[6].item() == 0.
    assert (freq - probs).abs().max().item() < 1.5e-2
    # the kernel's own log-probabilities are consistent with its samples
    lp = logp.view(-1)
    for a in range(8):
        sel = action == a
        if sel.any():
            assert abs(lp[sel][0].exp().item() - probs[a].item()) < 2e-2


def _reference_grads(model, batch, idx, ent_coef, clip, vcoef, l2c):
    obs = batch["obs"][idx]
    act = batch["actions"][idx]
    mask = batch["mask"][idx]
    old = batch["logp"][idx]
    adv = batch["adv"][idx].double()
    ret = batch["returns"][idx]
    mean = adv.mean()
    std = (adv.square().mean() - mean.square()).clamp_min(0).sqrt()
    advn = ((adv - mean) / (std + 1e-8)).float()
    model.zero_grad(set_to_none=True)
    logp, entropy, value, _ = model.score(obs, act, mask)
    ratio = (logp - old).exp()
    pg = torch.maximum(-advn * ratio, -advn * ratio.clamp(1 - clip, 1 + clip)).mean()
    vloss = .5 * (value - ret).square().mean()
    l2 = sum(p.square().sum() for p in model.parameters() if p.ndim > 1)
    loss = pg + vcoef * vloss - ent_coef * entropy.mean() + l2c * l2
    loss.backward()
    grads = {n: p.grad.detach().clone() for n, p in model.named_parameters()}
    stats = {"kl": ((ratio - 1) - (logp - old)).sum().item(), "entropy": entropy.mean().item(),
             "pg": pg.item(), "vloss": vloss.item(),
             "clipped": ((ratio - 1).abs() > clip).float().sum().item()}
    return grads, stats


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [1000, 128])
def test_train_gradients_match_autograd(rows):
    model, flat, tc = _policy(seed=5)
    n = 3000
    obs = _obs(n, seed=11)
    obs[:, -8] = 1.  # at least one valid action per row
    g = torch.Generator(device="cuda").manual_seed(2)
    mask = obs[:, -8:] > .5
    with torch.no_grad():
        logits, _, _ = _masked_logits(model, obs, 8)
        dist = torch.distributions.Categorical(logits=logits)
        actions = dist.sample()
        old = dist.log_prob(actions) + .15 * torch.randn(n, device="cuda", generator=g)
    batch = {"obs": obs, "actions": actions, "mask": mask, "logp": old,
             "adv": torch.randn(n, device="cuda", generator=g) * 2 + .3,
             "returns": torch.randn(n, device="cuda", generator=g)}
    idx = torch.randperm(n, device="cuda", generator=g)[:rows]
    ent, clip, vcoef, l2c = .01, .2, .5, 1e-3
    stats = torch.zeros(5, device="cuda")
    tc.train_minibatch(batch, idx, torch.full((1,), ent, device="cuda"), clip, vcoef, l2c, stats)
    torch.cuda.synchronize()
    tc._post_status()
    tc.check()
    got = {name: p.grad.detach().clone() for name, p in model.named_parameters()}
    # reference on an fp32 copy (the flat buffer holds the same weights)
    ref_model = ActorCritic(137, 8, "categorical").cuda()
    ref_model.load_state_dict(model.state_dict())
    ref, ref_stats = _reference_grads(ref_model, batch, idx, ent, clip, vcoef, l2c)
    for name in ref:
        err = (got[name] - ref[name]).norm().item() / max(ref[name].norm().item(), 1e-12)
        assert err < 3e-2, (name, err)
    assert abs(stats[0].item() - ref_stats["kl"]) < 2e-2 * rows ** .5 + 1e-3 * rows
    assert abs(stats[2].item() - ref_stats["entropy"]) < 2e-2
    assert abs(stats[3].item() - ref_stats["pg"]) < 2e-2
    assert abs(stats[4].item() - ref_stats["vloss"]) < 2e-2 * max(1., ref_stats["vloss"])


@pytest.mark.gpu
def test_first_epoch_ratio_is_one():
    """log-probabilities from act() and from the training forward agree exactly."""
    model, flat, tc = _policy(seed=9)
    n = 640
    obs = _obs(n, seed=4)
    obs[:, -8] = 1.
    action, logp, value, mask = tc.act(obs)
    batch = {"obs": obs, "actions": action, "mask": mask, "logp": logp,
             "adv": torch.randn(n, device="cuda"), "returns": value.clone()}
    stats = torch.zeros(5, device="cuda")
    idx = torch.arange(n, device="cuda")
    tc.train_minibatch(batch, idx, torch.zeros(1, device="cuda"), .2, .5, 0., stats)
    torch.cuda.synchronize()
    assert stats[0].item() == 0.          # sum of (ratio - 1) - log ratio
    assert stats[1].item() == 0.          # nothing clipped
    assert abs(stats[4].item()) < 1e-12   # returns == values


@pytest.mark.gpu
def test_fused_update_trains():
    from autodrive_b200.train.ppo import PPOConfig, PPOLearner
    torch.manual_seed(0)
    cfg = PPOConfig(epochs=4, minibatch_size=512, grad_backend="local", learning_rate=3e-3)
    learner = PPOLearner(137, 8, "categorical", "cuda", cfg, "mlp", 1)
    assert learner.tc is not None
    n = 2048
    obs = _obs(n, seed=21)
    obs[:, -8:] = 1.
    target = (obs[:, 0] > 0).long() * 3  # reward action 3 when feature 0 > 0, else action 0
    for _ in range(6):
        action, logp, value, mask = learner.act(obs)
        reward = (action == target).float()
        flat = {"obs": obs, "actions": action, "mask": mask, "logp": logp,
                "adv": reward - value, "returns": reward}
        out = learner.update(flat, .0)
    torch.cuda.synchronize()
    learner.tc.check()
    action, _, _, _ = learner.act(obs)
    acc = (action == target).float().mean().item()
    assert acc > .5, acc
    assert out["batches"] == 16 and torch.isfinite(out["approx_kl_sum"]).item()
