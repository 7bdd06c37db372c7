"""Discrete SAC: device-resident scenario replay and the update step (CPU)."""
import pytest
import torch

from autodrive_b200.train.sac import (DiscreteSAC, ScenarioReplayBuffer, make_sac_optimizers, masked_distribution,
                                      sac_update)


def _batch(n, scen_value, obs_dim=137):
    obs = torch.randn(n, obs_dim)
    obs[:, 0] = scen_value
    mask = torch.ones(n, 8, dtype=torch.bool)
    mask[:, 5] = False
    return {"obs": obs, "mask": mask, "action": torch.randint(0, 5, (n,)), "reward": torch.randn(n),
            "next_obs": torch.randn(n, obs_dim), "next_mask": mask.clone(), "done": torch.zeros(n, dtype=torch.bool)}


def test_masked_distribution_zeroes_invalid():
    logits = torch.randn(4, 8)
    mask = torch.rand(4, 8) > .4
    mask[:, 0] = True
    p, lp, m = masked_distribution(logits, mask)
    assert torch.allclose(p.sum(-1), torch.ones(4)) and torch.all(p[~mask] == 0) and torch.all(lp[~mask] == 0)
    with pytest.raises(ValueError):
        masked_distribution(logits, mask[:, :4])


def test_replay_balances_scenarios_and_wraps():
    rb = ScenarioReplayBuffer(100)
    rb.add_batch(_batch(90, 1.), "a")
    rb.add_batch(_batch(10, 2.), "b")
    g = torch.Generator().manual_seed(0)
    draws = torch.cat([rb.sample(100, generator=g)["obs"][:, 0] for _ in range(40)])
    frac_b = (draws == 2.).float().mean().item()
    assert .45 < frac_b < .55          # even across scenarios, not across rows
    rb.add_batch(_batch(95, 3.), "c")  # overwrites all of "a" but 5 rows... ring order
    assert len(rb) == 100
    vals = set(rb.sample(100, generator=g)["obs"][:, 0].tolist())
    assert 3. in vals and vals <= {1., 2., 3.}
    st = rb.state_dict()
    rb2 = ScenarioReplayBuffer(100)
    rb2.load_state_dict(st)
    assert len(rb2) == 100 and rb2.position == rb.position
    with pytest.raises(ValueError):
        ScenarioReplayBuffer(10).load_state_dict(st)
    with pytest.raises(ValueError):
        ScenarioReplayBuffer(100).sample(1)


def test_replay_stores_perception_dicts():
    rb = ScenarioReplayBuffer(16)
    b = _batch(8, 0.)
    b["obs"] = {"scalars": b["obs"], "field": torch.rand(8, 12, 4, 8)}
    b["next_obs"] = {"scalars": b["next_obs"], "field": torch.rand(8, 12, 4, 8)}
    rb.add_batch(b, "x")
    s = rb.sample(5)
    assert s["obs"]["field"].shape == (5, 12, 4, 8) and s["action"].dtype == torch.long


def test_sac_update_learns_a_bandit():
    torch.manual_seed(0)
    agent = DiscreteSAC("baseline_mlp", initial_alpha=.05)
    opt = make_sac_optimizers(agent, 3e-3)
    rb = ScenarioReplayBuffer(512)
    for _ in range(4):
        b = _batch(128, 0.)
        b["reward"] = (b["action"] == 2).float()
        b["done"] = torch.ones(128, dtype=torch.bool)
        rb.add_batch(b, "bandit")
    for _ in range(300):
        out = sac_update(agent, opt, rb.sample(128), gamma=.99, tau=.05, target_entropy_fraction=.3)
    assert torch.isfinite(out["critic_loss"]) and out["valid_action_count"].item() == 7.
    obs = torch.randn(256, 137)
    mask = torch.ones(256, 8, dtype=torch.bool)
    a, lp, _ = agent.sample(obs, deterministic=True, action_mask=mask)
    assert (a == 2).float().mean().item() > .75
    for pt, ps in zip(agent.target_q1.parameters(), agent.q1.parameters()):
        assert not pt.requires_grad
