"""Offense curriculum: tables, seeds, promotion, scenario env, teachers, training (CPU)."""
import json

import pytest
import torch

from autodrive_b200.train import curriculum as C


def test_scenario_graph_and_seed_partitions():
    assert len(C.SCENARIOS) == 12
    for sid, sc in C.SCENARIOS.items():
        assert set(sc.prerequisites) <= C.SCENARIOS.keys()
        assert sid not in C.ancestors(sid)
    pools = {sp: set(C.seed_partition("pickup_simple", sp, 50)) for sp in C.SPLITS}
    assert all(len(v) == 50 for v in pools.values())
    assert not (pools["train"] & pools["validation"]) and not (pools["test"] & pools["calibration"])
    assert all(s % 4 == C.SPLITS["validation"] for s in pools["validation"])
    assert C.seed_partition("pickup_simple", "train", 3) == C.seed_partition("pickup_simple", "train", 3)
    with pytest.raises(ValueError):
        C.seed_partition("pickup_simple", "bogus", 3)


def _result(sid, rate, eid, thr=1., ref=0., episodes=100):
    sc = C.get_scenario(sid)
    per = episodes // len(sc.required_categories)
    cats = tuple(C.CategoryResult(c, per, int(round(rate * per)), thr, ref) for c in sc.required_categories)
    return C.EvaluationResult(eid, sid, "validation", cats)


def test_promotion_streaks_duplicates_and_retention():
    st = C.CurriculumState()
    for i in range(2):
        d = C.evaluate_promotion(st, _result("pickup_simple", .95, f"r{i}"))
        assert d.passed and not d.promoted
    assert C.evaluate_promotion(st, _result("pickup_simple", .95, "r1")).failures == ("duplicate evaluation ID",)
    d = C.evaluate_promotion(st, _result("pickup_simple", .95, "r2"))
    assert d.promoted and "pickup_simple" in st.qualified
    # next stage needs retention of its ancestors at >= 90 % of the qualified throughput
    bad = C.evaluate_promotion(st, _result("pickup_scattered", .95, "s0"),
                               retention_results=[_result("pickup_simple", .95, "s0", thr=.5)])
    assert not bad.passed and st.consecutive_passes["pickup_scattered"] == 0
    ok = C.evaluate_promotion(st, _result("pickup_scattered", .95, "s1"),
                              retention_results=[_result("pickup_simple", .95, "s1", thr=1.)])
    assert ok.passed
    low = C.evaluate_promotion(st, _result("pickup_scattered", .5, "s2"),
                               retention_results=[_result("pickup_simple", .95, "s2")])
    assert not low.passed and any("success rate" in f for f in low.failures)
    again = C.CurriculumState.from_dict(json.loads(json.dumps(st.to_dict())))
    assert again.qualified == st.qualified
    mix = C.task_mixture(st, ["pickup_scattered"], ["active_shoot_preloaded"])
    assert abs(sum(mix.values()) - 1) < 1e-9 and mix["pickup_scattered"] == pytest.approx(.7)


@pytest.mark.parametrize("sid,cat", [("pickup_simple", "cluster"), ("active_shoot_preloaded", "active/preloaded"),
                                     ("inactive_ferry_preloaded", "inactive/preloaded")])
def test_curriculum_env_and_teachers(sid, cat):
    env = C.CurriculumEnv(sid, cat, 4, "cpu", seed=11)
    obs = env.reset()
    assert obs.shape == (4, 137)
    counts = env.metrics.counts()
    if sid != "pickup_simple":
        assert torch.all(counts["held"] >= 3)
    teacher = C.D2PredictivePolicy()
    done = torch.zeros(4, dtype=torch.bool)
    steps = 0
    while not bool(done.all()) and steps < 6:
        obs, rew, done = env.step(teacher.choose(env, obs))
        steps += 1
        assert rew.shape == (4,) and torch.isfinite(rew).all()
    ok = C.episode_success(sid, cat, env.metrics.counts(), env)
    assert ok.dtype == torch.bool and ok.shape == (4,)


def test_teacher_solves_pickup_simple():
    res = C.evaluate_scenario(None, "pickup_simple", episodes=8, teacher=C.D1HandWeightedPolicy())
    assert res.successes >= 8, res


def test_train_curriculum_runs_and_resumes_strictly(tmp_path):
    cfg = C.TrainingConfig(output=str(tmp_path / "run"), scenarios=("pickup_simple",), envs=8, updates=2,
                           rollout_decisions=6, eval_every=2, eval_episodes=4)
    res = C.train_curriculum(cfg)
    assert res["state"] == "complete"
    status = json.loads((tmp_path / "run" / "curriculum-status.json").read_text())
    assert status["state"] == "complete"
    cfg2 = C.TrainingConfig(output=str(tmp_path / "run"), scenarios=("pickup_simple",), envs=8, updates=3,
                            rollout_decisions=6, eval_every=2, eval_episodes=4)
    C.train_curriculum(cfg2, resume=str(tmp_path / "run" / "curriculum.pt"))
    cfg3 = C.TrainingConfig(output=str(tmp_path / "run"), scenarios=("pickup_simple",), envs=16, updates=3)
    with pytest.raises(ValueError):
        C.train_curriculum(cfg3, resume=str(tmp_path / "run" / "curriculum.pt"))
    out = C.evaluate_curriculum(str(tmp_path / "run" / "curriculum.pt"), ["pickup_simple"], episodes=4)
    assert 0. <= out["pickup_simple"]["success_rate"] <= 1.


def test_sac_curriculum_runs(tmp_path):
    cfg = C.TrainingConfig(output=str(tmp_path / "sac"), scenarios=("pickup_simple",), algorithm="sac", envs=8,
                           updates=2, rollout_decisions=40, eval_every=5, eval_episodes=4)
    assert C.train_curriculum(cfg)["state"] == "complete"


def test_cli_teacher_subcommand(capsys):
    from autodrive_b200.train.cli import main
    main(["curriculum", "teacher", "--scenarios", "pickup_simple", "--episodes", "4", "--teacher", "d2"])
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert "pickup_simple" in out
