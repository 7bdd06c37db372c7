"""MECO scorers, arbiter, forecasts, inputs and research operations (CPU)."""
import json
import sys

import pytest
import torch

from autodrive_b200 import meco
from autodrive_b200.meco import inputs as mi
from autodrive_b200.meco.tracks import CANDIDATE_FEATURES, GLOBALS


@pytest.fixture(scope="module")
def env():
    from autodrive_b200.sim.env3v3 import TensorThreeVsThreeEnv
    e = TensorThreeVsThreeEnv(num_envs=2, device="cpu", seed=2, fuel_physics=False)
    e.step_held(None, 25)
    return e


def test_tracks_forward_on_env_inputs(env):
    r = mi.build_raster(env, 3)
    g = mi.build_globals(env, 3)
    ids, valid, feats = mi.safe_action_candidates(env, 3)
    assert r.shape[:2] == (2, 6) and g.shape == (2, GLOBALS) and feats.shape == (2, 8, CANDIDATE_FEATURES)
    graph = mi.se2_lattice(r, stride=6)
    outs = {
        "A1": meco.make_meco_track("A1")(r, g),
        "A2": meco.make_meco_track("A2")(globals_=g, **graph),
        "A3": meco.make_meco_track("A3")(globals_=g, **{k: v for k, v in graph.items() if "coarse" not in k}),
        "C1": meco.make_meco_track("C1")(g, feats),
        "C2": meco.make_meco_track("C2")(r, g, feats),
    }
    for name, o in outs.items():
        assert torch.isfinite(o["utility"]).all() and (o["penalty"] >= 0).all(), name
        assert o["hidden"].shape == (2, 64) and o["behavior_logits"].shape == (2, 5)
    assert outs["A1"]["utility"].shape[1] == 8
    c1 = meco.make_meco_track("C1")
    h = c1(g, feats)["hidden"]
    assert c1(g, feats, hidden=h)["hidden"].shape == h.shape
    with pytest.raises(ValueError):
        c1(g, feats, hidden=torch.full((2, 64), float("nan")))
    with pytest.raises(ValueError):
        meco.make_meco_track("Z9")


def test_choose_candidate_fails_closed():
    req = meco.DecisionRequest(("a", "b", "c"), (True, False, True), "c", observation_time=10.)
    good = meco.ScorerOutput(("a", "b", "c"), (1., 9., .5), (0., 0., 0.), time=9.95)
    assert meco.choose_candidate(req, good) == ("a", "scorer")
    assert meco.choose_candidate(req, None)[1] == "no-scorer-output"
    assert meco.choose_candidate(req, meco.ScorerOutput(("a", "c", "b"), (1,) * 3, (0,) * 3, 9.99))[1] == "candidate-mismatch"
    assert meco.choose_candidate(req, meco.ScorerOutput(("a", "b", "c"), (1,) * 3, (0,) * 3, 9.))[1] == "stale-output"
    bad = meco.ScorerOutput(("a", "b", "c"), (float("nan"), 0., 0.), (0., 0., 0.), 10.)
    assert meco.choose_candidate(req, bad) == ("c", "invalid-output")
    lg = meco.candidate_policy_logits(torch.tensor([1., 2.]), torch.tensor([True, False]))
    assert lg.argmax().item() == 0


def test_opponent_forecast():
    cv = meco.opponent_forecast(mode="constant_velocity", valid=True, position_xy=(1., 1.), velocity_xy=(2., 0.),
                                age_s=.1, horizon_s=1.)
    assert cv["endpoints"][0] == pytest.approx((3.2, 1.))
    mm = meco.opponent_forecast(mode="multimodel", valid=True, position_xy=(0., 0.), velocity_xy=(1., 0.), age_s=0.)
    assert len(mm["endpoints"]) == 5 and abs(sum(mm["weights"]) - 1) < 1e-9
    assert meco.opponent_forecast(mode="multimodel", valid=False, position_xy=(0, 0), velocity_xy=(0, 0), age_s=0) is None
    assert meco.opponent_risk_penalty((3.2, 1.), cv) == pytest.approx(2.)
    assert meco.opponent_risk_penalty((9., 9.), cv) == 0.


def test_device_lease_is_exclusive(tmp_path):
    a = meco.DeviceLease(["cuda:1", "cuda:0"], lock_root=tmp_path)
    with a:
        assert a.acquired and a.devices == ("cuda:0", "cuda:1")
        with pytest.raises(RuntimeError):
            meco.DeviceLease(["cuda:1"], lock_root=tmp_path).acquire()
    with meco.DeviceLease(["cuda:1"], lock_root=tmp_path) as b:
        assert b.acquired
    for bad in (["cpu"], ["cuda:01"], ["cuda:0", "cuda:0"]):
        with pytest.raises(ValueError):
            meco.DeviceLease(bad)


def test_scheduler_resumes_deterministically():
    s1 = meco.MecoTaskScheduler(7, chunks_per_scenario=2)
    seq = []
    for _ in range(4):
        t = s1.next_task()
        seq.append(t["scenario"])
        s1.complete(t)
    s2 = meco.MecoTaskScheduler.from_json(7, s1.to_json(), chunks_per_scenario=2)
    assert s2.next_task() == s1.next_task()
    assert seq[:2] == ["pickup_simple", "pickup_simple"]
    with pytest.raises(ValueError):
        s1.complete({"scenario": "pickup_simple", "chunk": 0, "task_id": "x"})


def test_supervisor_timeout_restart_and_ok(tmp_path):
    tasks = [meco.SupervisedTask("sleepy", [sys.executable, "-c", "import time; time.sleep(30)"], timeout_s=.5,
                                 max_restarts=0),
             meco.SupervisedTask("flaky", [sys.executable, "-c", "import sys; sys.exit(3)"], max_restarts=2),
             meco.SupervisedTask("fine", [sys.executable, "-c", "print('ok')"])]
    res = meco.Supervisor(tasks, backoff_s=.01, grace_s=.5, log_dir=tmp_path).run()
    assert res["sleepy"]["status"] == "timeout"
    assert res["flaky"]["status"] == "failed" and len(res["flaky"]["attempts"]) == 3
    assert res["fine"]["status"] == "ok"


def test_release_gate_and_attestation(tmp_path):
    run = tmp_path / "run"
    run.mkdir()
    assert not meco.release_gate(run)["passed"]
    (run / "policy.pt").write_bytes(b"w")
    (run / "metadata.json").write_text("{}")
    (run / "status.json").write_text(json.dumps({"state": "complete"}))
    import hashlib
    ok = meco.release_gate(run, expected_sha256={"policy.pt": hashlib.sha256(b"w").hexdigest()})
    assert ok["passed"], ok
    assert not meco.release_gate(run, expected_sha256={"policy.pt": "0" * 64})["passed"]
    att = meco.gpu_attestation()
    assert att["extension"]["sha256"] and len(att["digest"]) == 64
