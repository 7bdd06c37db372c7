"""MECO track training / evaluation on the offense curriculum (host twins)."""
import json

import pytest
import torch

from autodrive_b200.meco.train import (MecoConfig, MecoPolicy, MetricLedger, counterfactual_labels, evaluate_meco,
                                       main, train_meco)
from autodrive_b200.train.curriculum import CurriculumEnv, get_scenario


def _env(n=2):
    cat = get_scenario("pickup_simple").required_categories[0]
    cenv = CurriculumEnv("pickup_simple", cat, n, "cpu")
    cenv.reset()
    return cenv


@pytest.mark.parametrize("track", ["A1", "A2", "A3", "C1", "C2"])
def test_every_track_scores_the_action_candidates(track):
    cenv = _env()
    util, pen, valid, value, hidden = MecoPolicy(track)(cenv.env)
    assert util.shape == pen.shape == valid.shape == (2, 8)
    assert value.shape == (2,) and hidden.shape == (2, 64)
    assert bool(torch.isfinite(util).all()) and bool((pen >= 0).all())


def test_ledger_chain_detects_tampering(tmp_path):
    led = MetricLedger(tmp_path / "ledger.jsonl")
    for k in range(3):
        led.append("row", {"k": k})
    assert led.verify() and len(led.records()) == 3
    lines = (tmp_path / "ledger.jsonl").read_text().splitlines()
    rec = json.loads(lines[1])
    rec["payload"]["k"] = 99
    lines[1] = json.dumps(rec, sort_keys=True)
    (tmp_path / "ledger.jsonl").write_text("\n".join(lines) + "\n")
    assert not led.verify()


def test_counterfactual_labels_pick_a_valid_best_action():
    cenv = _env(2)
    best, value = counterfactual_labels(cenv, horizon=2)
    valid = cenv.env.ws["obs"][:, 0, -8:] > .5
    assert best.shape == (2,) and value.shape == (2, 8)
    assert bool(valid.gather(1, best[:, None]).all())
    assert bool(torch.isinf(value[~valid]).all())


def test_train_and_evaluate_round_trip(tmp_path):
    led = MetricLedger(tmp_path / "ledger.jsonl")
    policy, hist = train_meco(MecoConfig(track="C1", envs=4, updates=1, epochs=1, warm_start_decisions=2), led)
    assert hist[0]["phase"] == "warm_start" and hist[-1]["update"] == 0
    assert led.verify()
    res = evaluate_meco(policy, "pickup_simple", episodes=2)
    assert set(res) >= {"meco", "teacher", "arbiter", "categories"}
    assert res["meco"]["episodes"] == res["teacher"]["episodes"]
    assert sum(res["arbiter"].values()) > 0


def test_cli_writes_checkpoint_and_ledger(tmp_path, capsys):
    assert main(["train", "--track", "C1", "--envs", "2", "--updates", "1", "--epochs", "1",
                 "--output", str(tmp_path)]) == 0
    payload = torch.load(tmp_path / "meco.pt", weights_only=False)
    assert payload["track"] == "C1" and len(payload["weights_sha256"]) == 64
    assert MetricLedger(tmp_path / "metric-ledger.jsonl").verify()
