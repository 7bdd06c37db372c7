"""Paired ablation matrix of MECO scorer tracks (host, tiny untrained C1).

Statistics are checked against closed forms: the exact McNemar test is a
two-sided binomial test on the discordant pairs, and Newcombe's interval for
paired proportions reduces to the Wilson-based bounds when nothing is
discordant."""
import json
import math

import pytest
import torch

from autodrive_b200.meco.ablation import ablation_matrix, main, mcnemar_exact, paired_difference_interval
from autodrive_b200.meco.train import ABLATIONS, MecoPolicy, MetricLedger, evaluate_meco


def test_mcnemar_exact_matches_the_binomial_tail():
    assert mcnemar_exact(0, 0) == 1.
    # 0 vs 6 discordant pairs: p = 2 * 0.5**6
    assert math.isclose(mcnemar_exact(0, 6), 2 * .5 ** 6)
    assert math.isclose(mcnemar_exact(6, 0), mcnemar_exact(0, 6))
    # 2 vs 8: 2 * sum_{i<=2} C(10, i) / 2**10
    assert math.isclose(mcnemar_exact(2, 8), 2 * (1 + 10 + 45) / 1024)
    assert mcnemar_exact(5, 5) == 1.


def test_paired_interval_brackets_the_difference():
    diff, lo, hi = paired_difference_interval(10, 2, 8, 20)
    assert math.isclose(diff, (18 - 12) / 40)
    assert lo < diff < hi and -1 <= lo and hi <= 1
    diff, lo, hi = paired_difference_interval(5, 0, 0, 5)
    assert diff == 0 and lo < 0 < hi
    # the interval narrows as the sample grows
    _, l1, h1 = paired_difference_interval(10, 2, 8, 20)
    _, l2, h2 = paired_difference_interval(100, 20, 80, 200)
    assert h2 - l2 < h1 - l1


def test_ablations_are_validated():
    with pytest.raises(ValueError, match="ablation"):
        evaluate_meco(None, "pickup_simple", episodes=1, ablation="no_scorer")


def test_matrix_pairs_matched_episodes(tmp_path):
    torch.manual_seed(0)
    pol = MecoPolicy("C1").eval()
    ledger = MetricLedger(tmp_path / "ledger.jsonl")
    out = ablation_matrix({"C1": pol}, ["pickup_simple"], episodes=2, ablations=("no_penalty", "no_memory"),
                          ledger=ledger)
    assert out["ablations"] == ["no_penalty", "no_memory"]
    assert [c["ablation"] for c in out["cells"]] == ["no_penalty", "no_memory"]
    for cell in out["cells"]:
        n = cell["episodes"]
        assert n > 0
        b, c = cell["discordant"]["full_only"], cell["discordant"]["ablated_only"]
        assert math.isclose(cell["difference"], cell["ablated_success"] - cell["full_success"])
        assert math.isclose(cell["difference"], (c - b) / n)
        assert 0 <= cell["mcnemar_p"] <= 1
        lo, hi = cell["difference_95"]
        assert lo <= cell["difference"] <= hi
    assert len(ledger.records()) == 2 and ledger.verify()
    # the full arm is deterministic on matched seeds: evaluating it again gives the same outcomes
    again = evaluate_meco(pol, "pickup_simple", episodes=2)
    first = evaluate_meco(pol, "pickup_simple", episodes=2)
    assert [r["meco_episodes"] for r in again["categories"]] == [r["meco_episodes"] for r in first["categories"]]


def test_cli_untrained_track(tmp_path, capsys):
    out = tmp_path / "matrix.json"
    assert main(["--untrained", "C1", "--scenarios", "pickup_simple", "--episodes", "1", "--ablations",
                 "uniform_utility", "--output", str(out)]) == 0
    data = json.loads(out.read_text())
    assert data["cells"][0]["ablation"] == "uniform_utility"
    assert set(ABLATIONS) >= set(data["ablations"])
    capsys.readouterr()
