"""Seeded match-outcome statistics: file format, pooling and the comparison
of the two simulators' outcome files (host only, synthetic files)."""
import json
import math

from autodrive_b200.bench.match_outcomes import _welch, compare, summarize


def _file(tmp_path, name, impl, worlds_by_seed, ticks=(250, 500)):
    seeds = {}
    for seed, scores in worlds_by_seed.items():
        seeds[str(seed)] = {"checkpoints": [
            {"tick": t, "score_by_team": [[s * t // 250, 0] for s in scores],
             "acquisitions_by_robot": [[s, s + 1, s + 2, 0, 0, 0] for s in scores], "elapsed_s": 0.}
            for t in ticks]}
    p = tmp_path / name
    p.write_text(json.dumps({"impl": impl, "seeds": seeds}))
    return str(p)


def test_welch_difference_and_interval():
    a, b = [10., 12., 14., 16.], [9., 10., 11.]
    w = _welch(a, b)
    assert math.isclose(w["difference"], 13. - 10.)
    lo, hi = w["ci95"]
    assert lo < 3. < hi and hi - lo < 12
    assert _welch([5., 5.], [5., 5.])["ci95"] == [0., 0.]


def test_compare_pools_seeds_at_the_common_tick(tmp_path):
    ours = _file(tmp_path, "ours.json", "ours", {1: [10, 20, 30], 2: [40]}, ticks=(250, 500, 750))
    r1 = _file(tmp_path, "ref1.json", "reference", {1: [12, 18]}, ticks=(250, 500))
    r2 = _file(tmp_path, "ref2.json", "reference", {2: [35]}, ticks=(250,))
    out = compare([ours], [r1, r2])
    assert out["tick"] == 250                    # the last tick every seed of both sides reached
    assert out["red_score_per_world"]["ours"]["n"] == 4
    assert out["red_score_per_world"]["reference"]["n"] == 3
    assert math.isclose(out["red_score_per_world"]["ours"]["mean"], 25.)
    at500 = compare([ours], [r1], tick=500)
    assert math.isclose(at500["red_score_per_world"]["reference"]["mean"], 30.)
    assert len(at500["acquisitions_per_robot"]) == 3
    assert summarize([ours])[f"ours:{tmp_path.joinpath('ours.json').name}"]["tick"] == 750
