"""Architecture study harness end to end on tiny CPU cases."""
import json

from autodrive_b200.train.architecture_study import main


def test_study_writes_metadata_and_curves(tmp_path):
    outs = main(["--architectures", "deep_sets", "full_field_cnn", "--scenarios", "pickup", "defense_3v3",
                 "--seeds", "3", "--output", str(tmp_path), "--device", "cpu", "--envs", "2", "--eval-envs", "2",
                 "--eval-ticks", "24", "--updates", "2", "--rollout-steps", "3", "--action-repeat", "12",
                 "--epochs", "1", "--minibatch-size", "4", "--eval-every", "1"])
    assert len(outs) == 4
    for out in outs:
        meta = json.loads((out / "metadata.json").read_text())
        curve = json.loads((out / "curve.json").read_text())
        assert meta["status"] == "complete" and meta["parameters"] > 0
        assert meta["perception_only_dynamic_inputs"] and meta["provenance"]["files"] > 10
        assert [c["update"] for c in curve] == [0, 1, 2]
        assert all("mean_score_difference" in c for c in curve)
