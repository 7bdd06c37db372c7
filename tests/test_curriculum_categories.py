"""The full curriculum category matrix: every scenario / category pair builds
its placement (host twin, one world), and the category semantics hold: the
HUB phase and time left before the switch, loads, hidden or absent FUEL and
the scripted blockers."""
import math

import pytest
import torch

from autodrive_b200.train.curriculum import SCENARIOS, CurriculumEnv


def test_category_lists_match_the_reference_matrix():
    counts = {sid: len(sc.required_categories) for sid, sc in SCENARIOS.items()}
    assert counts["hub_transition_cycles"] == 38
    assert counts["offense_vs_scripted_pressure"] == counts["full_match_offense"] == 38
    assert counts["team_delivery_cycles"] == 18
    assert counts["inactive_ferry_preloaded"] == 6 and counts["active_shoot_preloaded"] == 3
    assert "initially_hidden" in SCENARIOS["pickup_scattered"].required_categories
    assert "empty" in SCENARIOS["pickup_multi_zone"].required_categories


@pytest.mark.parametrize("sid", sorted(SCENARIOS))
def test_every_category_resets(sid):
    for cat in SCENARIOS[sid].required_categories:
        env = CurriculumEnv(sid, cat, 1, "cpu", seed=11)
        obs = env.reset(seed=11)
        assert obs.shape == (1, 137) and torch.isfinite(obs).all(), (sid, cat)


def _hub_after(env, ticks):
    full = torch.full((1, 6), 7, dtype=torch.int32)
    env.env.step_held(full, ticks)
    return bool(env.env.hub_active[0, 0])


@pytest.mark.parametrize("cat,now,switch_s", [
    ("active_to_inactive/full/enough_time/carrying_home", True, 12.),
    ("active_to_inactive/empty/too_little_time/collecting", True, 2.5),
    ("inactive_to_active/partial/enough_time/before_release", False, 12.),
    ("inactive_to_active/empty/too_little_time/staged_at_home", False, 2.5)])
def test_transition_categories_set_phase_and_time_left(cat, now, switch_s):
    env = CurriculumEnv("hub_transition_cycles", cat, 1, "cpu", seed=3)
    env.reset(seed=3)
    assert _hub_after(env, 1) == now
    assert _hub_after(env, int(switch_s / .02) - 10) == now          # still before the switch
    assert _hub_after(env, 20) == (not now)                           # switched
    held = int(((env.env.ws["f_owner"][0] == 0) & env.env.ws["f_active"][0].bool()).sum())
    load = cat.split("/")[1]
    if cat.endswith("staged_at_home"):
        free = env.env.ws["f_active"][0].bool() & (env.env.ws["f_owner"][0] < 0)
        assert int((free & (env.env.ws["f_pos"][0, 0] < env.env.alliance_zone_depth)).sum()) >= 8
    else:
        assert held <= {"empty": 0, "partial": 3, "full": 8}[load]


def test_hidden_fuel_starts_behind_the_robot_and_empty_zone_is_empty():
    env = CurriculumEnv("pickup_scattered", "initially_hidden", 1, "cpu", seed=5)
    env.reset(seed=5)
    ws = env.env.ws
    pose = ws["r_pose"][0, 0]
    free = ws["f_active"][0].bool()
    rel = ws["f_pos"][0, :2, free].T - pose[:2]
    ahead = rel[:, 0] * torch.cos(pose[2]) + rel[:, 1] * torch.sin(pose[2])
    assert bool((ahead < 0).all())
    env = CurriculumEnv("pickup_multi_zone", "empty", 1, "cpu", seed=5)
    env.reset(seed=5)
    ws = env.env.ws
    free = ws["f_active"][0].bool()
    dist = (ws["f_pos"][0, :2, free].T - ws["r_pose"][0, 0, :2]).norm(dim=-1)
    assert float(dist.min()) > 3.


@pytest.mark.parametrize("level,slot", [("level_1_stationary", 3), ("level_3_trench", 3), ("level_3_bump", 3),
                                        ("level_5_mixed", 5)])
def test_pressure_blockers_are_placed(level, slot):
    route = {"level_3_trench": "trench", "level_3_bump": "bump"}.get(level, "trench")
    env = CurriculumEnv("offense_vs_scripted_pressure", f"active/{route}/{level}", 1, "cpu", seed=7)
    env.reset(seed=7)
    ws = env.env.ws
    blocker = ws["r_pose"][0, slot, :2]
    x0, y0 = ws["r_pose"][0, 0, :2].tolist()
    if level == "level_3_trench":
        assert abs(float(blocker[0]) - 4.63) < .05 and min(abs(float(blocker[1]) - y) for y in (.83, 7.24)) < .05
    elif level == "level_3_bump":
        assert min(abs(float(blocker[1]) - y) for y in (2.51, 5.56)) < .05
    else:   # on the straight line home
        assert abs(float(blocker[1]) - y0) < .05 and float(blocker[0]) < x0
    assert math.isfinite(float(blocker.sum()))
