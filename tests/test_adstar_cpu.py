"""CPU AD* planner against a brute-force Dijkstra oracle and its own invariants."""
import heapq
import math

import pytest
import torch

from autodrive_b200 import field as fieldmod
from autodrive_b200.planning import ADStarPlanner


def _dijkstra(blocked, weight, start, goal, nx, ny):
    dist = {start: 0.}
    pq = [(0., start)]
    while pq:
        d, (x, y) = heapq.heappop(pq)
        if (x, y) == goal:
            return d
        if d > dist[(x, y)]:
            continue
        for dx, dy in ((1, 0), (-1, 0), (0, 1), (0, -1), (1, 1), (1, -1), (-1, 1), (-1, -1)):
            xx, yy = x + dx, y + dy
            if not (0 <= xx < nx and 0 <= yy < ny) or blocked[yy, xx]:
                continue
            if dx and dy and (blocked[y, x + dx] or blocked[y + dy, x]):
                continue
            c = (math.sqrt(2.) if dx and dy else 1.) * .5 * (float(weight[y, x]) + float(weight[yy, xx]))
            if d + c < dist.get((xx, yy), math.inf):
                dist[(xx, yy)] = d + c
                heapq.heappush(pq, (d + c, (xx, yy)))
    return math.inf


def _field_planner(**kw):
    boxes = fieldmod.qualification_field()
    return ADStarPlanner(fieldmod.FIELD_LENGTH, fieldmod.FIELD_WIDTH_SIM, fieldmod.static_collision_boxes(boxes),
                         fieldmod.bump_boxes(boxes), **kw)


def _cell_path_cost(pl, start, goal):
    s = pl._cell(start)
    g = pl._cell(goal)
    cells = pl.core.plan(s[1] * pl.nx + s[0], g[1] * pl.nx + g[0], 10 ** 7, 1., 1., .5)
    cost = 0.
    for a, b in zip(cells, cells[1:]):
        ax, ay, bx, by = a % pl.nx, a // pl.nx, b % pl.nx, b // pl.nx
        diag = ax != bx and ay != by
        cost += (math.sqrt(2.) if diag else 1.) * .5 * (float(pl.weight[ay, ax]) + float(pl.weight[by, bx]))
    return cost, cells


def test_optimal_cost_matches_dijkstra_at_epsilon_one():
    pl = _field_planner()
    start, goal = (2.0, 1.2), (14.5, 6.8)
    cost, cells = _cell_path_cost(pl, start, goal)
    ref = _dijkstra(pl.blocked, pl.weight, pl._cell(start), pl._cell(goal), pl.nx, pl.ny)
    assert cells and abs(cost - ref) < 1e-6


def test_path_is_collision_free_and_shortcut():
    pl = _field_planner()
    path = pl.plan((2.0, 1.2), (14.5, 6.8))
    assert len(path) >= 2 and path[0] == (2.0, 1.2) and path[-1] == (14.5, 6.8)
    for a, b in zip(path, path[1:]):
        assert pl.line_is_clear(a, b)
    assert pl.epsilon == pytest.approx(1.)


def test_dynamic_obstacle_replans_incrementally():
    pl = _field_planner()
    a, b = (6.5, 2.6), (10.0, 2.6)
    p1 = pl.plan(a, b)
    assert p1 == [a, b]  # open midfield: a straight segment
    pl.set_dynamic_obstacles([(8.27, 2.6, .5)])
    p2 = pl.plan(a, b)
    assert len(p2) > 2
    for u, v in zip(p2, p2[1:]):
        for k in range(21):
            x, y = u[0] + (v[0] - u[0]) * k / 20, u[1] + (v[1] - u[1]) * k / 20
            assert math.hypot(x - 8.27, y - 2.6) > .5
    pl.set_dynamic_obstacles([])
    assert pl.plan(a, b)


def test_unreachable_and_budget():
    pl = ADStarPlanner(4., 4., colliders=[(2., 2., .1, 2.)], robot_radius=.2)
    assert pl.plan((.5, 2.), (3.5, 2.)) == []
    pl2 = ADStarPlanner(8., 8.)
    assert pl2.plan((.5, .5), (7.5, 7.5), expansion_budget=3) == []


def test_speed_profile_intercept_and_reference():
    pl = _field_planner()
    path = [(1., 1.), (3., 1.), (3., 3.), (6., 3.)]
    v = pl.speed_profile(path, (0., 0.))
    assert v[0] == 0. and v[-1] == 0. and max(v) <= pl.max_speed
    assert v[2] < pl.max_speed  # the corner is speed limited
    ix, iy = ADStarPlanner.predict_intercept((1., 4.), (15., 4.), (8., 6.), (0., 0.))
    assert 1. < ix < 15. and iy == pytest.approx(4.)
    vx, vy = ADStarPlanner.path_reference(path, [1.] * 4, (1.5, 1.1), .35)
    assert vx > 0 and abs(vy) < vx
    assert pl.next_waypoint(path, (2.95, 1.)) == (3., 1.) or pl.next_waypoint(path, (2.95, 1.)) == (3., 3.)
    route = pl.plan_attacker((1.5, 4.), (6., 4.), (4., 4.5))
    assert route
