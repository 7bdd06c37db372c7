"""CPU AD* route planner (reference / dashboard route reconstruction).

``ADStarPlanner`` keeps the public surface of frc_defense/adstar.py:62-1119:
an incremental Anytime Dynamic A* search on an 8-connected field grid (the
native ``ADStarCore``: Likhachev et al., ICAPS 2005) with

* footprint-inflated static occupancy: a cell is blocked when the robot's
  oriented bumper rectangle (or its circle, when ``robot_radius`` is given)
  centred there overlaps a collider or leaves the field; bump cells cost 12 %
  more to cross;
* dynamic circular obstacles (``set_dynamic_obstacles``) repaired
  incrementally; the inflation factor epsilon decays from 2.5 to 1 while the
  expansion budget lasts;
* path finishing: endpoints projected to the nearest free cell, greedy
  line-of-sight shortcutting, exact start/goal points;
* ``speed_profile``: curvature-limited (lateral friction) speeds with forward
  acceleration and backward braking passes;
* ``predict_intercept`` / ``plan_attacker``: the earliest point on an
  attacker's goal line a defender can reach first;
* ``next_waypoint`` / ``path_reference``: lookahead point and a velocity
  command along the path.
"""
from __future__ import annotations

import math

import torch

from ..ops import require_extension

BUMP_WEIGHT = 1.12


def _box(box) -> tuple[float, float, float, float]:
    if hasattr(box, "length"):
        return float(box.x), float(box.y), float(box.length) / 2, float(box.width) / 2
    cx, cy, hx, hy = box
    return float(cx), float(cy), float(hx), float(hy)


class ADStarPlanner:
    def __init__(self, length: float, width: float, colliders=(), bumps=(), *, resolution: float = .2,
                 robot_length: float = .9, robot_width: float = .9, robot_radius: float | None = None,
                 robot_heading: float = 0., max_speed: float = 4.8, max_acceleration: float = 8.,
                 steering_rate: float = 12., lateral_friction: float = 1.2, max_angular_speed: float = 8.,
                 max_angular_acceleration: float = 18.):
        self.length, self.width, self.resolution = float(length), float(width), float(resolution)
        self.nx, self.ny = math.ceil(self.length / self.resolution), math.ceil(self.width / self.resolution)
        self.colliders = tuple(_box(b) for b in colliders)
        self.bumps = tuple(_box(b) for b in bumps)
        self.robot_radius = float(robot_radius or 0.)
        self.robot_length, self.robot_width = max(.01, float(robot_length)), max(.01, float(robot_width))
        self.robot_heading = float(robot_heading)
        self.configure_kinematics(max_speed, max_acceleration, steering_rate, lateral_friction,
                                  max_angular_speed, max_angular_acceleration)
        self.core = require_extension().ADStarCore(self.nx, self.ny)
        self._dynamic: tuple = ()
        self._rebuild()

    # ---------------------------------------------------------------- configuration
    def configure_kinematics(self, max_speed, max_acceleration, steering_rate=12., lateral_friction=1.2,
                             max_angular_speed=8., max_angular_acceleration=18.) -> None:
        self.max_speed, self.max_acceleration = max(.1, float(max_speed)), max(.1, float(max_acceleration))
        self.steering_rate, self.lateral_friction = max(.1, float(steering_rate)), max(.1, float(lateral_friction))
        self.max_angular_speed = max(.1, float(max_angular_speed))
        self.max_angular_acceleration = max(.1, float(max_angular_acceleration))

    def configure_footprint(self, robot_length: float, robot_width: float, heading: float) -> None:
        self.robot_length, self.robot_width = max(.01, float(robot_length)), max(.01, float(robot_width))
        self.robot_heading = float(heading)
        self._rebuild()

    def set_dynamic_obstacles(self, obstacles) -> None:
        """Circles (x, y, radius) blocking cells this planning cycle."""
        self._dynamic = tuple((float(x), float(y), float(r)) for x, y, r in obstacles)
        self._rebuild()

    # ---------------------------------------------------------------- occupancy
    def _centers(self):
        xs = (torch.arange(self.nx, dtype=torch.float64) + .5) * self.resolution
        ys = (torch.arange(self.ny, dtype=torch.float64) + .5) * self.resolution
        gy, gx = torch.meshgrid(ys, xs, indexing="ij")
        return gx, gy

    def _footprint_hits(self, gx, gy, box) -> torch.Tensor:
        cx, cy, hx, hy = box
        half = .5 * self.resolution  # colliders expanded by half a cell
        if self.robot_radius > 0:
            dx = ((gx - cx).abs() - hx - half).clamp_min(0)
            dy = ((gy - cy).abs() - hy - half).clamp_min(0)
            return dx * dx + dy * dy <= self.robot_radius ** 2
        c, s = math.cos(self.robot_heading), math.sin(self.robot_heading)
        hl, hw = self.robot_length / 2, self.robot_width / 2
        rx, ry = abs(c) * hl + abs(s) * hw, abs(s) * hl + abs(c) * hw
        sep = ((gx - cx).abs() > rx + hx + half) | ((gy - cy).abs() > ry + hy + half)
        # the robot's own axes
        for ax, ay, r in ((c, s, hl), (-s, c, hw)):
            proj = ((gx - cx) * ax + (gy - cy) * ay).abs()
            sep |= proj > r + (hx + half) * abs(ax) + (hy + half) * abs(ay)
        return ~sep

    def _rebuild(self) -> None:
        gx, gy = self._centers()
        if self.robot_radius > 0:
            mx = my = self.robot_radius
        else:
            c, s = abs(math.cos(self.robot_heading)), abs(math.sin(self.robot_heading))
            mx = (self.robot_length * c + self.robot_width * s) / 2
            my = (self.robot_length * s + self.robot_width * c) / 2
        blocked = (gx < mx) | (gx > self.length - mx) | (gy < my) | (gy > self.width - my)
        for box in self.colliders:
            blocked |= self._footprint_hits(gx, gy, box)
        reach = math.hypot(self.robot_length, self.robot_width) / 2 if self.robot_radius <= 0 else self.robot_radius
        for x, y, r in self._dynamic:
            blocked |= (gx - x) ** 2 + (gy - y) ** 2 <= (r + reach) ** 2
        weight = torch.ones_like(gx, dtype=torch.float32)
        for cx, cy, hx, hy in self.bumps:
            on = ((gx - cx).abs() <= hx) & ((gy - cy).abs() <= hy)
            weight = torch.where(on, torch.full_like(weight, BUMP_WEIGHT), weight)
        self.blocked = blocked
        self.weight = weight
        self.core.set_grid(blocked.reshape(-1).to(torch.uint8), weight.reshape(-1))

    # ---------------------------------------------------------------- search
    def _cell(self, p) -> tuple[int, int]:
        ix = min(max(int(p[0] / self.resolution), 0), self.nx - 1)
        iy = min(max(int(p[1] / self.resolution), 0), self.ny - 1)
        return ix, iy

    def _center(self, cell) -> tuple[float, float]:
        return ((cell[0] + .5) * self.resolution, (cell[1] + .5) * self.resolution)

    def _nearest_free(self, cell) -> tuple[int, int] | None:
        if not bool(self.blocked[cell[1], cell[0]]):
            return cell
        free = (~self.blocked).nonzero()
        if free.numel() == 0:
            return None
        d = (free[:, 1] - cell[0]) ** 2 + (free[:, 0] - cell[1]) ** 2
        k = int(d.argmin())
        return int(free[k, 1]), int(free[k, 0])

    def line_is_clear(self, a, b) -> bool:
        """Every grid cell sampled along a->b (quarter-cell steps) is free."""
        n = max(1, int(math.hypot(b[0] - a[0], b[1] - a[1]) / (self.resolution * .25)))
        for i in range(n + 1):
            t = i / n
            ix, iy = self._cell((a[0] + (b[0] - a[0]) * t, a[1] + (b[1] - a[1]) * t))
            if bool(self.blocked[iy, ix]):
                return False
        return True

    def plan(self, start, goal, *, expansion_budget: int = 12000, epsilon: float = 2.5):
        """Waypoints [(x, y), ...] from start to goal, or [] when unreachable."""
        s_cell = self._nearest_free(self._cell(start))
        g_cell = self._nearest_free(self._cell(goal))
        if s_cell is None or g_cell is None:
            return []
        cells = self.core.plan(s_cell[1] * self.nx + s_cell[0], g_cell[1] * self.nx + g_cell[0],
                               int(expansion_budget), float(epsilon), 1., .5)
        if not cells:
            return []
        pts = [self._center((c % self.nx, c // self.nx)) for c in cells]
        pts[0] = (float(start[0]), float(start[1])) if s_cell == self._cell(start) else pts[0]
        pts[-1] = (float(goal[0]), float(goal[1])) if g_cell == self._cell(goal) else pts[-1]
        return self.shortcut(pts)

    @property
    def epsilon(self) -> float:
        return self.core.epsilon

    def shortcut(self, pts):
        if len(pts) <= 2:
            return list(pts)
        out, i = [pts[0]], 0
        while i < len(pts) - 1:
            j = len(pts) - 1
            while j > i + 1 and not self.line_is_clear(pts[i], pts[j]):
                j -= 1
            out.append(pts[j])
            i = j
        return out

    # ---------------------------------------------------------------- kinematics
    def speed_profile(self, path, initial_velocity=(0., 0.)):
        """Per-waypoint speed limit: lateral friction on turns, then forward
        acceleration and backward braking passes (ends at rest)."""
        n = len(path)
        if n == 0:
            return []
        v = [self.max_speed] * n
        for k in range(1, n - 1):
            a = (path[k][0] - path[k - 1][0], path[k][1] - path[k - 1][1])
            b = (path[k + 1][0] - path[k][0], path[k + 1][1] - path[k][1])
            la, lb = math.hypot(*a), math.hypot(*b)
            if la < 1e-9 or lb < 1e-9:
                continue
            turn = math.acos(max(-1., min(1., (a[0] * b[0] + a[1] * b[1]) / (la * lb))))
            radius = min(la, lb) / max(2 * math.sin(turn / 2), 1e-9)
            v[k] = min(v[k], math.sqrt(self.lateral_friction * 9.81 * radius))
        v[0] = min(self.max_speed, math.hypot(*initial_velocity))
        v[-1] = 0.
        for k in range(1, n):
            d = math.hypot(path[k][0] - path[k - 1][0], path[k][1] - path[k - 1][1])
            v[k] = min(v[k], math.sqrt(v[k - 1] ** 2 + 2 * self.max_acceleration * d))
        for k in range(n - 2, -1, -1):
            d = math.hypot(path[k + 1][0] - path[k][0], path[k + 1][1] - path[k][1])
            v[k] = min(v[k], math.sqrt(v[k + 1] ** 2 + 2 * self.max_acceleration * d))
        return v

    @staticmethod
    def predict_intercept(attacker, goal, defender, defender_velocity=(0., 0.), *, attacker_speed=4.5,
                          defender_speed=4.8, samples: int = 64):
        """First point on the attacker->goal segment the defender reaches no
        later than the attacker (constant speeds); the goal when none is."""
        ax, ay = attacker
        gx, gy = goal
        seg = math.hypot(gx - ax, gy - ay)
        lead = .25  # defender velocity look-ahead (s)
        dx0, dy0 = defender[0] + defender_velocity[0] * lead, defender[1] + defender_velocity[1] * lead
        for i in range(samples + 1):
            t = i / samples
            px, py = ax + (gx - ax) * t, ay + (gy - ay) * t
            if math.hypot(px - dx0, py - dy0) / defender_speed + lead <= seg * t / attacker_speed:
                return px, py
        return float(gx), float(gy)

    def plan_attacker(self, attacker, goal, defender, defender_velocity=(0., 0.), *, block_radius=.6, **kw):
        """Route for the attacker avoiding the defender's predicted intercept."""
        ix, iy = self.predict_intercept(attacker, goal, defender, defender_velocity)
        saved = self._dynamic
        self.set_dynamic_obstacles(saved + ((ix, iy, block_radius),))
        try:
            return self.plan(attacker, goal, **kw)
        finally:
            self.set_dynamic_obstacles(saved)

    def next_waypoint_index(self, path, position, lookahead: float = .35) -> int:
        if not path:
            return -1
        d = [math.hypot(p[0] - position[0], p[1] - position[1]) for p in path]
        i = min(range(len(path)), key=d.__getitem__)
        while i < len(path) - 1 and d[i] < lookahead:
            i += 1
        return i

    def next_waypoint(self, path, position, lookahead: float = .35):
        i = self.next_waypoint_index(path, position, lookahead)
        return None if i < 0 else path[i]

    @staticmethod
    def path_reference(path, speeds, position, lookahead_distance: float = .35, *, max_speed: float = 4.8):
        """Velocity command (vx, vy) toward the lookahead point at the profile
        speed of the nearest path segment."""
        if not path:
            return 0., 0.
        best, seg_t, seg_i = float("inf"), 0., 0
        for i in range(len(path) - 1):
            ax, ay = path[i]
            bx, by = path[i + 1]
            vx, vy = bx - ax, by - ay
            ll = vx * vx + vy * vy
            t = 0. if ll < 1e-12 else max(0., min(1., ((position[0] - ax) * vx + (position[1] - ay) * vy) / ll))
            d = math.hypot(ax + vx * t - position[0], ay + vy * t - position[1])
            if d < best:
                best, seg_t, seg_i = d, t, i
        # walk lookahead_distance along the path from the projection
        remaining = lookahead_distance
        i, t = seg_i, seg_t
        tx, ty = path[-1]
        while i < len(path) - 1:
            ax, ay = path[i]
            bx, by = path[i + 1]
            seg = math.hypot(bx - ax, by - ay)
            left = seg * (1 - t)
            if left >= remaining:
                f = t + remaining / max(seg, 1e-9)
                tx, ty = ax + (bx - ax) * f, ay + (by - ay) * f
                break
            remaining -= left
            i, t = i + 1, 0.
        speed = min(max_speed, speeds[min(seg_i + 1, len(speeds) - 1)] if speeds else max_speed)
        dx, dy = tx - position[0], ty - position[1]
        d = math.hypot(dx, dy)
        if d < 1e-9:
            return 0., 0.
        speed = min(speed, d / .02 if seg_i >= len(path) - 2 else speed)
        return dx / d * speed, dy / d * speed
