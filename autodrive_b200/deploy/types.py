"""Data contracts between a robot's runtime and a learned chassis policy.

Field names and defaults match frc_defense/types.py:9-73 so a robot program
written against either package exchanges the same values: poses in metres and
radians in the field frame, velocities in m/s and rad/s, limits positive.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Protocol


def _finite(*values: float) -> bool:
    return all(math.isfinite(v) for v in values)


@dataclass(frozen=True)
class RobotState:
    x: float
    y: float
    theta: float
    vx: float = 0.0
    vy: float = 0.0
    omega: float = 0.0

    def values(self) -> tuple[float, ...]:
        return (self.x, self.y, self.theta, self.vx, self.vy, self.omega)


@dataclass(frozen=True)
class Obstacle:
    x: float
    y: float
    radius: float


@dataclass(frozen=True)
class RobotParameters:
    length: float = 0.9
    width: float = 0.9
    max_speed: float = 4.8
    max_acceleration: float = 8.0
    max_omega: float = 8.0
    max_alpha: float = 18.0
    mass: float = 55.0

    def __post_init__(self):
        limits = (self.length, self.width, self.max_speed, self.max_acceleration, self.max_omega,
                  self.max_alpha, self.mass)
        if not (_finite(*limits) and min(limits) > 0):
            raise ValueError("robot dimensions, mass, and motion limits must be finite and positive")


@dataclass(frozen=True)
class WorldState:
    own: RobotState
    opponent: RobotState
    timestamp: float
    field_length: float
    field_width: float
    obstacles: tuple[Obstacle, ...] = ()
    opponent_params: RobotParameters | None = None

    def is_valid(self) -> bool:
        """All numbers finite, field extent positive, obstacle radii positive."""
        flat = self.own.values() + self.opponent.values() + (self.field_length, self.field_width)
        for ob in self.obstacles:
            flat += (ob.x, ob.y, ob.radius)
        return (_finite(*flat) and self.field_length > 0 and self.field_width > 0
                and all(ob.radius > 0 for ob in self.obstacles))


@dataclass(frozen=True)
class Objective:
    x: float
    y: float
    radius: float = 0.5

    def __post_init__(self):
        if not _finite(self.x, self.y, self.radius) or self.radius <= 0:
            raise ValueError("objective coordinates must be finite and radius positive")


@dataclass(frozen=True)
class ChassisCommand:
    vx: float = 0.0
    vy: float = 0.0
    omega: float = 0.0

    def is_finite(self) -> bool:
        return _finite(self.vx, self.vy, self.omega)


class DefensePolicy(Protocol):
    def predict(self, state: WorldState, params: RobotParameters, goal: Objective) -> ChassisCommand: ...
