"""Safe command boundary between a learned policy and the drivetrain.

Behaviour (frc_defense/runtime.py:27-89):

* a state older than ``stale_after`` seconds, stamped more than 50 ms in the
  future, or holding a non-finite value is not given to the policy;
* a policy that raises or returns a non-finite command is replaced by the
  manual command when one is supplied (and finite), else by zero;
* every command, policy or fallback, then passes the limiter: per-axis and
  planar speed limit, acceleration limit and turn-rate / turn-acceleration
  limits against the previous output, and no motion further into a field wall
  the chassis footprint already touches (tangential motion is kept).

The result records the raw command, the limited command and the reason
("policy", "stale-state", "invalid-output", "policy-error").
"""
from __future__ import annotations

import math
import time
from dataclasses import asdict, dataclass
from typing import Callable

from .types import ChassisCommand, DefensePolicy, Objective, RobotParameters, WorldState

FUTURE_TOLERANCE_S = 0.05


def _clamp(v: float, limit: float) -> float:
    return min(limit, max(-limit, v))


@dataclass(frozen=True)
class CommandResult:
    raw: ChassisCommand
    constrained: ChassisCommand
    reason: str


class CommandLimiter:
    """Kinematic and field-boundary limits applied to successive commands."""

    def __init__(self, params: RobotParameters, dt: float):
        self.params, self.dt = params, dt
        self.last = ChassisCommand()

    def _boundary_margins(self, theta: float) -> tuple[float, float]:
        p = self.params
        c, s = abs(math.cos(theta)), abs(math.sin(theta))
        return .5 * (p.length * c + p.width * s), .5 * (p.length * s + p.width * c)

    def __call__(self, cmd: ChassisCommand, state: WorldState) -> ChassisCommand:
        p, last = self.params, self.last
        vx, vy = _clamp(cmd.vx, p.max_speed), _clamp(cmd.vy, p.max_speed)
        planar = math.hypot(vx, vy)
        if planar > p.max_speed:
            vx, vy = vx * (p.max_speed / planar), vy * (p.max_speed / planar)
        step_v = p.max_acceleration * self.dt
        vx = last.vx + _clamp(vx - last.vx, step_v)
        vy = last.vy + _clamp(vy - last.vy, step_v)
        omega = last.omega + _clamp(_clamp(cmd.omega, p.max_omega) - last.omega, p.max_alpha * self.dt)
        mx, my = self._boundary_margins(state.own.theta)
        x, y = state.own.x, state.own.y
        if (x <= mx and vx < 0) or (x >= state.field_length - mx and vx > 0):
            vx = 0.0
        if (y <= my and vy < 0) or (y >= state.field_width - my and vy > 0):
            vy = 0.0
        self.last = ChassisCommand(vx, vy, omega)
        return self.last


class SafePolicyRunner:
    """Constrain policy output and fall back to manual/zero on stale or invalid state."""

    def __init__(self, policy: DefensePolicy, params: RobotParameters, *, dt: float = 0.02,
                 stale_after: float = 0.15, clock: Callable[[], float] = time.time,
                 logger: Callable[[dict], None] | None = None):
        if dt <= 0 or stale_after <= 0:
            raise ValueError("dt and stale_after must be positive")
        self.policy, self.params = policy, params
        self.dt, self.stale_after, self.clock, self.logger = dt, stale_after, clock, logger
        self.limiter = CommandLimiter(params, dt)

    @property
    def previous(self) -> ChassisCommand:
        return self.limiter.last

    def _stale(self, state: WorldState, now: float) -> bool:
        ts = state.timestamp
        return not math.isfinite(ts) or now - ts > self.stale_after or ts > now + FUTURE_TOLERANCE_S

    def predict(self, state: WorldState, goal: Objective, *, manual: ChassisCommand | None = None) -> CommandResult:
        now = self.clock()
        zero = ChassisCommand()
        stale = self._stale(state, now)
        valid = state.is_valid() and math.isfinite(goal.x) and math.isfinite(goal.y)
        if stale:
            reason, raw = "stale-state", zero
        elif not valid:
            reason, raw = "invalid-output", zero
        else:
            try:
                raw = self.policy.predict(state, self.params, goal)
                reason = "policy" if isinstance(raw, ChassisCommand) and raw.is_finite() else "invalid-output"
            except Exception:  # noqa: BLE001 - any policy failure degrades to the fallback
                reason, raw = "policy-error", zero
        if reason != "policy":
            raw = manual if manual is not None and manual.is_finite() else zero
        limited = self.limiter(raw, state)
        result = CommandResult(raw, limited, reason)
        if self.logger is not None:
            self.logger({"timestamp": now, "raw": asdict(raw), "constrained": asdict(limited), "reason": reason})
        return result
