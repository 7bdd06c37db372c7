"""Simulator-independent deployment boundary for learned chassis policies.

``types``   plain, frozen data contracts (robot/world state, robot limits,
            objective, chassis command, the ``DefensePolicy`` protocol);
``runtime`` ``SafePolicyRunner``: validates state freshness and values,
            calls the policy, falls back to a manual or zero command, and
            limits speed, acceleration, turn rate and field-boundary motion.
"""
from .runtime import CommandLimiter, CommandResult, SafePolicyRunner  # noqa: F401
from .types import (ChassisCommand, DefensePolicy, Objective, Obstacle, RobotParameters,  # noqa: F401
                    RobotState, WorldState)
