"""Compatibility import path: ``frc_defense.types`` -> ``autodrive_b200.deploy.types``."""
from autodrive_b200.deploy.types import *  # noqa: F401,F403
from autodrive_b200.deploy.types import (ChassisCommand, DefensePolicy, Objective, Obstacle,  # noqa: F401
                                         RobotParameters, RobotState, WorldState)
