"""Compatibility import path: ``frc_defense.runtime`` -> ``autodrive_b200.deploy.runtime``."""
from autodrive_b200.deploy.runtime import CommandLimiter, CommandResult, SafePolicyRunner  # noqa: F401
from autodrive_b200.deploy.types import DefensePolicy as Policy  # noqa: F401
