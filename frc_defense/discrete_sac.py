"""Compatibility import path: ``frc_defense.discrete_sac`` -> ``autodrive_b200.train.sac``."""
from autodrive_b200.train.sac import *  # noqa: F401,F403
