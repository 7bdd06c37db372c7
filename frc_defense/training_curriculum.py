"""Compatibility import path: ``frc_defense.training_curriculum`` -> ``autodrive_b200.train.curriculum``."""
from autodrive_b200.train.curriculum import *  # noqa: F401,F403
