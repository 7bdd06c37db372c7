"""Compatibility import path: ``frc_defense.learning_inputs`` -> ``autodrive_b200.meco.inputs``."""
from autodrive_b200.meco.inputs import *  # noqa: F401,F403
