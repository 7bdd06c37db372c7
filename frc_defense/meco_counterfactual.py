"""Compatibility import path: ``frc_defense.meco_counterfactual`` -> ``autodrive_b200.meco.train``."""
from autodrive_b200.meco.train import *  # noqa: F401,F403
