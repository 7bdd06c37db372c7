"""Compatibility import path: ``frc_defense.meco_external_release_gate`` -> ``autodrive_b200.meco.ops``."""
from autodrive_b200.meco.ops import *  # noqa: F401,F403
