"""Compatibility import path: ``frc_defense.meco_device_lease`` -> ``autodrive_b200.meco.ops``."""
from autodrive_b200.meco.ops import *  # noqa: F401,F403
