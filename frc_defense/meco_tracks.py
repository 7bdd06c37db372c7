"""Compatibility import path: ``frc_defense.meco_tracks`` -> ``autodrive_b200.meco.tracks``."""
from autodrive_b200.meco.tracks import *  # noqa: F401,F403
