"""Compatibility import path: ``frc_defense.meco_request_capture`` -> ``autodrive_b200.meco.adapter``."""
from autodrive_b200.meco.adapter import *  # noqa: F401,F403
