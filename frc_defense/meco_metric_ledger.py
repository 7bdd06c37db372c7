"""Compatibility import path: ``frc_defense.meco_metric_ledger`` -> ``autodrive_b200.meco.train``."""
from autodrive_b200.meco.train import *  # noqa: F401,F403
