"""Compatibility import path: ``frc_defense.architecture_benchmark`` -> ``autodrive_b200.train.architecture_study``."""
from autodrive_b200.train.architecture_study import *  # noqa: F401,F403
from autodrive_b200.train.architecture_study import evaluate, main, train_case  # noqa: F401
