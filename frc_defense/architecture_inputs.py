"""Compatibility import path: ``frc_defense.architecture_inputs`` -> ``autodrive_b200.models.perception``."""
from autodrive_b200.models.perception import PerceptionInputs  # noqa: F401
