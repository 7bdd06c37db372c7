"""Compatibility import path: ``frc_defense.adstar`` -> ``autodrive_b200.planning.adstar``."""
from autodrive_b200.planning.adstar import ADStarPlanner  # noqa: F401
