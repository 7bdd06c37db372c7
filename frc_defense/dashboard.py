"""Compatibility import path and console entry point: ``frc_defense.dashboard``."""
from autodrive_b200.dashboard.server import create_handler, main, serve  # noqa: F401
from autodrive_b200.dashboard.simulation import field_layout_payload  # noqa: F401

if __name__ == "__main__":
    main()
