"""Reference-compatible public surface backed by the B200-native implementation.

Module names mirror the reference package (``frc_defense.tensor_training``,
``frc_defense.tensor_3v3``, ``frc_defense.tensor_sim`` ...) so existing
scripts switch by import path alone. All code lives in ``autodrive_b200``.
"""
