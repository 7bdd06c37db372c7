"""B200-native FRC REBUILT simulator and defense-policy trainer."""
__version__ = "0.1.0"
