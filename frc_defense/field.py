"""REBUILT field geometry under the reference module name."""
from autodrive_b200.field import *  # noqa: F401,F403
