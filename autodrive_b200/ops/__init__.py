"""Native operator access: the in-tree sm_100a extension and its host twins."""
from .ext import extension, require_extension  # noqa: F401
