"""Host-side route planning."""
from .adstar import ADStarPlanner  # noqa: F401
