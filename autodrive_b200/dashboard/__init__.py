"""Read-only training dashboard: HTTP JSON API over run directories, 3v3
playback recording jobs and a static Canvas 2-D field viewer."""
from .server import create_handler, main, serve  # noqa: F401
from .simulation import field_layout_payload, record_playback  # noqa: F401
