"""Stage ranges for timeline profilers.

``stage("rollout")`` opens an NVTX range (visible in Nsight Systems and in
ncu's NVTX filters) when ``AUTODRIVE_NVTX=1`` and CUDA is available; otherwise
it costs nothing. Ranges are host markers around kernel launches: inside a
CUDA-graph capture they mark the capture, not each replay.
"""
from __future__ import annotations

import contextlib
import os

import torch

_ENABLED = os.environ.get("AUTODRIVE_NVTX", "0") == "1"


def enabled() -> bool:
    return _ENABLED and torch.cuda.is_available()


def set_enabled(on: bool) -> None:
    global _ENABLED
    _ENABLED = bool(on)


@contextlib.contextmanager
def stage(name: str):
    if not enabled():
        yield
        return
    torch.cuda.nvtx.range_push(name)
    try:
        yield
    finally:
        torch.cuda.nvtx.range_pop()
