"""Count of this library's own kernel launches issued from Python wrappers.

The Python entry points of the native kernels (tensor-core GEMM, fused
LayerNorm, GAE, fused Adam, peer all-reduce) add the number of kernels each
call launches; benchmarks read the count around a timed region. Simulator
kernels are launched from C++ methods and are counted by their callers.
"""
from __future__ import annotations

_COUNT = [0]


def add(n: int = 1) -> None:
    _COUNT[0] += n


def read() -> int:
    return _COUNT[0]
