"""Loader for the in-tree native extension ``autodrive_b200._C``.

The extension is built in place by ``python setup.py build_ext --inplace``
(``__graft_entry__.build`` does this). It holds both the sm_100a kernels and
their host twins. There is deliberately no pure-Python fallback for the
simulator: a missing extension is an error on every device.
"""
from __future__ import annotations

import importlib

_EXT = None
_ERR: Exception | None = None


def extension():
    global _EXT, _ERR
    if _EXT is None and _ERR is None:
        try:
            import torch  # noqa: F401 - loads libc10 / libtorch, which _C links against
            _EXT = importlib.import_module("autodrive_b200._C")
        except Exception as exc:  # noqa: BLE001 - surfaced by require_extension
            _ERR = exc
    return _EXT


def require_extension():
    ext = extension()
    if ext is None:
        raise RuntimeError(
            "autodrive_b200._C is not built; run `python setup.py build_ext --inplace` "
            f"({type(_ERR).__name__}: {_ERR})")
    return ext
