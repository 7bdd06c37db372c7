"""Verified checkpoint loading.

``load_verified(path)`` reads a ``policy.pt``-style payload and refuses, with
a ``CheckpointError`` that names the file, anything that is not a complete
checkpoint: a missing or truncated file, bytes that do not unpickle, a payload
without ``model_state_dict``, or weights whose SHA-256 tree digest differs
from the ``weights_sha256`` recorded when the checkpoint was written (payloads
written before that key existed load without the check). Training resume,
evaluation and population loading go through it, so a corrupt file stops a
run with a clear error instead of training from damaged weights.
"""
from __future__ import annotations

import os
from pathlib import Path

import torch


class CheckpointError(RuntimeError):
    pass


def load_verified(path, *, map_location="cpu", weights_only: bool = True, require_digest: bool = False) -> dict:
    p = Path(path)
    if not p.is_file():
        raise CheckpointError(f"checkpoint {p} does not exist")
    if os.path.getsize(p) == 0:
        raise CheckpointError(f"checkpoint {p} is empty")
    try:
        payload = torch.load(p, map_location=map_location, weights_only=weights_only)
    except Exception as exc:             # truncated zip, bad pickle, foreign format
        raise CheckpointError(f"checkpoint {p} is unreadable ({type(exc).__name__}: {exc})") from exc
    if not isinstance(payload, dict) or not isinstance(payload.get("model_state_dict"), dict):
        raise CheckpointError(f"checkpoint {p} has no model_state_dict")
    recorded = payload.get("weights_sha256")
    if recorded is None:
        if require_digest:
            raise CheckpointError(f"checkpoint {p} carries no weights_sha256")
        return payload
    from .provenance import state_dict_digest
    actual = state_dict_digest(payload["model_state_dict"])
    if actual != recorded:
        raise CheckpointError(f"checkpoint {p} weights do not match their recorded SHA-256 "
                              f"({actual[:12]} != {str(recorded)[:12]})")
    return payload
