"""Provenance digests: SHA-256 (FIPS 180-4) of tensors and state dicts on the
device that holds them (``sha256_chunks`` / ``sha256_tree`` kernels).

``tensor_digest(t)`` is the hex root of a binary hash tree over 64 KB chunks of
the tensor's bytes; ``state_dict_digest(sd)`` hashes the sorted
``name:digest`` lines of every tensor. Identical bytes give identical digests
on CPU and GPU.
"""
from __future__ import annotations

import hashlib

import torch

from ..ops import require_extension


def tensor_digest(t: torch.Tensor, chunk: int = 1 << 16) -> str:
    root = require_extension().sha256_tree(t.detach().contiguous(), int(chunk))
    return bytes(root.cpu().tolist()).hex()


def chunk_digests(t: torch.Tensor, chunk: int = 1 << 16) -> list[str]:
    d = require_extension().sha256_chunks(t.detach().contiguous(), int(chunk)).cpu()
    return [bytes(row.tolist()).hex() for row in d]


def state_dict_digest(state: dict) -> str:
    lines = []
    for name in sorted(state):
        v = state[name]
        if torch.is_tensor(v):
            lines.append(f"{name}:{str(v.dtype)}:{tuple(v.shape)}:{tensor_digest(v)}")
    return hashlib.sha256("\n".join(lines).encode()).hexdigest()
