"""MECO Plan A: exact shortest routes on an SE(2) pose lattice.

``pose_graph(blocked, resolution, ...)`` builds the lattice over free grid
cells x 8 headings: translation edges one cell along the current heading
(cost = distance / speed) and rotation edges to the neighbouring heading bins
(cost = 45 degrees / turn rate), as one CSR shared by every world;
``shortest_paths`` runs the batched fp64 kernel (``csrc/plan_a.cu``: one CTA
per graph, frontier relaxation, exact distances, predecessors by tightness)
or its Dijkstra host twin; ``route(pred, target)`` walks predecessors back.
Reference: frc_defense/meco_plan_a_shortest_path.py, meco_plan_a_shortest_path_hip.py:55.
"""
from __future__ import annotations

import math

import torch

from ..ops import require_extension

DIRS = [(1, 0), (1, 1), (0, 1), (-1, 1), (-1, 0), (-1, -1), (0, -1), (1, -1)]


def pose_graph(blocked: torch.Tensor, resolution: float, speed: float = 4., turn_rate: float = 8.):
    """CSR (row_ptr int64 [n+1], col int32 [E], base weights float64 [E]) over
    node id = (y * W + x) * 8 + heading for every grid cell (blocked cells
    keep no out-edges and receive none)."""
    H, W = blocked.shape
    blk = blocked.bool().cpu()
    rows, cols, wts = [0], [], []
    rot = (math.pi / 4) / turn_rate
    for y in range(H):
        for x in range(W):
            for hb in range(8):
                if not bool(blk[y, x]):
                    dx, dy = DIRS[hb]
                    nx, ny = x + dx, y + dy
                    if 0 <= nx < W and 0 <= ny < H and not bool(blk[ny, nx]) and \
                            not (dx and dy and (bool(blk[y, nx]) or bool(blk[ny, x]))):
                        cols.append((ny * W + nx) * 8 + hb)
                        wts.append(resolution * math.hypot(dx, dy) / speed)
                    for r in (1, 7):
                        cols.append((y * W + x) * 8 + (hb + r) % 8)
                        wts.append(rot)
                rows.append(len(cols))
    return (torch.tensor(rows, dtype=torch.int64), torch.tensor(cols, dtype=torch.int32),
            torch.tensor(wts, dtype=torch.float64))


def shortest_paths(row_ptr, col, weights, sources):
    """weights [G, E] float64, sources [G] int64 -> (dist [G, n], pred [G, n], rounds [G])."""
    return require_extension().plan_a_shortest_paths(row_ptr.contiguous(), col.contiguous(),
                                                     weights.contiguous(), sources.contiguous())


def route(pred: torch.Tensor, target: int) -> list[int]:
    """Node ids from the source to `target` (empty when unreachable)."""
    p = pred.tolist()
    out, v = [], int(target)
    seen = set()
    while v >= 0 and v not in seen:
        out.append(v)
        seen.add(v)
        v = p[v]
    out.reverse()
    return out
