"""Plan-A exact shortest paths: host twin vs a Python Dijkstra, GPU vs host (exact fp64)."""
import heapq
import math

import pytest
import torch

from autodrive_b200.meco.plan_a import pose_graph, route, shortest_paths


def _random_csr(n, deg, seed):
    g = torch.Generator().manual_seed(seed)
    cols = torch.randint(0, n, (n, deg), generator=g)
    row = torch.arange(0, n * deg + 1, deg, dtype=torch.int64)
    return row, cols.reshape(-1).to(torch.int32)


def _dijkstra(row, col, w, s, n):
    d = [math.inf] * n
    d[s] = 0.
    pq = [(0., s)]
    while pq:
        du, u = heapq.heappop(pq)
        if du > d[u]:
            continue
        for e in range(int(row[u]), int(row[u + 1])):
            v = int(col[e])
            c = du + float(w[e])
            if c < d[v]:
                d[v] = c
                heapq.heappush(pq, (c, v))
    return d


def test_host_twin_matches_python_dijkstra():
    n = 300
    row, col = _random_csr(n, 4, 1)
    w = torch.rand(2, col.numel(), dtype=torch.float64, generator=torch.Generator().manual_seed(2)) * 3
    src = torch.tensor([0, 17])
    dist, pred, _ = shortest_paths(row, col, w, src)
    for gi in range(2):
        ref = _dijkstra(row, col, w[gi], int(src[gi]), n)
        assert dist[gi].tolist() == ref
        for v in range(n):
            if 0 < ref[v] < math.inf:
                u = int(pred[gi, v])
                e = [e for e in range(int(row[u]), int(row[u + 1])) if int(col[e]) == v]
                assert any(ref[u] + float(w[gi, k]) == ref[v] for k in e)


def test_pose_graph_route():
    blocked = torch.zeros(8, 12, dtype=torch.bool)
    blocked[2:7, 6] = True
    row, col, w = pose_graph(blocked, .3)
    src = (1 * 12 + 1) * 8 + 0
    dist, pred, _ = shortest_paths(row, col, w[None], torch.tensor([src]))
    goal_cell = 4 * 12 + 10
    best = min(range(8), key=lambda h: float(dist[0, goal_cell * 8 + h]))
    path = route(pred[0], goal_cell * 8 + best)
    assert path[0] == src and path[-1] == goal_cell * 8 + best
    cells = {p // 8 for p in path}
    assert not any(bool(blocked[c // 12, c % 12]) for c in cells)


@pytest.mark.gpu
def test_gpu_matches_host_exactly():
    n = 5000
    row, col = _random_csr(n, 6, 3)
    w = torch.rand(8, col.numel(), dtype=torch.float64, generator=torch.Generator().manual_seed(4)) * 2
    src = torch.randint(0, n, (8,), generator=torch.Generator().manual_seed(5))
    d_h, p_h, _ = shortest_paths(row, col, w, src)
    d_g, p_g, rounds = shortest_paths(row.cuda(), col.cuda(), w.cuda(), src.cuda())
    assert torch.equal(d_g.cpu(), d_h)
    assert torch.equal(p_g.cpu(), p_h)
    assert int(rounds.max()) < n
