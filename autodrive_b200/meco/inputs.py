"""Learning inputs for the MECO scorers from a TensorThreeVsThreeEnv.

* ``build_raster(env, slot)``  [n, 6, H, W] at 0.3302 m cells: solid field
  structure, bumps, FUEL-track density (perception), own robot, teammates,
  tracked opponent;
* ``build_globals(env, slot)`` [n, 7]: match progress, own / enemy HUB
  active, load fraction, own speed fraction, score difference, time to the
  next HUB switch;
* ``safe_action_candidates(env, slot)`` the strategic actions as a candidate
  table (ids, validity from the action mask, 16 features);
* ``se2_lattice(raster, stride)`` an SE(2) lattice graph over coarse cells x 8
  headings (translation edges along the heading, rotation edges to +-1 bin)
  with region ids for the A2 / A3 graph tracks.
"""
from __future__ import annotations

import math

import torch

from .tracks import CANDIDATE_FEATURES

CELL = .3302


def _grid(env):
    return math.ceil(env.field_width / CELL), math.ceil(env.field_length / CELL)


def build_raster(env, slot: int) -> torch.Tensor:
    h, w = _grid(env)
    n, dev, ws = env.n, env.device, env.ws
    out = torch.zeros((n, 6, h, w), device=dev)
    ys = (torch.arange(h, device=dev) + .5) * CELL
    xs = (torch.arange(w, device=dev) + .5) * CELL
    gy, gx = torch.meshgrid(ys, xs, indexing="ij")
    for ch, kinds in ((0, ("hub", "upright", "support")), (1, ("bump",))):
        for b in env.field_boxes:
            if b.kind in kinds:
                hit = ((gx - b.x).abs() <= b.length / 2 + CELL / 2) & ((gy - b.y).abs() <= b.width / 2 + CELL / 2)
                out[:, ch] = torch.maximum(out[:, ch], hit.float())

    def cells(xy):
        c = (xy / CELL).floor().long()
        return c[..., 1].clamp(0, h - 1) * w + c[..., 0].clamp(0, w - 1)

    flat = out.flatten(2)
    mask = ws["t_mask"][:, slot].bool()
    tpos = ws["t_pos"][:, slot].transpose(1, 2)
    cnt = torch.zeros((n, h * w), device=dev).scatter_add_(1, cells(torch.nan_to_num(tpos)), mask.float())
    flat[:, 2] = cnt.clamp(max=4) / 4
    own = ws["policy_pose"][:, slot, :2]
    flat[:, 3].scatter_(1, cells(own)[:, None], 1.)
    team = int(env.team_ids[slot])
    mates = [r for r in range(6) if r != slot and int(env.team_ids[r]) == team]
    for r in mates:
        flat[:, 4].scatter_(1, cells(ws["policy_pose"][:, r, :2])[:, None], 1.)
    ov = ws["o_valid"][:, slot].reshape(n).float()
    flat[:, 5].scatter_add_(1, cells(torch.nan_to_num(ws["o_pose"][:, slot, :2]))[:, None], ov[:, None])
    return out


def build_globals(env, slot: int) -> torch.Tensor:
    ws = env.ws
    team = int(env.team_ids[slot])
    el = ws["g_time"][:, 0]
    held = (ws["f_active"].bool() & (ws["f_owner"] == slot)).sum(-1).float()
    cap = float(env.robot_fuel_capacities[slot])
    speed = ws["r_vel"][:, slot, :2].norm(dim=-1) / ws["r_param"][:, slot, 3].clamp_min(.1)
    sc = ws["g_scores"][:, 2:4].float()
    diff = (sc[:, team] - sc[:, 1 - team]) / 50.
    to_switch = (30. - torch.remainder((el - 20.).clamp_min(0.), 30.)) / 30.
    return torch.stack((el / 160., ws["g_hub"][:, team].float(), ws["g_hub"][:, 1 - team].float(),
                        held / max(cap, 1.), speed.clamp(0, 1), diff, to_switch), -1)


def safe_action_candidates(env, slot: int):
    """(ids, valid [n, 8] bool, features [n, 8, 16])."""
    obs = env.ws["obs"][:, slot]
    valid = obs[:, -8:] > .5
    g = build_globals(env, slot)
    n = env.n
    onehot = torch.eye(8, device=env.device)[None].expand(n, -1, -1)
    feats = torch.cat((valid[..., None].float(), onehot, g[:, None].expand(-1, 8, -1)), -1)
    assert feats.shape[-1] == CANDIDATE_FEATURES
    return tuple(f"action-{k}" for k in range(8)), valid, feats


def se2_lattice(raster: torch.Tensor, stride: int = 4, regions: int = 64):
    """Graph inputs for the SE(2) tracks from a raster [b, 6, H, W]."""
    b, _, H, W = raster.shape
    coarse = torch.nn.functional.avg_pool2d(raster, stride, ceil_mode=True)
    h, w = coarse.shape[-2:]
    cells = h * w
    n = cells * 8
    dev = raster.device
    cy, cx = torch.meshgrid(torch.arange(h, device=dev), torch.arange(w, device=dev), indexing="ij")
    cy, cx = cy.reshape(-1).repeat_interleave(8), cx.reshape(-1).repeat_interleave(8)
    hb = torch.arange(8, device=dev).repeat(cells)
    vals = coarse.flatten(2).transpose(1, 2).repeat_interleave(8, 1)            # [b, n, 6]
    feats = torch.cat((vals, (cx.float() / max(w - 1, 1))[None, :, None].expand(b, -1, -1),
                       (cy.float() / max(h - 1, 1))[None, :, None].expand(b, -1, -1),
                       hb.float()[None, :, None].expand(b, -1, -1)), -1)
    ang = hb.float() * (2 * math.pi / 8)
    dx, dy = torch.round(torch.cos(ang)).long(), torch.round(torch.sin(ang)).long()
    nx, ny = cx + dx, cy + dy
    fwd = torch.where((nx >= 0) & (nx < w) & (ny >= 0) & (ny < h), (ny * w + nx) * 8 + hb, torch.full_like(hb, -1))
    base = (cy * w + cx) * 8
    left, right = base + (hb + 1) % 8, base + (hb + 7) % 8
    edges = torch.stack((fwd, left, right), -1)[None].expand(b, -1, -1).contiguous()
    edge_mask = edges >= 0
    ry = (cy * 8 // max(h, 1)).clamp(max=7)
    rx = (cx * 8 // max(w, 1)).clamp(max=7)
    region_ids = (ry * 8 + rx)[None].expand(b, -1).contiguous() % regions
    # coarse region graph: 8-neighbourhood on the 8 x 8 region grid
    rgy, rgx = torch.meshgrid(torch.arange(8, device=dev), torch.arange(8, device=dev), indexing="ij")
    rgy, rgx = rgy.reshape(-1), rgx.reshape(-1)
    cedges = []
    for ddx, ddy in ((1, 0), (-1, 0), (0, 1), (0, -1)):
        ax, ay = rgx + ddx, rgy + ddy
        cedges.append(torch.where((ax >= 0) & (ax < 8) & (ay >= 0) & (ay < 8), ay * 8 + ax, torch.full_like(ax, -1)))
    coarse_edges = torch.stack(cedges, -1)[None].expand(b, -1, -1).contiguous()
    node_valid = torch.ones((b, n), dtype=torch.bool, device=dev)
    return {"node_features": feats, "edges": edges, "edge_mask": edge_mask, "region_ids": region_ids,
            "coarse_edges": coarse_edges, "coarse_edge_mask": coarse_edges >= 0, "node_valid": node_valid}
