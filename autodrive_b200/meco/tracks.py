"""MECO research scorers and the fail-closed decision adapter.

Parity with frc_defense/meco_tracks.py:808-1988. Five scorer tracks rate
navigation goals or candidates; a deterministic arbiter keeps the final say:

* ``A1MultiscaleUNetGRU``      raster U-Net (3 scales) with a GRU context:
                               dense per-cell utility / penalty for 8 headings
                               and 5 behaviour logits;
* ``A2StructuredSE2UNetGRU``   SE(2) lattice graph U-Net: fine message passing,
                               region pooling, coarse message passing, region
                               self-attention, GRU, per-node decoder;
* ``A3HierarchicalSE2GNNGRU``  deeper fine propagation with region attention;
* ``CandidateMLPGRU`` (C1)     per-candidate MLP over candidate features and
                               the GRU context;
* ``C2MapCrossAttentionGRU``   candidates cross-attend to raster map tokens.

Every track returns ``utility`` (higher is better), ``penalty`` (>= 0),
``behavior_logits`` and the next GRU ``hidden`` state. ``choose_candidate``
takes the arg-max of utility - penalty over the caller's safe candidates and
falls back to the deterministic choice whenever the scorer output is missing,
non-finite, stale or does not cover the candidates ("fail closed").
``opponent_forecast`` predicts an opponent's endpoint under constant-velocity
or multi-hypothesis constant-turn-rate models; ``opponent_risk_penalty``
turns it into a goal penalty.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Mapping

import torch
from torch import nn
from torch.nn import functional as F

HIDDEN = 64
RASTER_CHANNELS = 6
GLOBALS = 7
CANDIDATE_FEATURES = 16
BEHAVIORS = 5


def _groups(c: int) -> int:
    return 8 if c % 8 == 0 else (4 if c % 4 == 0 else 1)


class ConvBlock(nn.Module):
    def __init__(self, cin: int, cout: int):
        super().__init__()
        self.block = nn.Sequential(nn.Conv2d(cin, cout, 3, padding=1), nn.GroupNorm(_groups(cout), cout), nn.SiLU(),
                                   nn.Conv2d(cout, cout, 3, padding=1), nn.GroupNorm(_groups(cout), cout), nn.SiLU())

    def forward(self, x):
        return self.block(x)


class RecurrentTrack(nn.Module):
    """Per-episode GRU context; the caller resets `hidden` at episode boundaries."""

    def __init__(self):
        super().__init__()
        self.gru = nn.GRUCell(HIDDEN, HIDDEN)

    def forward(self, x, hidden=None):
        if hidden is None:
            hidden = x.new_zeros((x.shape[0], HIDDEN))
        elif hidden.shape != (x.shape[0], HIDDEN) or not bool(torch.isfinite(hidden).all()):
            raise ValueError("GRU hidden state must be finite with shape [batch, 64]")
        return self.gru(x, hidden)


class A1MultiscaleUNetGRU(nn.Module):
    track_id = "A1"

    def __init__(self):
        super().__init__()
        self.enc0, self.enc1, self.enc2 = ConvBlock(RASTER_CHANNELS, 24), ConvBlock(24, 32), ConvBlock(32, HIDDEN)
        self.pool = nn.AvgPool2d(2, ceil_mode=True)
        self.global_mlp = nn.Sequential(nn.Linear(GLOBALS, HIDDEN), nn.SiLU(), nn.Linear(HIDDEN, HIDDEN))
        self.context = RecurrentTrack()
        self.fuse = nn.Conv2d(2 * HIDDEN, HIDDEN, 1)
        self.dec1, self.dec0 = ConvBlock(HIDDEN + 32, 32), ConvBlock(32 + 24, 24)
        self.pose_head = nn.Conv2d(24, 16, 1)      # 8 headings x (utility, penalty)
        self.behavior_head = nn.Linear(HIDDEN, BEHAVIORS)

    def forward(self, raster, globals_, hidden=None, **_):
        x0 = self.enc0(raster)
        x1 = self.enc1(self.pool(x0))
        x2 = self.enc2(self.pool(x1))
        state = self.context(x2.mean((-2, -1)) + self.global_mlp(globals_), hidden)
        x = self.fuse(torch.cat((x2, state[:, :, None, None].expand_as(x2)), 1))
        x = self.dec1(torch.cat((F.interpolate(x, size=x1.shape[-2:], mode="bilinear", align_corners=False), x1), 1))
        x = self.dec0(torch.cat((F.interpolate(x, size=x0.shape[-2:], mode="bilinear", align_corners=False), x0), 1))
        pose = self.pose_head(x).reshape(x.shape[0], 8, 2, *x.shape[-2:])
        return {"utility": pose[:, :, 0], "penalty": F.softplus(pose[:, :, 1]),
                "behavior_logits": self.behavior_head(state), "hidden": state}


class SE2MessageBlock(nn.Module):
    """Mean aggregation of messages along valid directed edges, residual update, LayerNorm."""

    def __init__(self, width: int = HIDDEN):
        super().__init__()
        self.message = nn.Sequential(nn.Linear(width, width), nn.SiLU(), nn.Linear(width, width))
        self.update = nn.Sequential(nn.Linear(2 * width, width), nn.SiLU(), nn.Linear(width, width))
        self.norm = nn.LayerNorm(width)

    def forward(self, nodes, edges, edge_mask, node_valid):
        b, n, w = nodes.shape
        ok = edge_mask & (edges >= 0) & (edges < n)
        idx = edges.clamp(0, n - 1)
        ok = ok & node_valid.gather(1, idx.reshape(b, -1)).reshape_as(idx) & node_valid[:, :, None]
        msg = self.message(nodes)
        gathered = msg.gather(1, idx.reshape(b, -1, 1).expand(-1, -1, w)).reshape(b, n, -1, w)
        m = ok[..., None].to(nodes.dtype)
        agg = (gathered * m).sum(2) / m.sum(2).clamp_min(1.)
        out = self.norm(nodes + self.update(torch.cat((nodes, agg), -1)))
        return torch.where(node_valid[..., None], out, torch.zeros_like(out))


def se2_node_inputs(node_features, globals_, node_valid):
    """[raster(6), x, y in [0,1], heading bin 0..7] + globals -> 17 features
    with the heading as (sin, cos) so bins 7 and 0 are neighbours."""
    if node_features.shape[-1] != 9 or globals_.shape[-1] != GLOBALS:
        raise ValueError("SE(2) nodes need six raster values, x/y, a heading bin and seven globals")
    f = torch.nan_to_num(torch.where(node_valid[..., None], node_features, torch.zeros_like(node_features)))
    ang = f[..., 8].round().clamp(0, 7) * (2 * math.pi / 8)
    return torch.cat((f[..., :6], f[..., 6:8].clamp(0, 1), ang.sin()[..., None], ang.cos()[..., None],
                      torch.nan_to_num(globals_)[:, None].expand(-1, f.shape[1], -1)), -1)


def pool_regions(nodes, region_ids, regions: int, node_valid):
    b, n, w = nodes.shape
    ok = node_valid & (region_ids >= 0) & (region_ids < regions)
    ids = torch.where(ok, region_ids, torch.zeros_like(region_ids))
    pooled = nodes.new_zeros((b, regions, w)).scatter_add_(1, ids[..., None].expand_as(nodes), nodes * ok[..., None])
    counts = nodes.new_zeros((b, regions, 1)).scatter_add_(1, ids[..., None], ok[..., None].to(nodes.dtype))
    occupied = counts.squeeze(-1) > 0
    occupied[:, 0] |= ~occupied.any(-1)
    return pooled / counts.clamp_min(1.), occupied


class _RegionAttention(nn.Module):
    def __init__(self, heads: int):
        super().__init__()
        self.attn = nn.MultiheadAttention(HIDDEN, heads, batch_first=True)

    def forward(self, tokens, occupied):
        out, _ = self.attn(tokens, tokens, tokens, key_padding_mask=~occupied, need_weights=False)
        return out


class A2StructuredSE2UNetGRU(nn.Module):
    track_id = "A2"

    def __init__(self, region_tokens: int = 64, heads: int = 4):
        super().__init__()
        if not 32 <= region_tokens <= 128 or HIDDEN % heads:
            raise ValueError("A2 needs 32-128 regions and a head count dividing 64")
        self.region_tokens = region_tokens
        self.lift = nn.Sequential(nn.Linear(17, HIDDEN), nn.SiLU(), nn.Linear(HIDDEN, HIDDEN))
        self.fine_layers = nn.ModuleList([SE2MessageBlock(), SE2MessageBlock()])
        self.coarse_layer = SE2MessageBlock()
        self.attention = _RegionAttention(heads)
        self.context = RecurrentTrack()
        self.decoder = nn.Sequential(nn.Linear(3 * HIDDEN, HIDDEN), nn.SiLU(), nn.Linear(HIDDEN, 2))
        self.behavior_head = nn.Linear(HIDDEN, BEHAVIORS)

    def forward(self, node_features, edges, edge_mask, region_ids, globals_, coarse_edges, coarse_edge_mask,
                node_valid, hidden=None, **_):
        nodes = self.lift(se2_node_inputs(node_features, globals_, node_valid)) * node_valid[..., None]
        for layer in self.fine_layers:
            nodes = layer(nodes, edges, edge_mask, node_valid)
        coarse, occupied = pool_regions(nodes, region_ids, self.region_tokens, node_valid)
        coarse = self.coarse_layer(coarse, coarse_edges, coarse_edge_mask, occupied)
        att = self.attention(coarse, occupied)
        state = self.context((att * occupied[..., None]).sum(1) / occupied.sum(1, keepdim=True).clamp_min(1), hidden)
        ids = torch.where((region_ids >= 0) & (region_ids < self.region_tokens), region_ids, torch.zeros_like(region_ids))
        up = coarse.gather(1, ids[..., None].expand(-1, -1, HIDDEN))
        dec = self.decoder(torch.cat((nodes, up, state[:, None].expand(-1, nodes.shape[1], -1)), -1))
        return {"utility": dec[..., 0], "penalty": F.softplus(dec[..., 1]),
                "behavior_logits": self.behavior_head(state), "hidden": state}


class A3HierarchicalSE2GNNGRU(nn.Module):
    track_id = "A3"

    def __init__(self, region_tokens: int = 64, heads: int = 4):
        super().__init__()
        self.region_tokens = region_tokens
        self.lift = nn.Sequential(nn.Linear(17, HIDDEN), nn.SiLU(), nn.Linear(HIDDEN, HIDDEN))
        self.layers = nn.ModuleList([SE2MessageBlock() for _ in range(3)])
        self.region_attention = _RegionAttention(heads)
        self.context = RecurrentTrack()
        self.decoder = nn.Sequential(nn.Linear(3 * HIDDEN, HIDDEN), nn.SiLU(), nn.Linear(HIDDEN, 2))
        self.behavior_head = nn.Linear(HIDDEN, BEHAVIORS)

    def forward(self, node_features, edges, edge_mask, region_ids, globals_, node_valid, hidden=None, **_):
        nodes = self.lift(se2_node_inputs(node_features, globals_, node_valid)) * node_valid[..., None]
        for layer in self.layers:
            nodes = layer(nodes, edges, edge_mask, node_valid)
        coarse, occupied = pool_regions(nodes, region_ids, self.region_tokens, node_valid)
        att = self.region_attention(coarse, occupied)
        state = self.context((att * occupied[..., None]).sum(1) / occupied.sum(1, keepdim=True).clamp_min(1), hidden)
        ids = torch.where((region_ids >= 0) & (region_ids < self.region_tokens), region_ids, torch.zeros_like(region_ids))
        up = att.gather(1, ids[..., None].expand(-1, -1, HIDDEN))
        dec = self.decoder(torch.cat((nodes, up, state[:, None].expand(-1, nodes.shape[1], -1)), -1))
        return {"utility": dec[..., 0], "penalty": F.softplus(dec[..., 1]),
                "behavior_logits": self.behavior_head(state), "hidden": state}


class CandidateMLPGRU(nn.Module):
    track_id = "C1"

    def __init__(self, candidate_features: int = CANDIDATE_FEATURES, width: int = HIDDEN):
        super().__init__()
        self.global_mlp = nn.Sequential(nn.Linear(GLOBALS, width), nn.SiLU(), nn.Linear(width, width))
        self.context = RecurrentTrack()
        self.candidate = nn.Sequential(nn.Linear(candidate_features + width, width), nn.SiLU(),
                                       nn.Linear(width, width), nn.SiLU(), nn.Linear(width, 2))
        self.behavior_head = nn.Linear(width, BEHAVIORS)

    def forward(self, globals_, candidate_features, hidden=None, **_):
        state = self.context(self.global_mlp(globals_), hidden)
        x = torch.cat((candidate_features, state[:, None].expand(-1, candidate_features.shape[1], -1)), -1)
        out = self.candidate(x)
        return {"utility": out[..., 0], "penalty": F.softplus(out[..., 1]),
                "behavior_logits": self.behavior_head(state), "hidden": state}


class C2MapCrossAttentionGRU(nn.Module):
    track_id = "C2"

    def __init__(self, candidate_features: int = CANDIDATE_FEATURES, tokens: int = 64, heads: int = 4):
        super().__init__()
        self.tokens = tokens
        self.map_encoder = nn.Sequential(ConvBlock(RASTER_CHANNELS, 32), nn.AvgPool2d(2, ceil_mode=True),
                                         ConvBlock(32, HIDDEN))
        self.token_pool = nn.AdaptiveAvgPool2d((4, tokens // 4))
        self.global_mlp = nn.Sequential(nn.Linear(GLOBALS, HIDDEN), nn.SiLU(), nn.Linear(HIDDEN, HIDDEN))
        self.context = RecurrentTrack()
        self.query = nn.Linear(candidate_features + HIDDEN, HIDDEN)
        self.cross = nn.MultiheadAttention(HIDDEN, heads, batch_first=True)
        self.head = nn.Sequential(nn.Linear(2 * HIDDEN, HIDDEN), nn.SiLU(), nn.Linear(HIDDEN, 2))
        self.behavior_head = nn.Linear(HIDDEN, BEHAVIORS)

    def forward(self, raster, globals_, candidate_features, hidden=None, **_):
        mp = self.token_pool(self.map_encoder(raster)).flatten(2).transpose(1, 2)   # [B, tokens, 64]
        state = self.context(mp.mean(1) + self.global_mlp(globals_), hidden)
        q = self.query(torch.cat((candidate_features, state[:, None].expand(-1, candidate_features.shape[1], -1)), -1))
        att, _ = self.cross(q, mp, mp, need_weights=False)
        out = self.head(torch.cat((q, att), -1))
        return {"utility": out[..., 0], "penalty": F.softplus(out[..., 1]),
                "behavior_logits": self.behavior_head(state), "hidden": state}


TRACKS = {"A1": A1MultiscaleUNetGRU, "A2": A2StructuredSE2UNetGRU, "A3": A3HierarchicalSE2GNNGRU,
          "C1": CandidateMLPGRU, "C2": C2MapCrossAttentionGRU}


def make_meco_track(track: str, **kwargs) -> nn.Module:
    if track not in TRACKS:
        raise ValueError(f"unknown MECO track {track!r}; choose from {sorted(TRACKS)}")
    return TRACKS[track](**kwargs)


# --------------------------------------------------------------------------- decisions
@dataclass(frozen=True)
class DecisionRequest:
    candidate_ids: tuple[str, ...]
    valid_mask: tuple[bool, ...]
    deterministic_choice: str
    observation_time: float
    max_age_s: float = .25


@dataclass(frozen=True)
class ScorerOutput:
    candidate_ids: tuple[str, ...]
    utility: tuple[float, ...]
    penalty: tuple[float, ...]
    time: float


def candidate_policy_logits(utility: torch.Tensor, valid_mask: torch.Tensor, penalty: torch.Tensor | None = None,
                            temperature: float = 1.) -> torch.Tensor:
    score = utility - (penalty if penalty is not None else 0.)
    return (score / max(temperature, 1e-6)).masked_fill(~valid_mask.bool(), torch.finfo(score.dtype).min)


def choose_candidate(request: DecisionRequest, output: ScorerOutput | None) -> tuple[str, str]:
    """(chosen id, reason). The scorer's arg-max over valid candidates, else the
    deterministic choice: missing / stale / mismatched / non-finite output."""
    if output is None:
        return request.deterministic_choice, "no-scorer-output"
    if output.candidate_ids != request.candidate_ids:
        return request.deterministic_choice, "candidate-mismatch"
    if request.observation_time - output.time > request.max_age_s or output.time > request.observation_time + 1e-6:
        return request.deterministic_choice, "stale-output"
    best, best_score = None, -math.inf
    for cid, ok, u, p in zip(request.candidate_ids, request.valid_mask, output.utility, output.penalty):
        if not ok:
            continue
        if not (math.isfinite(u) and math.isfinite(p)) or p < 0:
            return request.deterministic_choice, "invalid-output"
        if u - p > best_score:
            best, best_score = cid, u - p
    if best is None:
        return request.deterministic_choice, "no-valid-candidate"
    return best, "scorer"


# --------------------------------------------------------------------------- opponent forecast
def predict_opponent_endpoint(*, valid: bool, position_xy, velocity_xy, age_s: float, horizon_s: float = 1.,
                              max_age_s: float = 1., max_speed: float = 5.):
    if not valid or age_s > max_age_s:
        return None
    vx, vy = velocity_xy
    sp = math.hypot(vx, vy)
    if sp > max_speed:
        vx, vy = vx * max_speed / sp, vy * max_speed / sp
    t = horizon_s + age_s
    return position_xy[0] + vx * t, position_xy[1] + vy * t


def opponent_forecast(*, mode: str, valid: bool, position_xy, velocity_xy, age_s: float, horizon_s: float = 1.,
                      hypotheses: int = 5, turn_rate_max: float = 2., damping_per_s: float = .2) -> dict | None:
    """Endpoints under `constant_velocity` or `multimodel` (constant turn rates
    spread over [-max, max], velocity damped) with equal weights."""
    if mode not in ("constant_velocity", "multimodel"):
        raise ValueError("mode must be constant_velocity or multimodel")
    if not valid:
        return None
    t = horizon_s + age_s
    if mode == "constant_velocity":
        end = predict_opponent_endpoint(valid=valid, position_xy=position_xy, velocity_xy=velocity_xy, age_s=age_s,
                                        horizon_s=horizon_s, max_age_s=math.inf)
        return {"mode": mode, "endpoints": [end], "weights": [1.]}
    ends = []
    speed = math.hypot(*velocity_xy)
    heading = math.atan2(velocity_xy[1], velocity_xy[0])
    for k in range(hypotheses):
        w = turn_rate_max * (2 * k / max(1, hypotheses - 1) - 1) if hypotheses > 1 else 0.
        x, y, th, v = position_xy[0], position_xy[1], heading, speed
        steps = 20
        dt = t / steps
        for _ in range(steps):
            x += v * math.cos(th) * dt
            y += v * math.sin(th) * dt
            th += w * dt
            v *= math.exp(-damping_per_s * dt)
        ends.append((x, y))
    return {"mode": mode, "endpoints": ends, "weights": [1. / len(ends)] * len(ends)}


def opponent_risk_penalty(goal_xy, forecast: Mapping | None, threat_radius: float = 1.5,
                          max_penalty: float = 2.) -> float | None:
    """Expected closeness of the forecast endpoints to a goal, in [0, max]."""
    if forecast is None:
        return None
    risk = 0.
    for (x, y), w in zip(forecast["endpoints"], forecast["weights"]):
        d = math.hypot(goal_xy[0] - x, goal_xy[1] - y)
        risk += w * max(0., 1. - d / threat_radius)
    return max_penalty * risk
