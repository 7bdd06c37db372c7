"""Perception-only policy inputs for the architecture zoo.

``PerceptionInputs(env, robot_ids)`` turns a TensorThreeVsThreeEnv's simulated
perception into the dictionary the zoo networks read
(frc_defense/architecture_inputs.py:1-188):

* ``scalars``     the 137-feature strategic observation of each robot;
* ``field``       a world-aligned raster (default 32 rows x 64 columns) with 12
                  channels: 0 solid structures, 1 bumps, 2 log FUEL-track count,
                  3-4 mean track velocity / own max speed, 5 mean confidence x
                  freshness, 6 self, 7 teammates, 8 tracked opponent, 9 own HUB,
                  10 enemy HUB, 11 cells holding a retained track;
* ``entities``    every FUEL track slot, self, two teammates and the tracked
                  opponent (fuel_count + 4 tokens) with relative x/y (field
                  units), velocity / own max speed, age / track timeout,
                  confidence, four type flags (self/ally/opponent/FUEL) and x/y
                  extent (field units; a FUEL track's apparent-object extent);
                  ``entity_mask`` marks valid tokens.

Only perception state is read (tracks, the policy's pose estimate, teammates'
reported poses, the opponent track) — never FUEL truth or enemy truth.
"""
from __future__ import annotations

import math

import torch
from torch import Tensor


class PerceptionInputs:
    def __init__(self, env, robot_ids, field_shape: tuple[int, int] = (32, 64)):
        self.env = env
        self.robot_ids = tuple(int(r) for r in robot_ids)
        if not self.robot_ids or len(set(self.robot_ids)) != len(self.robot_ids):
            raise ValueError("robot_ids must be nonempty and unique")
        if any(r < 0 or r >= 6 for r in self.robot_ids):
            raise ValueError("robot_ids must be in [0, 6)")
        dev = env.device
        self.ids = torch.tensor(self.robot_ids, device=dev)
        self.rows, self.cols = int(field_shape[0]), int(field_shape[1])
        self.scales = torch.tensor((env.field_length, env.field_width), device=dev)
        self.grid = torch.tensor((self.cols, self.rows), device=dev, dtype=torch.float32)
        self.timeout = max(float(env.perception_track_timeout), 1e-3)
        teams = torch.as_tensor(env.team_ids, device=dev).long()
        mates = []
        for r in self.robot_ids:
            others = [j for j in range(6) if j != r and int(teams[j]) == int(teams[r])]
            if len(others) != 2:
                raise ValueError("PerceptionInputs needs two teams of three robots")
            mates.append(others)
        self.teammates = torch.tensor(mates, device=dev)
        self.own_team = teams[self.ids]
        self.static = self._static_channels(env)
        self.piece_extent = float(getattr(env, "fuel_ball_diameter", .15))

    def _cells(self, xy: Tensor) -> Tensor:
        g = (torch.nan_to_num(xy) / self.scales * self.grid).floor().long()
        return g[..., 1].clamp(0, self.rows - 1) * self.cols + g[..., 0].clamp(0, self.cols - 1)

    def _static_channels(self, env) -> Tensor:
        dev = env.device
        ys = (torch.arange(self.rows, device=dev) + .5) * (env.field_width / self.rows)
        xs = (torch.arange(self.cols, device=dev) + .5) * (env.field_length / self.cols)
        gy, gx = torch.meshgrid(ys, xs, indexing="ij")
        centers = torch.stack((gx, gy), -1)
        half = torch.tensor((env.field_length / self.cols / 2, env.field_width / self.rows / 2), device=dev)
        out = torch.zeros((len(self.robot_ids), 12, self.rows, self.cols), device=dev)
        for ch, kinds in ((0, ("hub", "upright", "support")), (1, ("bump",))):
            boxes = [b.as_tensor() for b in env.field_boxes if b.kind in kinds]
            if boxes:
                bt = torch.tensor(boxes, device=dev)
                hit = ((centers[..., None, :] - bt[:, :2]).abs() <= bt[:, 2:4] + half).all(-1).any(-1)
                out[:, ch] = hit.float()
        hub_cells = self._cells(env.hub_centers)
        flat = out.flatten(2)
        rows = torch.arange(len(self.robot_ids), device=dev)
        flat[rows, 9, hub_cells[self.own_team]] = 1.
        flat[rows, 10, hub_cells[1 - self.own_team]] = 1.
        return out

    def _sel(self, t: Tensor) -> Tensor:
        s = t.index_select(1, self.ids)
        return s.reshape(self.env.n * len(self.robot_ids), *t.shape[2:])

    @torch.no_grad()
    def __call__(self, obs: Tensor | None = None) -> dict[str, Tensor]:
        env, ws = self.env, self.env.ws
        k = len(self.robot_ids)
        batch = env.n * k
        if obs is None:
            obs = ws["obs"]
        if obs.ndim == 3:
            scalars = self._sel(obs)
        elif obs.shape[0] == env.n * 6:
            scalars = self._sel(obs.reshape(env.n, 6, -1))
        elif obs.shape[0] == batch:
            scalars = obs
        else:
            raise ValueError("expected a full [n, 6, 137] or selected [n*k, 137] observation batch")
        scalars = torch.nan_to_num(scalars.float())
        P = ws["t_mask"].shape[-1]
        mask_f = self._sel(ws["t_mask"]).bool()
        pos = self._sel(ws["t_pos"]).transpose(1, 2)                 # [B, P, 2]
        vel = self._sel(ws["t_vel"]).transpose(1, 2)
        age = torch.nan_to_num(self._sel(ws["t_age"]), nan=self.timeout, posinf=self.timeout).clamp_min(0.)
        conf = torch.nan_to_num(self._sel(ws["t_conf"])).clamp(0., 1.)
        mask_f = mask_f & torch.isfinite(pos).all(-1)
        pos = torch.nan_to_num(pos.masked_fill(~mask_f[..., None], 0.))
        vel = torch.nan_to_num(vel.masked_fill(~mask_f[..., None], 0.))
        own = self._sel(ws["policy_pose"])[:, :2]
        own_vel = self._sel(ws["r_vel"])[:, :2]
        params = self._sel(ws["r_param"])
        own_ext = params[:, :2]
        speed = params[:, 3].clamp_min(.1)[:, None, None]
        mates_pos = ws["policy_pose"][:, self.teammates, :2].reshape(batch, 2, 2)
        mates_vel = ws["r_vel"][:, self.teammates, :2].reshape(batch, 2, 2)
        mates_ext = ws["r_param"][:, self.teammates, :2].reshape(batch, 2, 2)
        opp_mask = self._sel(ws["o_valid"]).reshape(batch).bool()
        opp_pos = self._sel(ws["o_pose"])[:, :2]
        opp_mask = opp_mask & torch.isfinite(opp_pos).all(-1)
        opp_vel = self._sel(ws["o_vel"])[:, :2]
        opp_ext = self._sel(ws["o_size"])[:, :2]
        opp_age = self._sel(ws["o_age"]).reshape(batch)
        # stereo-cluster tracks carry the spatial extent of the apparent object;
        # per-piece tracks (zero extent) fall back to one FUEL diameter
        ext_f = torch.nan_to_num(self._sel(ws["t_spatial"]).transpose(1, 2))
        ext_f = torch.where(ext_f > 0., ext_f, torch.full_like(ext_f, self.piece_extent)) * mask_f[..., None]
        positions = torch.cat((pos, own[:, None], mates_pos, opp_pos[:, None]), 1)
        velocities = torch.cat((vel, own_vel[:, None], mates_vel, opp_vel[:, None]), 1)
        extents = torch.cat((ext_f, own_ext[:, None], mates_ext, opp_ext[:, None]), 1)
        ages = torch.cat((age, age.new_zeros((batch, 3)), opp_age[:, None]), 1)
        confs = torch.cat((conf, conf.new_ones((batch, 3)), opp_mask[:, None].float()), 1)
        mask = torch.cat((mask_f, mask_f.new_ones((batch, 3)), opp_mask[:, None]), 1)
        types = positions.new_zeros((batch, P + 4, 4))
        types[:, :P, 3] = 1.
        types[:, P, 0] = 1.
        types[:, P + 1:P + 3, 1] = 1.
        types[:, P + 3, 2] = 1.
        ents = torch.cat(((positions - own[:, None]) / self.scales, velocities / speed,
                          (ages / self.timeout).clamp(0., 1.)[..., None], confs[..., None], types,
                          extents / self.scales), -1)
        ents = torch.nan_to_num(ents.masked_fill(~mask[..., None], 0.))
        field = self.static[None].expand(env.n, -1, -1, -1, -1).reshape(batch, 12, self.rows, self.cols).clone()
        flat = field.flatten(2)
        cells = self._cells(pos)
        w = mask_f.float()
        fresh = conf * torch.exp(-age / self.timeout)
        vals = torch.stack((w, vel[..., 0] / speed[:, 0], vel[..., 1] / speed[:, 0], fresh), 1) * w[:, None]
        sums = field.new_zeros((batch, 4, self.rows * self.cols))
        sums.scatter_add_(2, cells[:, None].expand(-1, 4, -1), vals)
        count = sums[:, 0]
        flat[:, 2] = count.log1p() / math.log1p(max(P, 1))
        flat[:, 3:6] = sums[:, 1:4] / count[:, None].clamp_min(1.)
        flat[:, 11] = (count > 0).float()
        rc = self._cells(positions[:, P:])
        flat[:, 6].scatter_add_(1, rc[:, :1], field.new_ones((batch, 1)))
        flat[:, 7].scatter_add_(1, rc[:, 1:3], field.new_ones((batch, 2)))
        flat[:, 8].scatter_add_(1, rc[:, 3:4], opp_mask[:, None].float())
        return {"scalars": scalars, "field": field, "entities": ents, "entity_mask": mask}
