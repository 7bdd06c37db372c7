"""Playback recording for the dashboard (frc_defense/dashboard_simulation.py).

``record_playback`` runs a batch of 3v3 worlds on the simulator (scripted
offense and defense, or a trained policy for the defense slots) and records
world 0 every ``every`` ticks: robot poses and actions, free FUEL positions,
planned routes, HUB activity and scores. Frames are plain JSON for the
Canvas viewer.
"""
from __future__ import annotations

from pathlib import Path

import torch

from .. import field as fieldmod


def field_layout_payload(layout: str = "2026_rebuilt") -> dict:
    boxes = fieldmod.qualification_field(layout)
    return {"layout": layout, "length": fieldmod.FIELD_LENGTH, "width": fieldmod.FIELD_WIDTH_SIM,
            "boxes": [b.as_dict() for b in boxes]}


@torch.no_grad()
def record_playback(*, seconds: float = 20., every: int = 5, device="cpu", seed: int = 0, checkpoint=None,
                    fuel_physics: bool = False, progress=None, cancel=None, on_metadata=None,
                    on_frame=None) -> dict:
    """Record one world; `on_metadata(dict)` is called once before the first
    frame and `on_frame(dict)` with every frame as it is produced (the live
    stream of the dashboard)."""
    from ..sim.env3v3 import TensorThreeVsThreeEnv
    modes = ("deterministic",) * 3 + (("nn",) * 3 if checkpoint else ("deterministic",) * 3)
    env = TensorThreeVsThreeEnv(num_envs=1, device=device, seed=seed, fuel_physics=fuel_physics,
                                control_modes=modes)
    policy = None
    if checkpoint:
        from ..train.evaluation import load_policy
        policy = load_policy(checkpoint, device)
    ticks = int(round(seconds / env.dt))
    frames = []
    metadata = {"field": field_layout_payload(), "teams": [0, 0, 0, 1, 1, 1], "dt": env.dt, "every": every,
                "policy": str(checkpoint) if checkpoint else "scripted", "seed": seed, "ticks": ticks}
    if on_metadata is not None:
        on_metadata(metadata)
    actions = torch.full((1, 6), 7, dtype=torch.int32, device=env.device)
    ws = env.ws
    for t in range(0, ticks, every):
        if policy is not None:
            obs = ws["obs"][:, 3:6].reshape(-1, 137)
            a, _, _ = policy.sample(obs, deterministic=True, action_mask=obs[:, -8:] > .5)
            actions[0, 3:6] = a.to(torch.int32)
        env.step_held(actions, every)
        free = ws["f_active"][0].bool() & (ws["f_owner"][0] < 0)
        fuel = ws["f_pos"][0, :2].T[free]
        frame = {"tick": t + every, "time": round((t + every) * env.dt, 3),
                 "robots": ws["r_pose"][0].tolist(), "actions": ws["g_action"][0].tolist(),
                 "fuel": [[round(x, 3), round(y, 3)] for x, y in fuel.tolist()],
                 "routes": [ws["p_path"][0, r, :int(ws["p_len"][0, r])].tolist() for r in range(6)],
                 "targets": ws["c_target"][0].tolist(),
                 "tracks": [[[round(x, 3), round(y, 3)] for x, y in
                             ws["t_pos"][0, r].T[ws["t_mask"][0, r].bool()].tolist()] for r in range(6)],
                 "possession": [int(((ws["f_owner"][0] == r) & ws["f_active"][0].bool()).sum()) for r in range(6)],
                 "hub_active": ws["g_hub"][0].tolist(), "scores": ws["g_scores"][0].tolist()}
        frames.append(frame)
        if on_frame is not None:
            on_frame(frame)
        if progress is not None:
            progress(min(1., (t + every) / ticks))
        if cancel is not None and cancel():
            break
    return {**metadata, "frames": frames}


def write_json_atomic(path: Path, payload: dict) -> None:
    import json
    tmp = path.with_suffix(path.suffix + ".tmp")
    tmp.write_text(json.dumps(payload, separators=(",", ":")))
    tmp.replace(path)
