"""FRC 2026 REBUILT field geometry in field metres.

The field frame starts at the red alliance wall (x = 0) and runs downfield;
y = 0 is the lower guardrail. Every structure is an axis-aligned rectangle
given by its centre and full extents. The dimensions come from the public game
manual drawings (inches converted to metres) and are the same numbers the
reference simulator uses (``frc_defense/field.py:75-155``); the table has to
match so both simulators collide with the same field.

Structure kinds:

* ``hub``        solid, scoring target (one per alliance)
* ``bump``       traversable ramp terrain (two per alliance, either side of a HUB)
* ``tower``      open floor area under the climbing tower (not solid)
* ``upright``    the two solid tower posts
* ``trench``     overhead arm area (open floor, not solid)
* ``support``    the solid in-field trench support strip
* ``depot``      open floor area where FUEL is staged
"""
from __future__ import annotations

from dataclasses import dataclass
import math

INCH = 0.0254
FIELD_LENGTH = 651.22 * INCH          # 16.541 m
FIELD_WIDTH_SIM = 8.07                 # width used by both environments
ALLIANCE_ZONE_DEPTH = 158.6 * INCH

# Bump ramp profile: a 0.5 in panel step plus a linear rise to the crest.
BUMP_HEIGHT = 6.513 * INCH
BUMP_PANEL_THICKNESS = 0.5 * INCH
BUMP_RAMP_RISE = BUMP_HEIGHT - BUMP_PANEL_THICKNESS
BUMP_DEPTH = 44.4 * INCH
BUMP_WIDTH = 73.0 * INCH
BUMP_RAMP_GRADE = BUMP_RAMP_RISE / (BUMP_DEPTH / 2)
BUMP_ROLLING_RESISTANCE = 0.0125
BUMP_ROBOT_CG_HEIGHT = 0.30

HUB_SIZE = 47.0 * INCH


@dataclass(frozen=True)
class FieldBox:
    name: str
    kind: str
    alliance: str  # "red", "blue" or ""
    x: float
    y: float
    length: float  # full x extent
    width: float   # full y extent

    @property
    def half(self) -> tuple[float, float]:
        return self.length / 2, self.width / 2

    def as_tensor(self) -> tuple[float, float, float, float]:
        """``(cx, cy, half_x, half_y)`` as used by every kernel."""
        return self.x, self.y, self.length / 2, self.width / 2

    @property
    def solid(self) -> bool:
        return self.kind in ("hub", "upright", "support")

    def as_dict(self) -> dict:
        return {"name": self.name, "kind": self.kind, "x": self.x, "y": self.y,
                "length": self.length, "width": self.width,
                "color": f"{self.kind}-{self.alliance}" if self.alliance else self.kind}


def _mirror_x(length: float, x: float) -> float:
    return length - x


def rebuilt_field(length: float = FIELD_LENGTH, width: float = 317.7 * INCH) -> tuple[FieldBox, ...]:
    """All REBUILT structures, red side first then mirrored blue side."""
    cy = width / 2
    hub_x = ALLIANCE_ZONE_DEPTH + HUB_SIZE / 2
    bump_dy = (HUB_SIZE + BUMP_WIDTH) / 2
    tower_l, tower_w = 45.0 * INCH, 49.25 * INCH
    post_t, post_d, post_gap = 1.5 * INCH, 3.5 * INCH, 32.25 * INCH
    trench_d, trench_w, trench_clear = 47.0 * INCH, 65.65 * INCH, 50.34 * INCH
    support_w = trench_w - trench_clear
    depot_d, depot_w, depot_dy = 27.0 * INCH, 42.0 * INCH, 94.0 * INCH
    out: list[FieldBox] = []
    for alliance in ("red", "blue"):
        mx = (lambda v: v) if alliance == "red" else (lambda v: _mirror_x(length, v))
        out.append(FieldBox(f"{alliance}_hub", "hub", alliance, mx(hub_x), cy, HUB_SIZE, HUB_SIZE))
    for alliance in ("red", "blue"):
        mx = (lambda v: v) if alliance == "red" else (lambda v: _mirror_x(length, v))
        out.append(FieldBox(f"{alliance}_bump_lower", "bump", alliance, mx(hub_x), cy - bump_dy,
                            BUMP_DEPTH, BUMP_WIDTH))
        out.append(FieldBox(f"{alliance}_bump_upper", "bump", alliance, mx(hub_x), cy + bump_dy,
                            BUMP_DEPTH, BUMP_WIDTH))
    for alliance in ("red", "blue"):
        mx = (lambda v: v) if alliance == "red" else (lambda v: _mirror_x(length, v))
        out.append(FieldBox(f"{alliance}_tower", "tower", alliance, mx(tower_l / 2), cy, tower_l, tower_w))
    for alliance in ("red", "blue"):
        mx = (lambda v: v) if alliance == "red" else (lambda v: _mirror_x(length, v))
        px = tower_l - post_d / 2
        for side, sy in (("lower", cy - post_gap / 2), ("upper", cy + post_gap / 2)):
            out.append(FieldBox(f"{alliance}_tower_upright_{side}", "upright", alliance,
                                mx(px), sy, post_d, post_t))
    for alliance in ("red", "blue"):
        mx = (lambda v: v) if alliance == "red" else (lambda v: _mirror_x(length, v))
        tx = mx(hub_x)
        out.append(FieldBox(f"{alliance}_trench_lower", "trench", alliance, tx, trench_w / 2,
                            trench_d, trench_w))
        out.append(FieldBox(f"{alliance}_trench_upper", "trench", alliance, tx, width - trench_w / 2,
                            trench_d, trench_w))
        out.append(FieldBox(f"{alliance}_trench_support_lower", "support", alliance, tx,
                            trench_w - support_w / 2, trench_d, support_w))
        out.append(FieldBox(f"{alliance}_trench_support_upper", "support", alliance, tx,
                            width - trench_w + support_w / 2, trench_d, support_w))
    out.append(FieldBox("red_depot", "depot", "red", depot_d / 2, cy - depot_dy, depot_d, depot_w))
    out.append(FieldBox("blue_depot", "depot", "blue", length - depot_d / 2, cy + depot_dy,
                        depot_d, depot_w))
    return tuple(b for b in out if 0 <= b.y <= width)


LAYOUT_SHIFTS = {
    "2026_rebuilt": None,
    "2026_rebuilt_shifted_structures_v1": (.28, 1.),
    "2026_rebuilt_shifted_structures_v2": (.46, 1.),
    "2026_rebuilt_shifted_structures_v3": (.46, -1.),
}


def qualification_field(layout_id: str = "2026_rebuilt", length: float = FIELD_LENGTH,
                        width: float = 317.7 * INCH) -> tuple[FieldBox, ...]:
    """Named layout; shifted variants move bumps and trenches toward/away from centre.

    Mirrors ``frc_defense/field.py:158-181``.
    """
    if layout_id not in LAYOUT_SHIFTS:
        raise ValueError(f"unknown qualification field layout: {layout_id}")
    boxes = rebuilt_field(length, width)
    shift = LAYOUT_SHIFTS[layout_id]
    if shift is None:
        return boxes
    amount, orientation = shift
    cy = width / 2
    out = []
    for b in boxes:
        if b.kind in ("bump", "trench", "support"):
            direction = (1. if b.y < cy else -1.) * orientation
            out.append(FieldBox(b.name, b.kind, b.alliance, b.x, b.y + direction * amount,
                                b.length, b.width))
        else:
            out.append(b)
    return tuple(out)


def static_collision_boxes(boxes) -> tuple[FieldBox, ...]:
    """Ground-blocking structures (HUBs, tower uprights, trench supports)."""
    return tuple(b for b in boxes if b.solid)


def bump_boxes(boxes) -> tuple[FieldBox, ...]:
    return tuple(b for b in boxes if b.kind == "bump")


def depot_boxes(boxes) -> tuple[FieldBox, ...]:
    return tuple(b for b in boxes if b.kind == "depot")


def box_observation_radius(box: FieldBox) -> float:
    """Signed radius feature: positive for solids, negative for traversable bumps."""
    r = math.hypot(box.length, box.width) / 2
    return -r if box.kind == "bump" else r


def midfield_respawn_points(count: int, field_length: float, field_width: float):
    """Equal-density, low-discrepancy points in the central midfield band.

    x is stratified into ``count`` slices; y follows the golden-ratio sequence.
    Same construction as ``frc_defense/field.py:24-42`` so scored FUEL returns
    to the same corridor.
    """
    count = max(0, int(count))
    if count == 0:
        return []
    cx, cy = field_length / 2, field_width / 2
    x0, x1 = cx - 1.65, cx + 1.65
    y0, y1 = cy - 2.615, cy + 2.615
    if count == 1:
        return [(cx, cy)]
    phi = (math.sqrt(5.) - 1.) / 2.
    return [(x0 + (i + .5) * (x1 - x0) / count, y0 + ((i * phi) % 1.) * (y1 - y0))
            for i in range(count)]


def grid_array_points(count: int, x_min: float, x_max: float, y_min: float, y_max: float):
    """``count`` points at cell centres of a near-square rectangular array."""
    if count <= 0:
        return []
    cols = max(1, math.ceil(math.sqrt(count * (x_max - x_min) / (y_max - y_min))))
    rows = math.ceil(count / cols)
    return [(x_min + (i % cols + .5) * (x_max - x_min) / cols,
             y_min + (i // cols + .5) * (y_max - y_min) / rows) for i in range(count)]
