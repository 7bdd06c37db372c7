// Game rules, controllers, perception and observations for one environment.
//
// Reference behaviour:
//   match clock / HUB shifts    frc_defense/_tensor_3v3_gamepieces.py:148-179,
//                               frc_defense/tensor_defense_gamepieces.py:206-227
//   strategic targets           frc_defense/_tensor_3v3_actions.py:141-898
//   command synthesis           frc_defense/tensor_3v3.py:1121-1404
//   contention avoidance        frc_defense/_tensor_3v3_actions.py:900-1020
//   pickup / ferry / scoring    frc_defense/gamepiece_actions.py:128-511
//   perception and tracks       frc_defense/_tensor_3v3_observation.py:117-707
//   137-feature observation     frc_defense/_tensor_3v3_observation.py:775-896
//
// Everything here runs inside the per-environment CTA (GPU) or the per-env
// host loop. Robot-level work is spread across threads with PAR_FOR over the
// robot count; FUEL and track work with PAR_FOR over pieces.
#pragma once

#include "physics.h"

namespace ad {

enum Mode : int { MODE_NONE = 0, MODE_NN = 1, MODE_DET = 2, MODE_DIRECT = 3 };
enum OpponentKind : int {
  OPP_OFFENSE = 0, OPP_MIRROR, OPP_CUTOFF, OPP_VELOCITY_INTERCEPT, OPP_RANDOM,
  // scripted defenders of the two-robot counter-defense task (slot 1)
  OPP_DEF_INTERCEPT, OPP_DEF_LANE_BLOCK, OPP_DEF_FUEL_DENIAL, OPP_DEF_SHADOW, OPP_DEF_HUB_GUARD
};

// Accessor helpers for global state (env e, robot r, piece i).
struct G {
  World& w;
  const SimParams& sp;
  int e;
  AD_HD size_t er(int r) const { return (size_t)e * sp.R + r; }
  AD_HD size_t erp(int r, int i) const { return ((size_t)e * sp.R + r) * sp.P + i; }
  AD_HD float tx(int r, int i) const { return w.t_pos[(((size_t)e * sp.R + r) * 2 + 0) * sp.P + i]; }
  AD_HD float ty(int r, int i) const { return w.t_pos[(((size_t)e * sp.R + r) * 2 + 1) * sp.P + i]; }
  AD_HD float& txr(int r, int i) { return w.t_pos[(((size_t)e * sp.R + r) * 2 + 0) * sp.P + i]; }
  AD_HD float& tyr(int r, int i) { return w.t_pos[(((size_t)e * sp.R + r) * 2 + 1) * sp.P + i]; }
  AD_HD float& tvx(int r, int i) { return w.t_vel[(((size_t)e * sp.R + r) * 2 + 0) * sp.P + i]; }
  AD_HD float& tvy(int r, int i) { return w.t_vel[(((size_t)e * sp.R + r) * 2 + 1) * sp.P + i]; }
  AD_HD float param(int r, int k) const { return w.r_param[er(r) * kNumRobotParams + k]; }
  AD_HD float* ppose(int r) { return w.policy_pose + er(r) * 3; }
  AD_HD float* rvel(int r) { return w.r_vel + er(r) * 3; }
  AD_HD uint8_t& latch(int r, int k) { return w.g_rlatch[er(r) * kLatches + k]; }
  AD_HD float& rtime(int r, int k) { return w.g_rtime[er(r) * 3 + k]; }
  AD_HD int32_t& rcount(int r, int k) { return w.g_rcount[er(r) * 6 + k]; }
  AD_HD float elapsed() const { return w.g_time[(size_t)e * 2]; }
  AD_HD bool hub_active(int team) const { return w.g_hub[(size_t)e * 2 + team] != 0; }
};

AD_HD float robot_radius_of(float L, float W) { return .5f * sqrtf(L * L + W * W); }

AD_HD bool in_alliance_zone(const SimParams& sp, int team, float x) {
  return team == 0 ? x <= sp.alliance_depth : x >= sp.field_length - sp.alliance_depth;
}

// Robot footprint circle clear of every bump rectangle.
AD_HD bool clear_of_bumps(const SimParams& sp, float x, float y, float radius) {
  for (int b = 0; b < sp.num_bumps; ++b) {
    const Box& bx = sp.bumps[b];
    if (fabsf(x - bx.cx) <= bx.hx + radius && fabsf(y - bx.cy) <= bx.hy + radius) return false;
  }
  return true;
}

// ---------------------------------------------------------------------------
// Match clock and HUB schedule
// ---------------------------------------------------------------------------
AD_HD void update_match(World& w, const SimParams& sp, int e) {
  float* t = w.g_time + (size_t)e * 2;
  t[0] = fminf(t[0] + sp.dt, 160.f);
  t[1] = fmaxf(160.f - t[0], 0.f);
  uint8_t* hub = w.g_hub + (size_t)e * 2;
  const float el = t[0];
  if (sp.two_robot_schedule) {
    // 20 s autonomous with both HUBs active, then 30 s alternation starting
    // with a per-match random first inactive HUB.
    if (el < 20.f) {
      hub[0] = hub[1] = 1;
    } else {
      int cycle = (int)floorf((el - 20.f) / 30.f);
      int first = w.g_first_inactive[e];
      int inactive = (cycle % 2 == 0) ? first : 1 - first;
      hub[inactive] = 0;
      hub[1 - inactive] = 1;
    }
    return;
  }
  const int32_t* sc = w.g_scores + (size_t)e * 4;
  int first = sc[0] > sc[1] ? 0 : (sc[1] > sc[0] ? 1 : 0);
  int cycle = (int)floorf(fmaxf(el - 30.f, 0.f) / 25.f);
  int inactive = (cycle % 2 == 0) ? first : 1 - first;
  bool shifts = el >= 30.f && el < 130.f;
  hub[0] = hub[1] = 1;
  if (shifts) hub[inactive] = 0;
}

// ---------------------------------------------------------------------------
// Candidate ranking: top-4 lowest-cost entries (ties to the lower index).
// ---------------------------------------------------------------------------
struct Top4 {
  float c[4];
  int i[4];
  AD_HD void init() {
    for (int k = 0; k < 4; ++k) {
      c[k] = kInf;
      i[k] = 0;
    }
  }
  AD_HD void push(float cost, int idx) {
    if (!(cost < c[3] || (cost == c[3] && idx < i[3] && cost < kInf))) return;
    int k = 3;
    while (k > 0 && (cost < c[k - 1] || (cost == c[k - 1] && idx < i[k - 1]))) {
      c[k] = c[k - 1];
      i[k] = i[k - 1];
      --k;
    }
    c[k] = cost;
    i[k] = idx;
  }
};

// Segment vs inflated AABB detour estimate (frc_defense/_tensor_3v3_actions.py:22-53).
AD_HD float obstacle_detour(const SimParams& sp, float sx, float sy, float tx, float ty, float radius) {
  float total = 0.f;
  for (int set = 0; set < 2; ++set) {
    int count = set == 0 ? sp.num_boxes : sp.num_bumps;
    for (int b = 0; b < count; ++b) {
      const Box& bx = set == 0 ? sp.boxes[b] : sp.bumps[b];
      float hx = bx.hx + radius, hy = bx.hy + radius;
      float lo[2] = {bx.cx - hx, bx.cy - hy}, hi[2] = {bx.cx + hx, bx.cy + hy};
      float p0[2] = {sx, sy}, d[2] = {tx - sx, ty - sy};
      float enter = -kInf, leave = kInf;
      bool ok = true;
      for (int a = 0; a < 2; ++a) {
        if (fabsf(d[a]) < 1e-6f) {
          if (p0[a] < lo[a] || p0[a] > hi[a]) ok = false;
        } else {
          float t0 = (lo[a] - p0[a]) / d[a], t1 = (hi[a] - p0[a]) / d[a];
          enter = fmaxf(enter, fminf(t0, t1));
          leave = fminf(leave, fmaxf(t0, t1));
        }
      }
      enter = fmaxf(enter, 0.f);
      leave = fminf(leave, 1.f);
      if (ok && enter <= leave) total += 2.f * fminf(hx, hy);
    }
  }
  return fminf(total, 1.5f);
}

// Kinematic travel time from an initial speed under an acceleration cap.
AD_HD float travel_time(float distance, float v0, float vmax, float accel) {
  float d_to_speed = fmaxf(vmax * vmax - v0 * v0, 0.f) / (2.f * accel);
  float t_to_speed = fmaxf(vmax - v0, 0.f) / accel;
  float t_acc = (sqrtf(v0 * v0 + 2.f * accel * distance) - v0) / accel;
  return distance <= d_to_speed ? t_acc : t_to_speed + (distance - d_to_speed) / vmax;
}

// Ferry lane target inferred from a robot's own motion (no teammate intent).
AD_HD void ferry_target(G& g, int r, float& fx, float& fy) {
  const SimParams& sp = g.sp;
  int team = sp.team[r];
  float* p = g.ppose(r);
  fx = sp.field_length * .5f + (team == 0 ? -.45f : .45f);
  if (sp.teammate_coordination) {
    const float lanes[6] = {1.35f, 4.035f, 6.72f, 6.72f, 4.035f, 1.35f};
    fy = lanes[r % 6];
    return;
  }
  float mid = fabsf(fx - p[0]);
  float speed = fmaxf(g.param(r, RP_SPEED), .1f);
  float py = p[1] + g.rvel(r)[1] / speed * mid;
  float rad = robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH));
  fy = clampf(py, rad, sp.field_width - rad);
}

// Friendly-zone aim point that avoids the HUB backer net
// (frc_defense/fuel_physics_runtime.py:285-298).
AD_HD void ferry_aim_point(const SimParams& sp, int team, float ox, float oy, float& ax, float& ay) {
  ax = team == 0 ? sp.alliance_depth * .5f : sp.field_length - sp.alliance_depth * .5f;
  float side = fminf(3.f, sp.field_width * .5f - sp.fr - .1f);
  ay = sp.hub_y[team] + (oy <= sp.hub_y[team] ? -side : side);
  ay = clampf(ay, sp.fr, sp.field_width - sp.fr);
}

// Intake deployment rectangle (12 in ahead of the bumper) clear of the field.
AD_HD bool intake_deploy_clear(const SimParams& sp, float x, float y, float th, float L, float W) {
  const float il = .3048f;
  float c = cosf(th), s = sinf(th);
  float cx = x + (L * .5f + il * .5f) * c, cy = y + (L * .5f + il * .5f) * s;
  float ex = .5f * (il * fabsf(c) + W * fabsf(s)), ey = .5f * (il * fabsf(s) + W * fabsf(c));
  if (cx - ex < 0.f || cx + ex > sp.field_length || cy - ey < 0.f || cy + ey > sp.field_width) return false;
  for (int b = 0; b < sp.num_boxes; ++b) {
    const Box& bx = sp.boxes[b];
    if (fabsf(cx - bx.cx) < ex + bx.hx && fabsf(cy - bx.cy) < ey + bx.hy) return false;
  }
  return true;
}

// Nearest scoring pose inside the alliance zone that clears bumps and solids
// (frc_defense/_tensor_3v3_actions.py:564-631, side-candidate + score grid form).
AD_HD void safe_score_target(G& g, int r, float& outx, float& outy) {
  const SimParams& sp = g.sp;
  int team = sp.team[r];
  float* p = g.ppose(r);
  float rad = robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH));
  float xmin = team == 0 ? rad : sp.field_length - sp.alliance_depth + rad;
  float xmax = team == 0 ? fmaxf(sp.alliance_depth - rad, 0.f) : sp.field_length - rad;
  float bx0 = fmaxf(xmin, fminf(p[0], xmax));
  float by0 = fmaxf(rad, fminf(p[1], sp.field_width - rad));
  auto is_clear = [&](float x, float y) -> bool {
    for (int set = 0; set < 3; ++set) {
      int count = set == 0 ? sp.num_boxes : sp.num_bumps;
      for (int b = 0; b < count; ++b) {
        const Box& bx = set == 0 ? sp.boxes[b] : sp.bumps[b];
        if (fabsf(x - bx.cx) <= bx.hx + rad + .15f && fabsf(y - bx.cy) <= bx.hy + rad + .15f) return false;
      }
    }
    return true;
  };
  float best = kInf, bx = bx0, by = by0;
  bool any = false;
  auto consider = [&](float x, float y) {
    x = fmaxf(xmin, fminf(x, xmax));
    y = fminf(fmaxf(y, rad), sp.field_width - rad);
    if (!is_clear(x, y)) return;
    float d = sqrtf(sqr(x - p[0]) + sqr(y - p[1]));
    if (d < best) {
      best = d;
      bx = x;
      by = y;
      any = true;
    }
  };
  consider(bx0, by0);
  const float clearance = .40f;
  for (int set = 0; set < 2; ++set) {
    int count = set == 0 ? sp.num_boxes : sp.num_bumps;
    for (int b = 0; b < count; ++b) {
      const Box& q = set == 0 ? sp.boxes[b] : sp.bumps[b];
      consider(q.cx - q.hx - rad - clearance, by0);
      consider(q.cx + q.hx + rad + clearance, by0);
      consider(bx0, q.cy - q.hy - rad - clearance);
      consider(bx0, q.cy + q.hy + rad + clearance);
    }
  }
  const float xf[5] = {.12f, .30f, .48f, .66f, .84f};
  const float yf[6] = {.12f, .28f, .44f, .60f, .76f, .90f};
  for (int a = 0; a < 5; ++a)
    for (int b = 0; b < 6; ++b)
      consider(xmin + (xmax - xmin) * xf[a], rad + (sp.field_width - 2.f * rad) * yf[b]);
  outx = any ? bx : bx0;
  outy = any ? by : by0;
}

// Attacker objective of the two-robot roster: the HUB approach ring when
// carrying FUEL to an active HUB, else the nearest perceived FUEL track
// (frc_defense/tensor_sim.py:366-383).
AD_HD void attacker_objective(G& g, int r, const int32_t* possession, float& gx, float& gy) {
  const SimParams& sp = g.sp;
  World& w = g.w;
  const int team = sp.team[r];
  const float* p = g.ppose(r);
  float dx = p[0] - sp.hub_x[team], dy = p[1] - sp.hub_y[team];
  float dn = fmaxf(sqrtf(dx * dx + dy * dy), 1e-6f);
  float rad = .595f + robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH)) + .02f;
  float ax = sp.hub_x[team] + dx / dn * rad, ay = sp.hub_y[team] + dy / dn * rad;
  if (possession[r] > 0 && g.hub_active(team)) {
    gx = ax;
    gy = ay;
    return;
  }
  float best = kInf;
  gx = ax;
  gy = ay;
  for (int i = 0; i < sp.P; ++i) {
    if (!w.t_mask[g.erp(r, i)]) continue;
    float d = sqr(g.tx(r, i) - p[0]) + sqr(g.ty(r, i) - p[1]);
    if (d < best) {
      best = d;
      gx = g.tx(r, i);
      gy = g.ty(r, i);
    }
  }
}

// Waypoint of a scripted defender (robot r) against `attacker`, built from
// r's own pose estimate and its track of the attacker only
// (frc_defense/tensor_defense_opponent.py:176-214): intercept ahead of the
// attacker's motion (look-ahead = time to reach it, at most 1.25 s, plus
// 0.55 m along its heading), block the attacker's lane to its HUB (40 % of
// the way, at most 1 m), deny the nearest perceived FUEL (else block),
// shadow 0.35 s ahead of it, or guard the HUB front along that lane. Without
// a track (or, for FUEL denial, a FUEL candidate) the defender holds.
AD_HD void defense_target(G& g, int r, int attacker, int kind, bool fuel_valid, int fuel_index, float& tx,
                          float& ty) {
  const SimParams& sp = g.sp;
  World& w = g.w;
  const size_t er = g.er(r);
  const float* dp = g.ppose(r);
  const float* ap = w.o_pose + er * 3;
  const float* av = w.o_vel + er * 3;
  bool tracked = w.o_valid[er] != 0;
  const float vx = av[0], vy = av[1];
  const float spd = sqrtf(vx * vx + vy * vy);
  const float tox = dp[0] - ap[0], toy = dp[1] - ap[1];
  const float dist = sqrtf(tox * tox + toy * toy), tn = fmaxf(dist, 1e-6f);
  const float hx = spd > .15f ? vx / fmaxf(spd, .15f) : tox / tn;
  const float hy = spd > .15f ? vy / fmaxf(spd, .15f) : toy / tn;
  const float eta = clampf(dist / fmaxf(g.param(r, RP_SPEED), .1f), 0.f, 1.25f);
  const int team = sp.team[attacker];
  const float hubx = sp.hub_x[team], huby = sp.hub_y[team];
  float lx = hubx - ap[0], ly = huby - ap[1];
  const float hd = fmaxf(sqrtf(lx * lx + ly * ly), 1e-6f);
  lx /= hd;
  ly /= hd;
  const float reach = fminf(hd * .4f, 1.f);
  const float bx = ap[0] + lx * reach, by = ap[1] + ly * reach;
  const float L = g.param(r, RP_LENGTH), W = g.param(r, RP_WIDTH);
  const float guard = .595f + .5f * sqrtf(L * L + W * W) + .15f;
  switch (kind) {
    case OPP_DEF_FUEL_DENIAL:
      tx = fuel_valid ? g.tx(r, fuel_index) : bx;
      ty = fuel_valid ? g.ty(r, fuel_index) : by;
      tracked = tracked || fuel_valid;
      break;
    case OPP_DEF_LANE_BLOCK:
      tx = bx;
      ty = by;
      break;
    case OPP_DEF_SHADOW:
      tx = ap[0] + vx * .35f;
      ty = ap[1] + vy * .35f;
      break;
    case OPP_DEF_HUB_GUARD:
      tx = hubx - lx * guard;
      ty = huby - ly * guard;
      break;
    default:  // intercept
      tx = ap[0] + vx * eta + hx * .55f;
      ty = ap[1] + vy * eta + hy * .55f;
  }
  if (!tracked) {
    tx = dp[0];
    ty = dp[1];
  }
  tx = clampf(tx, 0.f, sp.field_length);
  ty = clampf(ty, 0.f, sp.field_width);
}

// ---------------------------------------------------------------------------
// Control: strategic action -> navigation target (one thread per robot).
// `actions` holds the policy's categorical action for nn-mode robots.
// ---------------------------------------------------------------------------
// Track-scan results consumed by control_robot, produced by the two scans
// below (one warp per robot on the GPU, lane-strided over the track slots;
// one lane on the host).
struct ControlScan {
  float top_c[kMaxRobots][4];
  int top_i[kMaxRobots][4];
  uint8_t intake[kMaxRobots], alliance[kMaxRobots], nearby[kMaxRobots];
  float yield[kMaxRobots][4];
  // cluster collection of the scripted offense (set by control_robot)
  uint8_t edge[kMaxRobots];      // collecting: trace the FUEL cloud's contour this tick
  uint8_t approach[kMaxRobots];  // heading for the intake-strip approach pose
  int cluster_count[kMaxRobots];
  float cluster_center[kMaxRobots][2];
  float boundary[kMaxRobots][2];  // intake right corner along the collect heading
  float inward[kMaxRobots][2];    // density-weighted pull of the tracks (control_scan_cloud)
};

// Intake reference point (front-right intake corner plus a short momentum
// lead) and the mid-field detour limit shared by the scans and the controller.
AD_HD void intake_reference(G& g, int r, int poss, float& rrx, float& rry, float& detour_limit) {
  const SimParams& sp = g.sp;
  const float* p = g.ppose(r);
  const float* v = g.rvel(r);
  const float L = g.param(r, RP_LENGTH), W = g.param(r, RP_WIDTH);
  const float c = cosf(p[2]), s = sinf(p[2]);
  const float irx = p[0] + c * (L * .5f + .15f) + s * (W * .5f);
  const float iry = p[1] + s * (L * .5f + .15f) - c * (W * .5f);
  const float horizon = fminf(sp.replan_interval * sp.dt * .5f, .2f);
  const float mx = v[0] * horizon, my = v[1] * horizon;
  const float md = sqrtf(mx * mx + my * my);
  const float mscale = fminf(.5f / fmaxf(md, 1e-6f), 1.f);
  rrx = irx + mx * mscale;
  rry = iry + my * mscale;
  const int cap = sp.capacity[r];
  const float remaining = 1.f - (float)poss / (float)(cap > 0 ? cap : 1);
  detour_limit = 2.f + 1.5f * clampf(remaining, 0.f, 1.f);
}

// Rank the live, legal FUEL tracks of robot r: top-4 by (cost, index) plus the
// intake / alliance / nearby-midfield flags. Lanes scan strided slots and the
// top-4 lists merge through a butterfly; (cost, index) is a total order, so the
// result equals the serial scan's.
AD_HD void control_scan_tracks(G& g, int r, const int32_t* possession, ControlScan& cs, int lane, int nlanes) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const int team = sp.team[r];
  const bool det_offense = sp.mode[r] == MODE_DET && sp.role[r] == 0;
  const bool hub_on = g.hub_active(team);
  const float* p = g.ppose(r);
  float rrx, rry, detour_limit;
  intake_reference(g, r, possession[r], rrx, rry, detour_limit);
  Top4 top;
  top.init();
  bool intake = false, alliance = false, nearby = false;
  for (int i = lane; i < sp.P; i += nlanes) {
    size_t k = g.erp(r, i);
    if (!w.t_mask[k] || !(w.t_age[k] <= sp.track_timeout)) continue;
    const float x = g.tx(r, i), y = g.ty(r, i);
    const bool in_all = in_alliance_zone(sp, team, x);
    if (det_offense && !hub_on && in_all) continue;
    intake = true;
    if (in_all) alliance = true;
    if (!in_all && sqrtf(sqr(x - p[0]) + sqr(y - p[1])) <= detour_limit) nearby = true;
    const float cost = sqrtf(sqr(x - rrx) + sqr(y - rry)) + fminf(fmaxf(w.t_age[k], 0.f), 2.f) * .4f;
    top.push(cost, i);
  }
#if defined(__CUDA_ARCH__)
  if (nlanes > 1) {
    for (int o = 16; o > 0; o >>= 1) {
      float oc[4];
      int oi[4];
      for (int k = 0; k < 4; ++k) {
        oc[k] = __shfl_xor_sync(0xffffffffu, top.c[k], o);
        oi[k] = __shfl_xor_sync(0xffffffffu, top.i[k], o);
      }
      for (int k = 0; k < 4; ++k)
        if (oc[k] < kInf) top.push(oc[k], oi[k]);
    }
    intake = __any_sync(0xffffffffu, intake);
    alliance = __any_sync(0xffffffffu, alliance);
    nearby = __any_sync(0xffffffffu, nearby);
  }
#endif
  if (lane == 0) {
    for (int k = 0; k < 4; ++k) {
      cs.top_c[r][k] = top.c[k];
      cs.top_i[r][k] = top.i[k];
    }
    cs.intake[r] = intake;
    cs.alliance[r] = alliance;
    cs.nearby[r] = nearby;
  }
}

// Expected FUEL yield around each candidate (confidence x freshness of the
// live tracks within two robot radii), needed only by the scripted offense
// while its HUB is active.
AD_HD void control_scan_yields(G& g, int r, const ControlScan& cs_in, ControlScan& cs, int lane, int nlanes) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const int team = sp.team[r];
  const bool det_offense = sp.mode[r] == MODE_DET && sp.role[r] == 0;
  float y[4] = {0.f, 0.f, 0.f, 0.f};
  const bool needed = det_offense && g.hub_active(team) && cs_in.intake[r];
  if (needed) {
    const float rad = robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH));
    float cx[4], cy[4];
    bool cv[4];
    for (int k = 0; k < 4; ++k) {
      cv[k] = cs_in.top_c[r][k] < kInf;
      cx[k] = cv[k] ? g.tx(r, cs_in.top_i[r][k]) : 0.f;
      cy[k] = cv[k] ? g.ty(r, cs_in.top_i[r][k]) : 0.f;
    }
    for (int j = lane; j < sp.P; j += nlanes) {
      size_t kj = g.erp(r, j);
      if (!w.t_mask[kj] || !(w.t_age[kj] <= sp.track_timeout)) continue;
      const float ax = g.tx(r, j), ay = g.ty(r, j);
      const float contrib = clampf(w.t_conf[kj], 0.f, 1.f) *
                            expf(-fmaxf(w.t_age[kj], 0.f) / fmaxf(sp.track_timeout, 1e-6f));
      for (int k = 0; k < 4; ++k)
        if (cv[k] && sqrtf(sqr(ax - cx[k]) + sqr(ay - cy[k])) <= 2.f * rad) y[k] += contrib;
    }
#if defined(__CUDA_ARCH__)
    if (nlanes > 1)
      for (int k = 0; k < 4; ++k)
        for (int o = 16; o > 0; o >>= 1) y[k] += __shfl_xor_sync(0xffffffffu, y[k], o);
#endif
  }
  if (lane == 0)
    for (int k = 0; k < 4; ++k) cs.yield[r][k] = y[k];
}


// ---------------------------------------------------------------------------
// Scripted offense collection (frc_defense/_tensor_3v3_actions.py:677-890,
// frc_defense/_tensor_3v3_navigation.py:84-127).
// ---------------------------------------------------------------------------
AD_HD bool env_has_det_offense(const SimParams& sp) {
  for (int r = 0; r < sp.R; ++r)
    if (sp.mode[r] == MODE_DET && sp.role[r] == 0) return true;
  return false;
}

// Each robot's closed raster route: kRasterPoints samples; the cursor is the
// sample the robot was last nearest to.
AD_HD const float* raster_point(const World& w, int r, int k) {
  return w.raster_pts + ((size_t)r * kRasterPoints + k) * 2;
}

AD_HD int raster_nearest(const World& w, int r, int from, int count, float x, float y) {
  int best_k = from;
  float best = kInf;
  for (int o = 0; o < count; ++o) {
    const int k = (from + o) % kRasterPoints;
    const float* q = raster_point(w, r, k);
    const float d2 = sqr(q[0] - x) + sqr(q[1] - y);
    if (d2 < best) {
      best = d2;
      best_k = k;
    }
  }
  return best_k;
}

// Before target selection: a robot that was not sweeping re-anchors to the
// nearest route sample, a sweeping one searches the next 33 samples.
AD_HD void raster_prepare(G& g, int r) {
  int32_t& c = g.w.c_raster[g.er(r)];
  const float* p = g.ppose(r);
  c = 1 + (c <= 0 ? raster_nearest(g.w, r, 0, kRasterPoints, p[0], p[1])
                  : raster_nearest(g.w, r, (c - 1) % kRasterPoints, 33, p[0], p[1]));
}

// After the tick: a sweeping robot's cursor follows it; any other robot
// re-anchors at its next decision.
AD_HD void raster_finish(G& g, int r) {
  int32_t& c = g.w.c_raster[g.er(r)];
  if (g.latch(r, RL_RASTER_SWEEP) && c > 0) {
    const float* p = g.ppose(r);
    c = 1 + raster_nearest(g.w, r, (c - 1) % kRasterPoints, 33, p[0], p[1]);
  } else {
    c = 0;
  }
}

// Route sample `raster_lookahead` ahead of the cursor and the route tangent there.
AD_HD void raster_target(G& g, int r, float& tx, float& ty, float& dirx, float& diry) {
  const int c = g.w.c_raster[g.er(r)] > 0 ? g.w.c_raster[g.er(r)] - 1 : 0;
  const int k = (c + g.sp.raster_lookahead) % kRasterPoints;
  const float* a = raster_point(g.w, r, k);
  const float* b = raster_point(g.w, r, (k + 1) % kRasterPoints);
  tx = a[0];
  ty = a[1];
  const float dx = b[0] - a[0], dy = b[1] - a[1];
  const float n = fmaxf(sqrtf(dx * dx + dy * dy), 1e-6f);
  dirx = dx / n;
  diry = dy / n;
}

// Chassis pose that puts the selected ball in the front intake strip: short
// of the ball on the approach line, or, for a ball in the robot's own depot,
// the nearest reachable pose beside the depot's field side or open ends.
AD_HD void approach_pose(G& g, int r, float fx, float fy, float fdx, float fdy, float& tx, float& ty) {
  const SimParams& sp = g.sp;
  const float L = g.param(r, RP_LENGTH), W = g.param(r, RP_WIDTH);
  const float rad = robot_radius_of(L, W);
  const float d = fmaxf(sqrtf(fdx * fdx + fdy * fdy), 1e-6f);
  tx = clampf(fx - fdx / d * .45f, rad, sp.field_length - rad);
  ty = clampf(fy - fdy / d * .45f, rad, sp.field_width - rad);
  const int team = sp.team[r];
  if (team >= sp.num_depots) return;
  const Box& dp = sp.depots[team];
  if (!(fabsf(fx - dp.cx) <= dp.hx && fabsf(fy - dp.cy) <= dp.hy)) return;
  const float hl = L * .5f, hw = W * .5f;
  const float xmin = hl, xmax = sp.field_length - hl, ymin = hw, ymax = sp.field_width - hw;
  const float side_x = team == 0 ? dp.cx + dp.hx + hl - .20f : dp.cx - dp.hx - hl + .20f;
  const float cand[3][2] = {{side_x, clampf(fy, ymin, ymax)},
                            {clampf(fx, xmin, xmax), dp.cy - dp.hy - .015f - hw},
                            {clampf(fx, xmin, xmax), dp.cy + dp.hy + .015f + hw}};
  const float* p = g.ppose(r);
  float best = kInf;
  int best_k = -1;
  for (int k = 0; k < 3; ++k) {
    const float ox = fabsf(fx - cand[k][0]), oy = fabsf(fy - cand[k][1]);
    const float along = k == 0 ? ox : oy, across = k == 0 ? oy : ox;
    const bool reachable = along <= hl + .35f + .083f && across <= hw + .075f + .083f && cand[k][0] >= xmin &&
                           cand[k][0] <= xmax && cand[k][1] >= ymin && cand[k][1] <= ymax;
    const float dist = sqrtf(sqr(cand[k][0] - p[0]) + sqr(cand[k][1] - p[1]));
    if (reachable && dist < best) {
      best = dist;
      best_k = k;
    }
  }
  if (best_k >= 0) {
    tx = cand[best_k][0];
    ty = cand[best_k][1];
  }
}

// Cluster collection state machine of a scripted robot (targets for target-
// based collection, the intake-strip approach, search targets). Robots that
// collect inside a cluster are marked for contour tracing (cs.edge).
AD_HD void collection_targets(G& g, int r, int action, int poss, bool no_track_search, bool alliance_fuel,
                              const bool* cand_valid, const int* cand, float irx, float iry, float fx, float fy,
                              float& fdx, float& fdy, float& tx, float& ty, ControlScan& cs) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const size_t er = g.er(r);
  const float* p = g.ppose(r);
  const int team = sp.team[r];
  const bool det_offense = sp.mode[r] == MODE_DET && sp.role[r] == 0;
  const bool tbc = det_offense && (action < 4 || (action == 6 && poss == 0));
  // the pickup candidates near the intake form a cluster
  int count = 0;
  float nearest = kInf, ccx = 0.f, ccy = 0.f;
  for (int k = 0; k < 4; ++k) {
    if (!cand_valid[k]) continue;
    const float x = g.tx(r, cand[k]), y = g.ty(r, cand[k]);
    const float ld = sqrtf(sqr(x - irx) + sqr(y - iry));
    nearest = fminf(nearest, ld);
    if (ld < 1.7f) {
      ++count;
      ccx += x;
      ccy += y;
    }
  }
  ccx /= (float)(count > 1 ? count : 1);
  ccy /= (float)(count > 1 ? count : 1);
  bool depot_target = false;
  for (int k = 0; k < sp.num_depots; ++k)
    depot_target = depot_target || (fabsf(fx - sp.depots[k].cx) <= sp.depots[k].hx &&
                                    fabsf(fy - sp.depots[k].cy) <= sp.depots[k].hy);
  const float herr = fabsf(angle_diff(atan2f(fdy, fdx), p[2]));
  const bool depot_ready = sqrtf(fdx * fdx + fdy * fdy) <= 1.15f && herr <= .35f;
  const bool at_cluster = count >= 2 && nearest <= 1.25f && (!depot_target || depot_ready);
  const bool current_cluster = count >= 2 && nearest <= 2.4f;
  uint8_t& collecting_latch = g.latch(r, RL_TARGET_COLLECTING);
  int32_t& empty = w.c_empty_ticks[er];
  const bool was = collecting_latch != 0;
  const int empty_next = (was && !current_cluster) ? empty + 1 : 0;
  int grace = (int)ceilf(.4f / sp.dt);
  grace = grace < 1 ? 1 : grace;
  bool next = was ? empty_next < grace : at_cluster;
  next = next && tbc;
  if (next && !was) {
    // enter on the line to the selected ball
    const float td = sqrtf(fdx * fdx + fdy * fdy);
    w.c_collect_heading[er] = td > .1f ? atan2f(fdy, fdx) : p[2];
  }
  collecting_latch = next ? 1 : 0;
  empty = empty_next;
  // search: the raster route while no track is known, else the ferry lane
  const bool positioned = in_alliance_zone(sp, team, p[0]) && g.hub_active(team);
  const bool no_alliance_fuel_search = positioned && !alliance_fuel && poss > 0;
  if (tbc && !next && action == 6 && !no_alliance_fuel_search) {
    if (no_track_search) {
      float dx, dy;
      raster_target(g, r, tx, ty, dx, dy);
    } else {
      ferry_target(g, r, tx, ty);
    }
  }
  if (no_alliance_fuel_search) ferry_target(g, r, tx, ty);
  // contour tracing inputs
  if (next) {
    const float course = w.c_collect_heading[er];
    const float L = g.param(r, RP_LENGTH), W = g.param(r, RP_WIDTH);
    const float fwx = cosf(course), fwy = sinf(course);
    cs.edge[r] = 1;
    cs.boundary[r][0] = p[0] + fwx * (L * .5f + .15f) + fwy * (W * .5f);
    cs.boundary[r][1] = p[1] + fwy * (L * .5f + .15f) - fwx * (W * .5f);
    cs.cluster_count[r] = count;
    cs.cluster_center[r][0] = ccx;
    cs.cluster_center[r][1] = ccy;
  }
  // approach pose for a ball outside a cluster (or a depot ball not lined up)
  if (tbc && action < 4 && (!next || (depot_target && !depot_ready))) {
    approach_pose(g, r, fx, fy, fdx, fdy, tx, ty);
    cs.approach[r] = 1;
  }
}

// Density-weighted pull of the live eligible tracks on the intake's boundary
// corner (Gaussian kernel of max(1.5 W, 0.7 m), fading with track age), one
// warp per robot.
AD_HD void control_scan_cloud(G& g, int r, ControlScan& cs, int lane, int nlanes) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const int team = sp.team[r];
  const bool hub_on = g.hub_active(team);
  const float W = g.param(r, RP_WIDTH);
  const float sigma = fmaxf(W * 1.5f, .7f);
  const float bx = cs.boundary[r][0], by = cs.boundary[r][1];
  float sx = 0.f, sy = 0.f;
  for (int j = lane; j < sp.P; j += nlanes) {
    const size_t k = g.erp(r, j);
    if (!w.t_mask[k] || !(w.t_age[k] <= sp.track_timeout)) continue;
    const float x = g.tx(r, j), y = g.ty(r, j);
    if (!hub_on && in_alliance_zone(sp, team, x)) continue;  // scripted offense: inactive-HUB rule
    const float dx = x - bx, dy = y - by;
    const float dist = sqrtf(dx * dx + dy * dy);
    const float wt = expf(-.5f * sqr(dist / sigma)) * expf(-fmaxf(w.t_age[k], 0.f) * .2f);
    sx += dx * wt;
    sy += dy * wt;
  }
#if defined(__CUDA_ARCH__)
  if (nlanes > 1)
    for (int o = 16; o > 0; o >>= 1) {
      sx += __shfl_xor_sync(0xffffffffu, sx, o);
      sy += __shfl_xor_sync(0xffffffffu, sy, o);
    }
#endif
  if (lane == 0) {
    cs.inward[r][0] = sx;
    cs.inward[r][1] = sy;
  }
}

// Contour tracing: keep the cluster on the intake's right side, turning the
// collect heading toward the local edge tangent at most half the chassis
// turn rate; the target is 3 m along the new heading while that stays inside
// the field.
AD_HD void control_edge_finish(G& g, int r, const ControlScan& cs) {
  if (!cs.edge[r]) return;
  World& w = g.w;
  const SimParams& sp = g.sp;
  const size_t er = g.er(r);
  const float* p = g.ppose(r);
  const float course = w.c_collect_heading[er];
  const float fwx = cosf(course), fwy = sinf(course);
  const float ix = cs.inward[r][0], iy = cs.inward[r][1];
  const float in_n = sqrtf(ix * ix + iy * iy);
  const bool grad_valid = in_n > .15f;
  const float cx = cs.cluster_center[r][0] - cs.boundary[r][0], cy = cs.cluster_center[r][1] - cs.boundary[r][1];
  const float c_n = sqrtf(cx * cx + cy * cy);
  const bool center_valid = cs.cluster_count[r] >= 2 && c_n > .15f;
  if (!(grad_valid || center_valid)) return;
  const float nx = grad_valid ? ix / fmaxf(in_n, 1e-6f) : cx / fmaxf(c_n, 1e-6f);
  const float ny = grad_valid ? iy / fmaxf(in_n, 1e-6f) : cy / fmaxf(c_n, 1e-6f);
  float tnx = -ny, tny = nx;
  if (tnx * fwx + tny * fwy < 0.f) {
    tnx = -tnx;
    tny = -tny;
  }
  const float turn = g.param(r, RP_OMEGA) * .5f * sp.dt;
  const float next_course = course + clampf(angle_diff(atan2f(tny, tnx), course), -turn, turn);
  const float tfx = cosf(next_course), tfy = sinf(next_course);
  const float rad = robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH));
  const float gx = p[0] + tfx * 3.f, gy = p[1] + tfy * 3.f;
  if (!(gx >= rad && gx <= sp.field_length - rad && gy >= rad && gy <= sp.field_width - rad)) return;
  w.c_collect_heading[er] = next_course;
  if (!cs.approach[r]) {
    w.c_target[er * 2] = gx;
    w.c_target[er * 2 + 1] = gy;
  }
  w.c_fuel_delta[er * 2] = tfx;
  w.c_fuel_delta[er * 2 + 1] = tfy;
}

AD_HD void control_robot(G& g, int r, const int32_t* actions, const int32_t* possession, ControlScan& cs) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const int e = g.e;
  const int mode = sp.mode[r];
  float* p = g.ppose(r);
  const float* v = g.rvel(r);
  const int team = sp.team[r];
  const bool det_offense = mode == MODE_DET && sp.role[r] == 0;
  const bool defense_role = sp.role[r] == 1;
  const bool dumper = sp.kind[r] == 0;
  const int cap = sp.capacity[r];
  const int poss = possession[r];
  const bool hub_on = g.hub_active(team);
  const float L = g.param(r, RP_LENGTH), W = g.param(r, RP_WIDTH);
  const float speed = fmaxf(g.param(r, RP_SPEED), .1f);
  const float accel = fmaxf(g.param(r, RP_ACCEL), 1e-4f);
  const float rad = robot_radius_of(L, W);
  const float c = cosf(p[2]), s = sinf(p[2]);
  // intake reference (front-right corner of the intake) plus momentum
  float irx = p[0] + c * (L * .5f + .15f) + s * (W * .5f);
  float iry = p[1] + s * (L * .5f + .15f) - c * (W * .5f);
  // ranked FUEL tracks (control_scan_tracks)
  Top4 top;
  for (int k = 0; k < 4; ++k) {
    top.c[k] = cs.top_c[r][k];
    top.i[k] = cs.top_i[r][k];
  }
  const bool intake_available = cs.intake[r], alliance_fuel = cs.alliance[r], nearby_mid = cs.nearby[r];
  bool cand_valid[4];
  for (int k = 0; k < 4; ++k) {
    cand_valid[k] = top.c[k] < kInf;
    w.c_cand[g.er(r) * 4 + k] = cand_valid[k] ? top.i[k] : -1;
  }
  // legal action mask
  bool mask[8];
  for (int k = 0; k < 4; ++k) mask[k] = cand_valid[k] && poss < cap;
  mask[4] = poss > 0;
  mask[5] = w.o_valid[g.er(r)] || defense_role;
  mask[6] = mask[7] = true;
  // deterministic strategy
  int det_action = 5;
  bool ferry_inactive = false;
  if (!defense_role) {
    bool in_zone = in_alliance_zone(sp, team, p[0]);
    bool positioned = in_zone && hub_on;
    bool active_hub_return = hub_on && !nearby_mid && !positioned;
    bool gather_more = poss < cap && intake_available;
    uint8_t& sc = g.latch(r, RL_SCORE_COMMITTED);
    bool score_commit = hub_on && poss > 0 && (sc || poss >= cap || (positioned && !alliance_fuel));
    uint8_t& fc = g.latch(r, RL_FERRY_COMMITTED);
    bool begin_ferry = poss >= cap || !intake_available;
    bool ferry_commit = !hub_on && poss > 0 && (fc || begin_ferry);
    if (det_offense) {
      sc = score_commit ? 1 : 0;
      fc = ferry_commit ? 1 : 0;
    }
    ferry_inactive = !hub_on && poss > 0 && ferry_commit;
    float vs = sqrtf(v[0] * v[0] + v[1] * v[1]);
    bool braking = ferry_inactive && dumper && vs > .15f;
    det_action = ferry_inactive ? (braking ? 7 : 6) : (score_commit ? 4 : (gather_more ? 0 : 6));
    if (hub_on && !dumper && intake_available && poss < cap) det_action = 0;
    if (active_hub_return && poss > 0) det_action = 4;
  }
  int action;
  if (mode == MODE_NN) {
    action = clampi(actions ? actions[g.er(r)] : 7, 0, 7);
    if (!mask[action]) {
      int first = 7;
      for (int k = 0; k < 8; ++k)
        if (mask[k]) {
          first = k;
          break;
        }
      action = first;
    }
  } else if (mode == MODE_DET) {
    action = det_action;
    if (!mask[action]) {
      for (int k = 0; k < 8; ++k)
        if (mask[k]) {
          action = k;
          break;
        }
    }
  } else {
    action = 7;
  }
  if (mode == MODE_DIRECT) action = 7;
  bool no_track_search = det_offense && action == 6 && poss == 0 && !intake_available;
  g.latch(r, RL_NO_TRACK_SEARCH) = no_track_search;
  bool collecting = (action < 4 || no_track_search) &&
                    (!dumper || intake_deploy_clear(sp, p[0], p[1], p[2], L, W));
  w.g_action[g.er(r)] = action;
  g.latch(r, RL_INTAKE_COLLECTING) = collecting ? 1 : 0;
  bool intent = action == 4;
  if (det_offense && !dumper && hub_on && poss > 0 && !ferry_inactive) intent = true;
  g.latch(r, RL_SCORE_INTENT) = intent ? 1 : 0;
  // choose the FUEL candidate
  int sel = action < 4 ? action : 0;
  int selected = cand_valid[sel] ? top.i[sel] : (cand_valid[0] ? top.i[0] : 0);
  if (det_offense && action < 4 && intake_available) {
    // cycle-time cost per candidate; inactive HUB keeps the staging rank
    int lock = w.c_target_index[g.er(r)];
    float best = kInf;
    int best_k = -1;
    for (int k = 0; k < 4; ++k) {
      if (!cand_valid[k]) continue;
      int i = top.i[k];
      float tx = g.tx(r, i), ty = g.ty(r, i);
      size_t kk = g.erp(r, i);
      float age = fminf(fmaxf(w.t_age[kk], 0.f), 2.f);
      float detour = obstacle_detour(sp, irx, iry, tx, ty, rad);
      float cost;
      if (!hub_on) {
        cost = top.c[k];
      } else {
        float yield = fminf(cs.yield[r][k], (float)(cap - poss > 0 ? cap - poss : 0));
        float dx = tx - irx, dy = ty - iry;
        float dist = sqrtf(dx * dx + dy * dy);
        float ux = dx / fmaxf(dist, 1e-6f), uy = dy / fmaxf(dist, 1e-6f);
        float out = fminf(fmaxf(v[0] * ux + v[1] * uy, 0.f), speed);
        float drive = travel_time(dist, out, speed, accel);
        float herr = fabsf(angle_diff(atan2f(dy, dx), p[2]));
        float turn = herr / fmaxf(g.param(r, RP_OMEGA), 1e-3f);
        float pick = fmaxf(drive, turn);
        float boundary = team == 0 ? sp.alliance_depth : sp.field_length - sp.alliance_depth;
        float ret = team == 0 ? fmaxf(tx - boundary, 0.f) : fmaxf(boundary - tx, 0.f);
        float rtime = travel_time(ret, 0.f, speed, accel);
        float wait = fmaxf(g.rtime(r, RT_NEXT_INTAKE) - g.elapsed(), 0.f);
        float cycle = pick + rtime + wait + .2f + (age * .4f + detour) / speed;
        cost = cycle / fmaxf(yield, .1f);
      }
      if (i == lock) {
        best_k = k;
        best = -kInf;
        break;
      }
      if (cost < best) {
        best = cost;
        best_k = k;
      }
    }
    if (best_k >= 0) selected = top.i[best_k];
  }
  bool target_based = det_offense && (action < 4 || (action == 6 && poss == 0));
  w.c_target_index[g.er(r)] = (target_based && intake_available) ? selected : -1;
  // FUEL target with short observed-motion intercept
  float fx = g.tx(r, selected), fy = g.ty(r, selected);
  if (sp.fuel_physics) {
    float tt = fminf(sqrtf(sqr(fx - p[0]) + sqr(fy - p[1])) / speed, .5f);
    fx = clampf(fx + g.tvx(r, selected) * tt, .075f, sp.field_length - .075f);
    fy = clampf(fy + g.tvy(r, selected) * tt, .075f, sp.field_width - .075f);
  }
  w.c_fuel_target[g.er(r) * 2] = fx;
  w.c_fuel_target[g.er(r) * 2 + 1] = fy;
  float fdx = fx - p[0], fdy = fy - p[1];
  // per-action navigation targets
  float tx = p[0], ty = p[1];
  if (action < 4) {
    tx = fx;
    ty = fy;
  } else if (action == 4) {
    safe_score_target(g, r, tx, ty);
  } else if (action == 5) {
    const float* op = w.o_pose + g.er(r) * 3;
    const float* ov = w.o_vel + g.er(r) * 3;
    bool valid = w.o_valid[g.er(r)] != 0;
    if (defense_role) {
      int oteam = 1 - team;
      float post_x = sp.hub_x[oteam] + (oteam == 0 ? -1.f : 1.f) * fmaxf(.595f + rad - .15f, .85f);
      float post_y = sp.hub_y[oteam];
      if (valid) {
        float es = sqrtf(ov[0] * ov[0] + ov[1] * ov[1]);
        float dx = p[0] - op[0], dy = p[1] - op[1];
        float dn = fmaxf(sqrtf(dx * dx + dy * dy), 1e-6f);
        float ux = es > .15f ? ov[0] / fmaxf(es, .15f) : dx / dn;
        float uy = es > .15f ? ov[1] / fmaxf(es, .15f) : dy / dn;
        float ti = clampf(sqrtf(sqr(op[0] - p[0]) + sqr(op[1] - p[1])) / speed, 0.f, 1.25f);
        tx = op[0] + ov[0] * ti + ux * .55f;
        ty = op[1] + ov[1] * ti + uy * .55f;
      } else {
        tx = post_x;
        ty = post_y;
      }
    } else if (valid) {
      tx = op[0];
      ty = op[1];
    }
  } else if (action == 6) {
    float ftx, fty;
    ferry_target(g, r, ftx, fty);
    bool dumper_ferry = dumper && poss > 0 && !hub_on;
    tx = dumper_ferry ? p[0] : ftx;
    ty = dumper_ferry ? p[1] : fty;
  }
  // scripted offense collection: raster sweep, or cluster collection with
  // contour tracing and intake-strip approach poses
  bool raster_sweep = det_offense && no_track_search;
  cs.edge[r] = 0;
  cs.approach[r] = 0;
  if (sp.sweeping) {
    const bool sweeping = det_offense && (action < 4 || (action == 6 && poss == 0));
    if (sweeping) {
      raster_target(g, r, tx, ty, fdx, fdy);
      raster_sweep = true;
    }
  } else if (env_has_det_offense(sp)) {
    collection_targets(g, r, action, poss, no_track_search, alliance_fuel, cand_valid, top.i, irx, iry, fx, fy,
                       fdx, fdy, tx, ty, cs);
  }
  g.latch(r, RL_RASTER_SWEEP) = raster_sweep ? 1 : 0;
  if (sp.R == 2 && r == 1 && mode == MODE_DET && sp.opponent_kind >= OPP_DEF_INTERCEPT) {
    // scripted defender of the counter-defense task: a waypoint from its
    // tracks, reached through the route planner and path follower
    defense_target(g, r, 0, sp.opponent_kind, cand_valid[0], top.i[0], tx, ty);
  } else if (sp.R == 2 && r == 1 && mode == MODE_DET && sp.opponent_kind != OPP_OFFENSE) {
    // scripted two-robot attacker variants steer straight at a derived point
    // (frc_defense/tensor_defense_step.py:108-180)
    float gx, gy;
    attacker_objective(g, r, possession, gx, gy);
    const float* dp = g.ppose(0);
    const float* dv = g.rvel(0);
    if (sp.opponent_kind == OPP_MIRROR) {
      tx = 2.f * gx - dp[0];
      ty = 2.f * gy - dp[1];
    } else if (sp.opponent_kind == OPP_CUTOFF) {
      float rx = gx - dp[0], ry = gy - dp[1];
      float rn = fmaxf(sqrtf(rx * rx + ry * ry), 1e-8f);
      tx = dp[0] + dv[0] * .45f + rx / rn * .65f;
      ty = dp[1] + dv[1] * .45f + ry / rn * .65f;
    } else if (sp.opponent_kind == OPP_VELOCITY_INTERCEPT) {
      float dist = sqrtf(sqr(dp[0] - p[0]) + sqr(dp[1] - p[1]));
      float t = clampf(dist / speed, 0.f, 1.5f);
      tx = dp[0] + dv[0] * t;
      ty = dp[1] + dv[1] * t;
    } else {
      tx = gx;
      ty = gy;
    }
    tx = clampf(tx, 0.f, sp.field_length);
    ty = clampf(ty, 0.f, sp.field_width);
  }
  w.c_target[g.er(r) * 2] = tx;
  w.c_target[g.er(r) * 2 + 1] = ty;
  w.c_fuel_delta[g.er(r) * 2] = fdx;
  w.c_fuel_delta[g.er(r) * 2 + 1] = fdy;
  (void)e;
}

// ---------------------------------------------------------------------------
// Path following (frc_defense/tensor_adstar.py:1470-1536).
// ---------------------------------------------------------------------------
AD_HD void path_reference(G& g, int r, float& cmdx, float& cmdy, float& tanx, float& tany) {
  World& w = g.w;
  const size_t er = g.er(r);
  const float* path = w.p_path + er * kPathPoints * 2;
  const float* prof = w.p_profile + er * kPathPoints;
  const int len = w.p_len[er];
  float& progress_ref = w.p_progress[er];
  const float* pp = g.ppose(r);
  const float* vv = g.rvel(r);
  const float px = pp[0], py = pp[1], vx = vv[0], vy = vv[1];
  cmdx = cmdy = tanx = tany = 0.f;
  if (len <= 1) return;
  const int K = kPathPoints;
  // stations
  float station[kPathPoints];
  station[0] = 0.f;
  for (int k = 0; k < K - 1; ++k) {
    float dx = path[(k + 1) * 2] - path[k * 2], dy = path[(k + 1) * 2 + 1] - path[k * 2 + 1];
    station[k + 1] = station[k] + sqrtf(dx * dx + dy * dy);
  }
  float best = kInf;
  int idx = 0;
  float best_frac = 0.f;
  const float lo = fmaxf(progress_ref - .08f, 0.f);
  for (int k = 0; k < K - 1 && k < len - 1; ++k) {
    if (!(station[k + 1] >= lo)) continue;
    float sx = path[(k + 1) * 2] - path[k * 2], sy = path[(k + 1) * 2 + 1] - path[k * 2 + 1];
    float d2 = fmaxf(sx * sx + sy * sy, 1e-12f);
    float f = clampf(((px - path[k * 2]) * sx + (py - path[k * 2 + 1]) * sy) / d2, 0.f, 1.f);
    float qx = path[k * 2] + f * sx, qy = path[k * 2 + 1] + f * sy;
    float sq = sqr(qx - px) + sqr(qy - py);
    if (sq < best) {
      best = sq;
      idx = k;
      best_frac = f;
    }
  }
  float seg = station[idx + 1] - station[idx];
  float progress = station[idx] + best_frac * seg;
  progress = fminf(fmaxf(progress, progress_ref), station[K - 1]);
  float sxi = path[(idx + 1) * 2] - path[idx * 2], syi = path[(idx + 1) * 2 + 1] - path[idx * 2 + 1];
  float projx = path[idx * 2] + best_frac * sxi, projy = path[idx * 2 + 1] + best_frac * syi;
  progress_ref = progress;
  float current = sqrtf(vx * vx + vy * vy);
  float look = clampf(.2f + .2f * fminf(current, 4.5f), .2f, 1.2f);
  float target_station = fminf(progress + look, station[K - 1]);
  int ts = 0;
  for (int k = 0; k < K - 1; ++k)
    if (station[k + 1] < target_station) ts++;
  ts = ts > K - 2 ? K - 2 : ts;
  float td = station[ts + 1] - station[ts];
  float tsx = path[(ts + 1) * 2] - path[ts * 2], tsy = path[(ts + 1) * 2 + 1] - path[ts * 2 + 1];
  tanx = tsx / fmaxf(td, 1e-6f);
  tany = tsy / fmaxf(td, 1e-6f);
  float nx = -tany, ny = tanx;
  float cross = (px - projx) * nx + (py - projy) * ny;
  float cross_v = vx * nx + vy * ny;
  float lateral = clampf(-3.f * cross - 4.f * cross_v, -.75f, .75f);
  int ss = 0;
  for (int k = 0; k < K - 1; ++k)
    if (station[k + 1] < progress) ss++;
  ss = ss > K - 2 ? K - 2 : ss;
  float sd = station[ss + 1] - station[ss];
  float sf = clampf((progress - station[ss]) / fmaxf(sd, 1e-8f), 0.f, 1.f);
  float planned = prof[ss] * (1.f - sf) + prof[ss + 1] * sf;
  planned = fmaxf(fminf(planned, g.param(r, RP_SPEED)), 0.f);
  float target = fmaxf(planned - .55f * fmaxf(current - planned, 0.f), 0.f);
  cmdx = tanx * target + nx * lateral;
  cmdy = tany * target + ny * lateral;
}

// Teammate right-of-way and reaction to the anonymous opponent track
// (frc_defense/_tensor_3v3_actions.py:900-1020). cmd is [R][2], updated in place.
AD_HD void avoid_contention(G& g, float* cmd) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  float avoid[kMaxRobots * 2];
  float count[kMaxRobots];
  for (int r = 0; r < sp.R; ++r) {
    avoid[r * 2] = avoid[r * 2 + 1] = 0.f;
    count[r] = 0.f;
    if (sp.mode[r] == MODE_NONE) cmd[r * 2] = cmd[r * 2 + 1] = 0.f;
  }
  for (int q = 0; q < sp.Q; ++q) {
    int i = sp.pair_i[q], j = sp.pair_j[q];
    int32_t& winner_slot = w.c_avoid[(size_t)g.e * sp.Q + q];
    bool teammates = sp.team[i] == sp.team[j];
    bool ic = sp.mode[i] != MODE_NONE, jc = sp.mode[j] != MODE_NONE;
    if (!teammates || !(ic || jc)) {
      winner_slot = -1;
      continue;
    }
    const float* pi = g.ppose(i);
    const float* pj = g.ppose(j);
    float rx = pi[0] - pj[0], ry = pi[1] - pj[1];
    float rvx = cmd[i * 2] - cmd[j * 2], rvy = cmd[i * 2 + 1] - cmd[j * 2 + 1];
    float cs = rvx * rvx + rvy * rvy;
    float t = clampf(-(rx * rvx + ry * rvy) / fmaxf(cs, 1e-6f), 0.f, .7f);
    float clx = rx + rvx * t, cly = ry + rvy * t;
    float cd = sqrtf(clx * clx + cly * cly), cur = sqrtf(rx * rx + ry * ry);
    float ri = robot_radius_of(g.param(i, RP_LENGTH), g.param(i, RP_WIDTH));
    float rj = robot_radius_of(g.param(j, RP_LENGTH), g.param(j, RP_WIDTH));
    float clearance = ri + rj + .25f;
    bool conflict;
    if (sp.teammate_coordination)
      conflict = (cs > .0225f && cd < clearance) || cur < clearance - .08f;
    else
      conflict = cur < clearance + .05f;
    int preferred = i < j ? i : j;
    if (sp.teammate_coordination) {
      float di = sqrtf(sqr(w.c_target[g.er(i) * 2] - pi[0]) + sqr(w.c_target[g.er(i) * 2 + 1] - pi[1]));
      float dj = sqrtf(sqr(w.c_target[g.er(j) * 2] - pj[0]) + sqr(w.c_target[g.er(j) * 2 + 1] - pj[1]));
      preferred = di <= dj ? i : j;
      if (ic && !jc) preferred = j;
      if (!ic && jc) preferred = i;
    }
    bool retained = winner_slot >= 0 && cur < clearance + .35f && sp.teammate_coordination;
    int winner = retained ? winner_slot : (conflict ? preferred : -1);
    winner_slot = winner;
    if (!conflict) continue;
    bool i_pri = winner == i;
    int loser = i_pri ? j : i;
    float lcx = cmd[loser * 2], lcy = cmd[loser * 2 + 1];
    float sx = i_pri ? -clx : clx, sy = i_pri ? -cly : cly;
    if (sqrtf(sx * sx + sy * sy) < .1f) {
      sx = i_pri ? -rx : rx;
      sy = i_pri ? -ry : ry;
    }
    float sn = fmaxf(sqrtf(sx * sx + sy * sy), 1e-5f);
    float radx = sx / sn, rady = sy / sn;
    float tgx = -rady, tgy = radx;
    if (tgx * lcx + tgy * lcy < 0.f) {
      tgx = -tgx;
      tgy = -tgy;
    }
    float ds = fmaxf(sqrtf(lcx * lcx + lcy * lcy), .65f);
    avoid[loser * 2] += ds * (tgx + .75f * radx);
    avoid[loser * 2 + 1] += ds * (tgy + .75f * rady);
    count[loser] += 1.f;
  }
  for (int r = 0; r < sp.R; ++r) {
    if (count[r] > 0.f) {
      float ax = avoid[r * 2] / count[r], ay = avoid[r * 2 + 1] / count[r];
      float as = fmaxf(sqrtf(ax * ax + ay * ay), 1e-6f);
      float k = fminf(1.f, g.param(r, RP_SPEED) / as);
      cmd[r * 2] = ax * k;
      cmd[r * 2 + 1] = ay * k;
    }
    // react to the anonymous observed opponent
    size_t er = g.er(r);
    const float* op = w.o_pose + er * 3;
    const float* ov = w.o_vel + er * 3;
    const float* os = w.o_size + er * 3;
    bool valid = w.o_valid[er] && os[0] > 0.f && os[1] > 0.f && sp.mode[r] != MODE_NONE;
    if (!valid) continue;
    const float* p = g.ppose(r);
    float rx = p[0] - op[0], ry = p[1] - op[1];
    float rvx = cmd[r * 2] - ov[0], rvy = cmd[r * 2 + 1] - ov[1];
    float s2 = rvx * rvx + rvy * rvy;
    float t = clampf(-(rx * rvx + ry * rvy) / fmaxf(s2, 1e-6f), 0.f, .7f);
    float clx = rx + rvx * t, cly = ry + rvy * t;
    float cn = sqrtf(clx * clx + cly * cly);
    float clearance = robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH)) +
                      .5f * sqrtf(os[0] * os[0] + os[1] * os[1]) + .25f;
    bool conflict = (s2 > .0225f && cn < clearance) || sqrtf(rx * rx + ry * ry) < clearance - .08f;
    if (!conflict) continue;
    float sx = cn < .1f ? rx : clx, sy = cn < .1f ? ry : cly;
    float sn = fmaxf(sqrtf(sx * sx + sy * sy), 1e-5f);
    float radx = sx / sn, rady = sy / sn;
    float tgx = -rady, tgy = radx;
    if (tgx * cmd[r * 2] + tgy * cmd[r * 2 + 1] < 0.f) {
      tgx = -tgx;
      tgy = -tgy;
    }
    float ds = fmaxf(sqrtf(sqr(cmd[r * 2]) + sqr(cmd[r * 2 + 1])), .65f);
    float ax = ds * (tgx + .75f * radx), ay = ds * (tgy + .75f * rady);
    float as = fmaxf(sqrtf(ax * ax + ay * ay), 1e-6f);
    float k = fminf(1.f, g.param(r, RP_SPEED) / as);
    cmd[r * 2] = ax * k;
    cmd[r * 2 + 1] = ay * k;
  }
}

// Command synthesis for one tick: path following, heading control, intake
// approach rules, stopping rules and contention avoidance. Writes c_command.
AD_HD void synthesize_commands(G& g, const int32_t* possession) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  float cmd[kMaxRobots * 2];
  float omega[kMaxRobots];
  for (int r = 0; r < sp.R; ++r) {
    const size_t er = g.er(r);
    const float* p = g.ppose(r);
    const float* v = g.rvel(r);
    const int action = w.g_action[er];
    const int team = sp.team[r];
    const bool dumper = sp.kind[r] == 0;
    const bool carrying = possession[r] > 0;
    const bool det_offense = sp.mode[r] == MODE_DET && sp.role[r] == 0;
    const float omega_lim = g.param(r, RP_OMEGA), alpha = g.param(r, RP_ALPHA);
    const float speed = g.param(r, RP_SPEED);
    float cx, cy, tnx, tny;
    path_reference(g, r, cx, cy, tnx, tny);
    // heading
    float hb = atan2f(sp.hub_y[team] - p[1], sp.hub_x[team] - p[0]);
    float aerr = angle_diff(hb, p[2]);
    bool scoring_dumper = action == 4 && carrying && dumper;
    bool centered = scoring_dumper && fabsf(aerr) <= 0.0872665f;
    float om = swerve_heading_rate(centered ? 0.f : aerr, omega_lim, alpha, v[2], sp.dt, true);
    if (scoring_dumper && fabsf(aerr) <= 0.261799f) {
      om = centered ? 0.f : clampf(3.f * aerr - 1.5f * v[2], -omega_lim, omega_lim);
    }
    if (!scoring_dumper) om = 0.f;
    float ax, ay;
    ferry_aim_point(sp, team, p[0], p[1], ax, ay);
    float ferr = angle_diff(atan2f(ay - p[1], ax - p[0]), p[2]);
    bool ferrying = action == 6 && carrying && dumper;
    bool braking = action == 7 && carrying && dumper && !g.hub_active(team);
    if (ferrying || braking) om = swerve_heading_rate(ferr, omega_lim, alpha, v[2], sp.dt, true);
    bool pickup_active = det_offense && (action < 4 || (action == 6 && !carrying));
    const float* ft = w.c_fuel_target + er * 2;
    const float* fd = w.c_fuel_delta + er * 2;
    const float* tg = w.c_target + er * 2;
    float pfx = ft[0] - p[0], pfy = ft[1] - p[1];
    float pfd = sqrtf(pfx * pfx + pfy * pfy);
    float dirx = fd[0], diry = fd[1];
    if (pickup_active) {
      float tn = sqrtf(tnx * tnx + tny * tny);
      float fbx = action < 4 ? fd[0] : tg[0] - p[0], fby = action < 4 ? fd[1] : tg[1] - p[1];
      float tbx = tn > .5f ? tnx : fbx, tby = tn > .5f ? tny : fby;
      float ferr2 = fabsf(angle_diff(atan2f(pfy, pfx), p[2]));
      float turn_dist = speed * ferr2 / fmaxf(omega_lim, .1f);
      float approach = fmaxf(.9f, turn_dist);
      if (!w.g_rlatch[er * kLatches + RL_TARGET_COLLECTING] && pfd <= approach) {
        tbx = fd[0];
        tby = fd[1];
      }
      dirx = tbx;
      diry = tby;
    }
    float perr = angle_diff(atan2f(diry, dirx), p[2]);
    if (pickup_active) om = swerve_heading_rate(perr, omega_lim, alpha, v[2], sp.dt, true);
    const bool trench = w.p_trench[er] != 0;
    float therr = angle_diff(w.p_heading[er], p[2]);
    if (trench) om = swerve_heading_rate(therr, omega_lim, alpha, v[2], sp.dt, true);
    if (trench && fabsf(therr) > .25f) cx = cy = 0.f;
    float tdx = tg[0] - p[0], tdy = tg[1] - p[1];
    float dist = sqrtf(tdx * tdx + tdy * tdy);
    if (det_offense) {
      // direct bridge for a stalled collector whose straight path is clear
      float dn = fmaxf(dist, 1e-6f);
      float ds = fminf(speed, dist * 6.f);
      bool stalled = pickup_active && !trench && dist > .03f &&
                     (dist < 1.6f || sqrtf(cx * cx + cy * cy) < .05f);
      if (stalled) {
        // straight-line footprint check against solid boxes
        float rad = robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH)) * .5f;
        float det = obstacle_detour(sp, p[0], p[1], tg[0], tg[1], rad);
        bool clear = det <= 0.f;
        if (clear) {
          cx = tdx / dn * ds;
          cy = tdy / dn * ds;
        }
      }
      // nonholonomic final intake approach
      float fwx = cosf(p[2]), fwy = sinf(p[2]);
      float rtx = sinf(p[2]), rty = -cosf(p[2]);
      if (pickup_active && pfd <= .7f) {
        float fs = cx * fwx + cy * fwy;
        cx = fwx * fs;
        cy = fwy * fs;
        float latv = v[0] * rtx + v[1] * rty;
        if (fabsf(perr) > .25f || fabsf(latv) > .15f) cx = cy = 0.f;
      }
      // stop at the first bump-clear pose inside the scoring zone
      bool scorer = action == 4 && carrying;
      if (scorer && in_alliance_zone(sp, team, p[0]) &&
          clear_of_bumps(sp, p[0], p[1], robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH))))
        cx = cy = 0.f;
      float stop = scorer ? .02f : (pickup_active ? 0.f : .3f);
      if (dist <= stop) cx = cy = 0.f;
    } else if (dist <= .3f) {
      cx = cy = 0.f;
    }
    if (action == 7) cx = cy = 0.f;
    // trench crossing at the aligned heading
    if (trench && fabsf(therr) <= .25f && w.p_len[er] > 1) {
      float fwx = cosf(w.p_heading[er]), fwy = sinf(w.p_heading[er]);
      const float* gl = w.p_goal + er * 2;
      float rem = fmaxf((gl[0] - p[0]) * fwx + (gl[1] - p[1]) * fwy, 0.f);
      float cs = fminf(speed, rem * 6.f);
      cx = fwx * cs;
      cy = fwy * cs;
    }
    cmd[r * 2] = cx;
    cmd[r * 2 + 1] = cy;
    omega[r] = om;
  }
  avoid_contention(g, cmd);
  if (sp.R == 2 && sp.mode[1] == MODE_DET && sp.opponent_kind != OPP_OFFENSE &&
      sp.opponent_kind < OPP_DEF_INTERCEPT) {
    const size_t er = g.er(1);
    const float* p = g.ppose(1);
    const float* tg = w.c_target + er * 2;
    float dx = tg[0] - p[0], dy = tg[1] - p[1];
    float dn = fmaxf(sqrtf(dx * dx + dy * dy), 1e-8f);
    float speed = g.param(1, RP_SPEED);
    if (sp.opponent_kind == OPP_RANDOM) {
      const Rng rng{sp.seed0, sp.seed1};
      U4 u = rng.draw((uint32_t)g.e, (uint32_t)w.g_steps[(size_t)g.e * 2] ^ ((uint32_t)w.e_episode[g.e] << 14),
                      RNG_DEFENSE, 1u);
      float th = u01(u.x) * kTwoPi, sv = u01(u.y) * speed;
      cmd[2] = cosf(th) * sv;
      cmd[3] = sinf(th) * sv;
    } else {
      cmd[2] = dx / dn * speed;
      cmd[3] = dy / dn * speed;
    }
    bool carrying = possession[1] > 0;
    float hb = atan2f(sp.hub_y[1] - p[1], sp.hub_x[1] - p[0]);
    omega[1] = carrying ? swerve_heading_rate(angle_diff(hb, p[2]), g.param(1, RP_OMEGA), g.param(1, RP_ALPHA),
                                              g.rvel(1)[2], sp.dt, true)
                        : 0.f;
  }
  for (int r = 0; r < sp.R; ++r) {
    const size_t er = g.er(r);
    const float* p = g.ppose(r);
    if (sp.mode[r] == MODE_DIRECT) continue;  // command supplied by the caller
    if (w.g_rlatch[er * kLatches + RL_STATIC_OPPONENT]) {       // parked (static) opponent this episode
      float* out = w.c_command + er * 3;
      out[0] = out[1] = out[2] = 0.f;
      continue;
    }
    bool trench = w.p_trench[er] != 0;
    float therr = angle_diff(w.p_heading[er], p[2]);
    float cx = cmd[r * 2], cy = cmd[r * 2 + 1];
    if (trench && fabsf(therr) > .25f) cx = cy = 0.f;
    bool enabled = sp.mode[r] != MODE_NONE;
    float* out = w.c_command + er * 3;
    out[0] = enabled ? cx : 0.f;
    out[1] = enabled ? cy : 0.f;
    out[2] = enabled ? omega[r] : 0.f;
  }
}

}  // namespace ad
