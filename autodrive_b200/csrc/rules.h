// FUEL actions (pickup, ferry, scoring, respawn), perception, observations and
// rewards for one environment. See game.h for the reference map.
#pragma once

#include "game.h"

namespace ad {

// Segment of a robot footprint (circle of `radius`) against solid boxes.
AD_HD bool segment_clear(const SimParams& sp, float x0, float y0, float x1, float y1, float radius) {
  for (int b = 0; b < sp.num_boxes; ++b) {
    const Box& bx = sp.boxes[b];
    float hx = bx.hx + radius, hy = bx.hy + radius;
    float lo[2] = {bx.cx - hx, bx.cy - hy}, hi[2] = {bx.cx + hx, bx.cy + hy};
    float p0[2] = {x0, y0}, d[2] = {x1 - x0, y1 - y0};
    float enter = 0.f, leave = 1.f;
    bool ok = true;
    for (int a = 0; a < 2; ++a) {
      if (fabsf(d[a]) < 1e-9f) {
        if (p0[a] < lo[a] || p0[a] > hi[a]) ok = false;
      } else {
        float t0 = (lo[a] - p0[a]) / d[a], t1 = (hi[a] - p0[a]) / d[a];
        enter = fmaxf(enter, fminf(t0, t1));
        leave = fminf(leave, fmaxf(t0, t1));
      }
    }
    if (ok && enter <= leave) return false;
  }
  return true;
}

// Launch a FUEL piece on a ballistic arc (frc_defense/fuel_physics_runtime.py:383-450).
// `ground` places it on the terrain at (px, py) with zero vertical speed.
AD_HD void launch_piece(TickShared& s, const SimParams& sp, int i, float px, float py, float vx, float vy,
                        float height, float flight, bool ground) {
  s.fpos[0][i] = px;
  s.fpos[1][i] = py;
  if (ground) {
    s.fpos[2][i] = fuel_spawn_height(sp, px, py);
    s.fvel[2][i] = 0.f;
  } else {
    float z = fmaxf(height, sp.fr);
    s.fpos[2][i] = z;
    s.fvel[2][i] = (sp.fr - z) / flight + .5f * sp.fg * flight;
  }
  s.fvel[0][i] = vx;
  s.fvel[1][i] = vy;
  for (int k = 0; k < 3; ++k) s.fang[k][i] = 0.f;
  s.sleep[i] = 0;
  s.clock[i] = 0.f;
}

// Shooter respawn: HUB exit point and midfield launch target inside a 45-degree
// cone (frc_defense/fuel_physics_runtime.py:223-243).
AD_HD void shooter_cone(const SimParams& sp, int team, float u, float& sx, float& sy, float& tx, float& ty) {
  float hx = sp.hub_x[team], hy = sp.hub_y[team];
  float mx = sp.field_length * .5f, my = sp.field_width * .5f;
  float bearing = atan2f(my - hy, mx - hx);
  float angle = bearing + (u - .5f) * (kPi / 4.f);
  float dx = cosf(angle), dy = sinf(angle);
  float clearance = 47.f * .0254f / 2.f + sp.fr + .05f;
  float dist = clearance / fmaxf(fabsf(dx), 1e-6f);
  sx = hx + dist * dx;
  sy = hy + dist * dy;
  float ld = sqrtf(sqr(mx - hx) + sqr(my - hy));
  tx = hx + ld * dx;
  ty = hy + ld * dy;
}

// Midfield respawn corridor point k of `count` (golden-ratio sequence).
AD_HD void midfield_point(const SimParams& sp, int k, int count, float& x, float& y) {
  float cx = sp.field_length * .5f, cy = sp.field_width * .5f;
  float x0 = cx - 1.65f, x1 = cx + 1.65f, y0 = cy - 2.615f, y1 = cy + 2.615f;
  const float phi = 0.6180339887498949f;
  float frac = (float)k * phi;
  frac -= floorf(frac);
  x = x0 + ((float)k + .5f) * (x1 - x0) / (float)count;
  y = y0 + frac * (y1 - y0);
}

// Ferry landing: 10-degree cone toward the friendly aim point, clipped at the
// field edge; a path through the exposed HUB backer net returns to midfield
// (frc_defense/fuel_physics_runtime.py:246-311). Returns true on a net hit.
AD_HD bool ferry_landing(const SimParams& sp, int team, float ox, float oy, float u_angle, float u_mid,
                         float& lx, float& ly) {
  float ax, ay;
  ferry_aim_point(sp, team, ox, oy, ax, ay);
  float dx = ax - ox, dy = ay - oy;
  float bearing = atan2f(dy, dx);
  float angle = bearing + (u_angle - .5f) * 0.17453293f;
  float dist = sqrtf(dx * dx + dy * dy);
  float tx = ox + dist * cosf(angle), ty = oy + dist * sinf(angle);
  float ddx = tx - ox, ddy = ty - oy;
  float lo[2] = {sp.fr, sp.fr}, hi[2] = {sp.field_length - sp.fr, sp.field_width - sp.fr};
  float o[2] = {ox, oy}, d[2] = {ddx, ddy};
  float travel = 1.f;
  for (int a = 0; a < 2; ++a) {
    if (fabsf(d[a]) > 1e-8f) {
      float bound = d[a] > 0.f ? hi[a] : lo[a];
      travel = fminf(travel, (bound - o[a]) / d[a]);
    }
  }
  travel = clampf(travel, 0.f, 1.f);
  lx = clampf(ox + travel * ddx, sp.fr, sp.field_length - sp.fr);
  ly = clampf(oy + travel * ddy, sp.fr, sp.field_width - sp.fr);
  const float inch = .0254f;
  float net_half = (47.f * inch + 73.f * inch) / 2.f - 73.f * inch / 2.f - sp.fr;
  float face = sp.hub_x[team] + (team == 0 ? 47.f * inch / 2.f : -47.f * inch / 2.f);
  float fdx = lx - ox;
  if (fabsf(fdx) > 1e-8f) {
    float f = (face - ox) / fdx;
    float cy = oy + f * (ly - oy);
    if (f >= 0.f && f <= 1.f && fabsf(cy - sp.hub_y[team]) <= net_half) {
      int k = clampi((int)(u_mid * sp.P), 0, sp.P - 1);
      midfield_point(sp, k, sp.P, lx, ly);
      return true;
    }
  }
  return false;
}

// Scratch words in TickShared::red used by fuel_actions (no other user then).
constexpr int kFaWords = (kMaxPieces + 31) / 32;       // one bit per piece
constexpr int kFaElig = 0;                              // eligible-piece bitmap
constexpr int kFaHeld = kFaElig + kFaWords;             // held-piece bitmap per robot
constexpr int kFaPoss = kFaHeld + kMaxRobots * kFaWords;  // possession counts
constexpr int kFaMin = (kFaPoss + kMaxRobots + 1) & ~1;   // packed (d^2, index) minimum, 8-byte aligned
static_assert(kFaMin + 2 <= kRedSlots * 20, "fuel_actions scratch exceeds TickShared::red");

AD_HD uint32_t* fa_words(TickShared& s) { return reinterpret_cast<uint32_t*>(s.red); }

AD_HD void fa_set_bit(uint32_t* words, int i) {
#if defined(__CUDA_ARCH__)
  atomicOr(&words[i >> 5], 1u << (i & 31));
#else
  words[i >> 5] |= 1u << (i & 31);
#endif
}

// Index of the lowest set bit at or after `from` in a kFaWords bitmap, or -1.
AD_HD int fa_next_bit(const uint32_t* words, int from, int n) {
  for (int wi = from >> 5; wi < kFaWords && (wi << 5) < n; ++wi) {
    uint32_t m = words[wi];
    if (wi == (from >> 5)) m &= ~0u << (from & 31);
    if (m) {
#if defined(__CUDA_ARCH__)
      const int b = (wi << 5) + __ffs(m) - 1;
#else
      const int b = (wi << 5) + __builtin_ctz(m);
#endif
      return b < n ? b : -1;
    }
  }
  return -1;
}

// Pickup, carried-piece follow, ferry release and scoring for one tick
// (frc_defense/gamepiece_actions.py:128-511). s.pos/vel/ang hold the FUEL state.
// Robots act in slot order. Element scans run across the CTA; the per-robot decisions stay on
// one thread in slot order, so the outcome equals the serial definition:
// a sweeping robot takes the first `room` eligible pieces by index, a single
// intake takes the nearest eligible piece (ties to the lower index), and
// ferry / scoring act on a robot's lowest-index held piece.
AD_HD void fuel_actions(G& g, TickShared& s, const Rng& rng, uint32_t tick) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const int e = g.e;
  const float el = g.elapsed();
  const size_t base = (size_t)e * sp.P;
  uint32_t* fw = fa_words(s);
  int32_t* possession = reinterpret_cast<int32_t*>(fw + kFaPoss);
  unsigned long long* best_key = reinterpret_cast<unsigned long long*>(fw + kFaMin);
  PAR_FOR(k, kFaPoss + kMaxRobots) { fw[k] = 0u; }
  SERIAL_BEGIN
  for (int r = 0; r < sp.R; ++r) {
    g.rcount(r, RC_ACQUIRED_EVENT) = 0;
    g.rcount(r, RC_SCORED_EVENT) = 0;
    g.rcount(r, RC_PASSED_EVENT) = 0;
    g.rcount(r, RC_DENIED_EVENT) = 0;
  }
  SERIAL_END
  BARRIER();
  PAR_FOR(i, sp.P) {
    const int o = w.f_owner[base + i];
    if (o >= 0 && o < sp.R) {
#if defined(__CUDA_ARCH__)
      atomicAdd(&possession[o], 1);
#else
      possession[o]++;
#endif
    }
  }
  BARRIER();
  // ---- pickup, robots in slot order
  for (int r = 0; r < sp.R; ++r) {
    if (sp.mode[r] == MODE_NONE) continue;
    const bool extended = sp.kind[r] == 1 || g.latch(r, RL_INTAKE_COLLECTING);
    if (!extended) continue;
    const float* rp = w.r_pose + g.er(r) * 3;
    const float L = g.param(r, RP_LENGTH), W = g.param(r, RP_WIDTH);
    const bool det_offense = sp.mode[r] == MODE_DET && sp.role[r] == 0;
    const int team = sp.team[r];
    const bool hub_on = g.hub_active(team);
    const float c = cosf(rp[2]), sn = sinf(rp[2]);
    const float fr = sp.fuel_radius_rules;
    const float lon_lo = L * .5f - .075f - fr, lon_hi = L * .5f + .35f + .3048f + fr;
    const float lat_hi = W * .5f + .075f + fr;
    const int room = sp.capacity[r] - possession[r];
    const bool can_single = el + 1e-6f >= g.rtime(r, RT_NEXT_INTAKE) && possession[r] < sp.capacity[r];
    if (!det_offense && !can_single) continue;
    PAR_FOR(k, kFaWords) { fw[kFaElig + k] = 0u; }
    SERIAL_BEGIN
    *best_key = ~0ull;
    SERIAL_END
    BARRIER();
    PAR_FOR(i, sp.P) {
      if (w.f_active[base + i] && w.f_owner[base + i] < 0 && !(sp.fuel_physics && s.fpos[2][i] > .20f)) {
        const float dx = s.fpos[0][i] - rp[0], dy = s.fpos[1][i] - rp[1];
        const bool skip = det_offense && !hub_on && in_alliance_zone(sp, team, s.fpos[0][i]);
        const float lon = dx * c + dy * sn, lat = fabsf(-dx * sn + dy * c);
        if (!skip && lon >= lon_lo && lon <= lon_hi && lat <= lat_hi) {
          if (det_offense) {
            fa_set_bit(fw + kFaElig, i);
          } else {
            const float d2 = dx * dx + dy * dy;
            // non-negative floats order like their bit patterns
            const unsigned long long key = ((unsigned long long)float_bits(d2) << 32) | (unsigned)i;
            if (d2 < kInf) {
#if defined(__CUDA_ARCH__)
              atomicMin(best_key, key);
#else
              if (key < *best_key) *best_key = key;
#endif
            }
          }
        }
      }
    }
    BARRIER();
    SERIAL_BEGIN
    int picked = 0;
    if (det_offense) {
      for (int i = fa_next_bit(fw + kFaElig, 0, sp.P); i >= 0 && picked < room; i = fa_next_bit(fw + kFaElig, i + 1, sp.P)) {
        w.f_owner[base + i] = (int8_t)r;
        ++picked;
      }
    } else if (*best_key != ~0ull) {
      const int i = (int)(*best_key & 0xffffffffull);
      w.f_owner[base + i] = (int8_t)r;
      g.rtime(r, RT_NEXT_INTAKE) = el + .20f;
      picked = 1;
    }
    possession[r] += picked;
    g.rcount(r, RC_ACQUIRED_EVENT) = picked;
    SERIAL_END
    BARRIER();
  }
  // held-piece bitmaps (lowest index = the piece a robot releases or scores first)
  PAR_FOR(i, sp.P) {
    const int o = w.f_owner[base + i];
    if (w.f_active[base + i] && o >= 0 && o < sp.R) fa_set_bit(fw + kFaHeld + o * kFaWords, i);
  }
  BARRIER();
  SERIAL_BEGIN
  int next_held[kMaxRobots];
  for (int r = 0; r < sp.R; ++r) next_held[r] = fa_next_bit(fw + kFaHeld + r * kFaWords, 0, sp.P);
  // ---- ferry release: first held piece of each robot facing home
  for (int r = 0; r < sp.R; ++r) {
    if (sp.mode[r] == MODE_NONE || w.g_action[g.er(r)] != 6 || possession[r] == 0) continue;
    const float* rp = w.r_pose + g.er(r) * 3;
    const int team = sp.team[r];
    const bool dumper = sp.kind[r] == 0;
    float ftx, fty;
    ferry_target(g, r, ftx, fty);
    bool at_ferry = sqrtf(sqr(rp[0] - ftx) + sqr(rp[1] - fty)) <= .35f;
    float ax, ay;
    ferry_aim_point(sp, team, rp[0], rp[1], ax, ay);
    float herr = fabsf(angle_diff(atan2f(ay - rp[1], ax - rp[0]), rp[2]));
    bool facing = herr <= kPi / 4.f || !dumper;
    bool ready = el + 1e-6f >= g.rtime(r, RT_NEXT_FERRY);
    if (!((at_ferry || dumper) && facing && ready)) continue;
    const int first = next_held[r];
    if (first < 0) continue;
    next_held[r] = fa_next_bit(fw + kFaHeld + r * kFaWords, first + 1, sp.P);
    U4 u = rng.draw((uint32_t)e, tick, RNG_LAUNCH, (uint32_t)(r * 2));
    float lx, ly;
    bool net = ferry_landing(sp, team, rp[0], rp[1], u01(u.x), u01(u.y), lx, ly);
    if (!sp.fuel_physics) {
      s.fpos[0][first] = lx;
      s.fpos[1][first] = ly;
      for (int k = 0; k < 3; ++k) s.fvel[k][first] = 0.f;
    } else if (!net) {
      launch_piece(s, sp, first, lx, ly, (lx - rp[0]) * .1f / .5f, (ly - rp[1]) * .1f / .5f, 0.f, .5f, true);
    } else {
      float sx, sy, tx, ty;
      shooter_cone(sp, team, u01(u.z), sx, sy, tx, ty);
      float vx = tx - sp.hub_x[team], vy = ty - sp.hub_y[team];
      float d = fmaxf(sqrtf(vx * vx + vy * vy), 1e-6f);
      float tgx = lx + vx / d * d, tgy = ly + vy / d * d;
      launch_piece(s, sp, first, lx, ly, (tgx - lx) * .1f, (tgy - ly) * .1f, 1.83f, 1.f, false);
    }
    w.f_owner[base + first] = -1;
    bool home = in_alliance_zone(sp, team, lx);
    w.f_zone[base + first] = (int8_t)(home ? team + 1 : 0);
    possession[r]--;
    g.rcount(r, RC_PASSED_EVENT) = 1;
    g.rtime(r, RT_NEXT_FERRY) = el + sp.score_interval[r];
  }
  // ---- scoring
  for (int r = 0; r < sp.R; ++r) {
    if (sp.mode[r] == MODE_NONE) continue;
    const float* rp = w.r_pose + g.er(r) * 3;
    const float* rv = w.r_vel + g.er(r) * 3;
    const int team = sp.team[r];
    float err = fabsf(angle_diff(atan2f(sp.hub_y[team] - rp[1], sp.hub_x[team] - rp[0]), rp[2]));
    bool stationary = sqrtf(rv[0] * rv[0] + rv[1] * rv[1]) <= .20f && fabsf(rv[2]) <= .20f;
    bool aimed = sp.kind[r] == 0 ? (err <= kPi / 9.f && stationary) : true;
    bool in_zone = in_alliance_zone(sp, team, rp[0]);
    float rad = robot_radius_of(g.param(r, RP_LENGTH), g.param(r, RP_WIDTH));
    bool ready = in_zone && aimed && clear_of_bumps(sp, rp[0], rp[1], rad);
    bool has_fuel = possession[r] > 0;
    bool hub_on = g.hub_active(team);
    bool entering = ready && !g.latch(r, RL_LAST_HUB_ZONE) && has_fuel && (!hub_on || !in_zone);
    if (entering) {
      g.rcount(r, RC_DENIED_EVENT) = 1;
      g.rcount(r, RC_DENIED_TOTAL) += 1;
    }
    bool can_score = ready && g.latch(r, RL_SCORE_INTENT) && hub_on && in_zone &&
                     el + 1e-6f >= g.rtime(r, RT_NEXT_SCORE);
    g.latch(r, RL_LAST_HUB_ZONE) = ready ? 1 : 0;
    if (!can_score || !has_fuel) continue;
    const int first = next_held[r];
    if (first < 0) continue;
    next_held[r] = fa_next_bit(fw + kFaHeld + r * kFaWords, first + 1, sp.P);
    g.rcount(r, RC_SCORED_EVENT) = 1;
    w.g_scores[(size_t)e * 4 + 2 + team] += 1;
    if (el <= 20.f + sp.dt) w.g_scores[(size_t)e * 4 + team] += 1;
    g.rtime(r, RT_NEXT_SCORE) = el + sp.score_interval[r];
    possession[r]--;
    // scored FUEL re-enters play from the HUB toward midfield
    U4 u = rng.draw((uint32_t)e, tick, RNG_LAUNCH, (uint32_t)(100 + r));
    float sx, sy, tx, ty;
    shooter_cone(sp, team, u01(u.x), sx, sy, tx, ty);
    if (sp.fuel_physics) {
      launch_piece(s, sp, first, sx, sy, (tx - sp.hub_x[team]) * .15f, (ty - sp.hub_y[team]) * .15f, 1.83f,
                   1.f, false);
    } else {
      s.fpos[0][first] = sx;
      s.fpos[1][first] = sy;
      s.fpos[2][first] = sp.fr;
      s.fvel[0][first] = (tx - sp.hub_x[team]) * .1f;
      s.fvel[1][first] = (ty - sp.hub_y[team]) * .1f;
      s.fvel[2][first] = 0.f;
    }
    w.f_owner[base + first] = -1;
    w.f_zone[base + first] = 0;
  }
  for (int r = 0; r < sp.R; ++r) g.rcount(r, RC_ACQUIRED_TOTAL) += g.rcount(r, RC_ACQUIRED_EVENT);
  SERIAL_END
  BARRIER();
  // ---- carried pieces ride with their owner
  PAR_FOR(i, sp.P) {
    int o = w.f_owner[base + i];
    if (w.f_active[base + i] && o >= 0 && o < sp.R) {
      const float* rp = w.r_pose + g.er(o) * 3;
      s.fpos[0][i] = rp[0];
      s.fpos[1][i] = rp[1];
      s.fpos[2][i] = fuel_spawn_height(sp, rp[0], rp[1]);
      for (int k = 0; k < 3; ++k) {
        s.fvel[k][i] = 0.f;
        s.fang[k][i] = 0.f;
      }
      s.sleep[i] = 0;
      s.clock[i] = 0.f;
    }
  }
  BARRIER();
}

// Tracks inside a known chassis footprint (own team, physical) or an observed
// opponent footprint are retired (frc_defense/gamepiece_actions.py:79-125).
AD_HD void invalidate_contact_tracks(G& g) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const float fr = sp.fuel_radius_rules;
  PAR_FOR(i, sp.P) {
    for (int r = 0; r < sp.R; ++r) {
      size_t k = g.erp(r, i);
      if (!w.t_mask[k]) continue;
      float x = g.tx(r, i), y = g.ty(r, i);
      bool hit = false;
      for (int q = 0; q < sp.R && !hit; ++q) {
        if (sp.team[q] != sp.team[r]) continue;
        const float* p = w.r_pose + g.er(q) * 3;
        float dx = x - p[0], dy = y - p[1];
        float c = cosf(p[2]), sn = sinf(p[2]);
        float lon = dx * c + dy * sn, lat = fabsf(-dx * sn + dy * c);
        float L = g.param(q, RP_LENGTH), W = g.param(q, RP_WIDTH);
        hit = lon >= -L * .5f - fr && lon <= L * .5f + .35f + fr && lat <= W * .5f + .075f + fr;
      }
      const size_t er = g.er(r);
      const float* op = w.o_pose + er * 3;
      const float* os = w.o_size + er * 3;
      if (!hit && w.o_valid[er] && os[0] > 0.f && os[1] > 0.f) {
        float dx = x - op[0], dy = y - op[1];
        float c = cosf(op[2]), sn = sinf(op[2]);
        float lon = dx * c + dy * sn, lat = fabsf(-dx * sn + dy * c);
        hit = lon >= -os[0] * .5f - fr && lon <= os[0] * .5f + .35f + fr && lat <= os[1] * .5f + .075f + fr;
      }
      if (hit) {
        w.t_mask[k] = 0;
        w.t_age[k] = kInf;
      }
    }
  }
  BARRIER();
}

// Line of sight from (ox, oy) to (px, py) blocked by a solid box.
AD_HD bool ray_blocked_by_boxes(const SimParams& sp, float ox, float oy, float px, float py) {
  float d[2] = {px - ox, py - oy}, o[2] = {ox, oy};
  for (int b = 0; b < sp.num_boxes; ++b) {
    const Box& bx = sp.boxes[b];
    float lo[2] = {bx.cx - bx.hx, bx.cy - bx.hy}, hi[2] = {bx.cx + bx.hx, bx.cy + bx.hy};
    float enter = 0.f, leave = 1.f;
    bool ok = true;
    for (int a = 0; a < 2; ++a) {
      if (fabsf(d[a]) < 1e-9f) {
        if (o[a] < lo[a] || o[a] > hi[a]) ok = false;
      } else {
        float t0 = (lo[a] - o[a]) / d[a], t1 = (hi[a] - o[a]) / d[a];
        enter = fmaxf(enter, fminf(t0, t1));
        leave = fminf(leave, fmaxf(t0, t1));
      }
    }
    if (ok && enter <= leave && leave > 0.f && enter < 1.f) return true;
  }
  return false;
}

// Simulated stereo perception of free FUEL and of the nearest opponent,
// plus track prediction/aging (frc_defense/_tensor_3v3_observation.py:117-707).
// Each robot carries a forward and a rearward stereo pair with a
// `perception_fov` half field of view; detections are per piece, with range,
// field-structure and chassis occlusion, quality-dependent dropout and
// range-dependent position noise from the counter-based generator.
AD_HD void perception_update(G& g, TickShared& s, const Rng& rng, uint32_t tick, bool sensor_tick) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const int e = g.e;
  const size_t base = (size_t)e * sp.P;
  PAR_FOR(i, sp.P) {
    for (int r = 0; r < sp.R; ++r) {
      size_t k = g.erp(r, i);
      if (w.t_mask[k]) {
        w.t_age[k] += sp.dt;
        g.txr(r, i) += g.tvx(r, i) * sp.dt;
        g.tyr(r, i) += g.tvy(r, i) * sp.dt;
      }
    }
    if (sensor_tick && !sp.stereo_tracks) {  // stereo-cluster tracks: sense_row()
      bool free_piece = w.f_active[base + i] && w.f_owner[base + i] < 0;
      float px = s.fpos[0][i], py = s.fpos[1][i];
      for (int r = 0; r < sp.R; ++r) {
        if (sp.mode[r] == MODE_NONE || !free_piece) continue;
        const float* rp = w.r_pose + g.er(r) * 3;
        float dx = px - rp[0], dy = py - rp[1];
        float dist = sqrtf(dx * dx + dy * dy);
        if (dist > sp.perception_range) continue;
        float err = fabsf(angle_diff(atan2f(dy, dx), rp[2]));
        if (!(err <= sp.perception_fov || err >= kPi - sp.perception_fov)) continue;
        if (ray_blocked_by_boxes(sp, rp[0], rp[1], px, py)) continue;
        bool occluded = false;
        float d2 = fmaxf(dx * dx + dy * dy, 1e-8f);
        for (int q = 0; q < sp.R && !occluded; ++q) {
          if (q == r) continue;
          const float* qp = w.r_pose + g.er(q) * 3;
          float f = ((qp[0] - rp[0]) * dx + (qp[1] - rp[1]) * dy) / d2;
          if (!(f > .02f && f < .98f)) continue;
          float fc = clampf(f, 0.f, 1.f);
          float cx = rp[0] + fc * dx - qp[0], cy = rp[1] + fc * dy - qp[1];
          float rad = robot_radius_of(g.param(q, RP_LENGTH), g.param(q, RP_WIDTH));
          occluded = sqrtf(cx * cx + cy * cy) <= rad;
        }
        if (occluded) continue;
        size_t k = g.erp(r, i);
        float width = 2.f * atanf((sp.ball_diameter * .5f) / fmaxf(dist, .05f));
        float inst = clampf(expf(-dist / 8.f) * fminf(width / .012f, 1.f), 0.f, 1.f);
        float quality = .8f * w.t_quality[k] + .2f * inst;
        w.t_quality[k] = quality;
        U4 u = rng.draw((uint32_t)e, tick, RNG_PERCEPTION, (uint32_t)(r * kMaxPieces + i));
        if (!(u01(u.x) < quality * (1.f - sp.perception_dropout))) continue;
        float size_q = clampf(width / .012f, .15f, 1.f);
        float ns = sp.position_noise * (1.f + dist / 8.f) / sqrtf(size_q);
        U4 u2 = rng.draw((uint32_t)e, tick, RNG_PERCEPTION, (uint32_t)(0x80000000u | (r * kMaxPieces + i)));
        float mx = px + normal_from(u.y, u.z) * ns;
        float my = py + normal_from(u.w, u2.x) * ns;
        float nvx = normal_from(u2.y, u2.z) * sp.velocity_noise;
        float nvy = normal_from(u2.w, u.x ^ 0x9E3779B9u) * sp.velocity_noise;
        bool prior = w.t_mask[k] && w.t_age[k] < sp.track_timeout;
        float elapsed = fmaxf(w.t_age[k], sp.dt);
        float evx = prior ? g.tvx(r, i) + .5f * (mx - g.tx(r, i)) / elapsed : 0.f;
        float evy = prior ? g.tvy(r, i) + .5f * (my - g.ty(r, i)) / elapsed : 0.f;
        g.txr(r, i) = mx;
        g.tyr(r, i) = my;
        g.tvx(r, i) = evx + nvx;
        g.tvy(r, i) = evy + nvy;
        w.t_age[k] = 0.f;
        w.t_mask[k] = 1;
        w.t_conf[k] = quality;
      }
    }
    for (int r = 0; r < sp.R; ++r) {
      size_t k = g.erp(r, i);
      if (w.t_mask[k] && w.t_age[k] > sp.track_timeout) w.t_mask[k] = 0;
    }
  }
  // opponent tracks (defence-role and learned robots observe the nearest enemy)
  PAR_FOR(r, sp.R) {
    const size_t er = g.er(r);
    float* op = w.o_pose + er * 3;
    float* ov = w.o_vel + er * 3;
    if (w.o_valid[er]) {
      op[0] += ov[0] * sp.dt;
      op[1] += ov[1] * sp.dt;
      op[2] += ov[2] * sp.dt;
      w.o_age[er] += sp.dt;
    }
    bool observer = sp.mode[r] != MODE_NONE && (sp.role[r] == 1 || sp.mode[r] == MODE_NN);
    if (sensor_tick && observer) {
      const float* rp = w.r_pose + er * 3;
      float best = kInf;
      int best_q = -1;
      for (int q = 0; q < sp.R; ++q) {
        if (sp.team[q] == sp.team[r] || sp.mode[q] == MODE_NONE) continue;
        const float* qp = w.r_pose + g.er(q) * 3;
        float dx = qp[0] - rp[0], dy = qp[1] - rp[1];
        float dist = sqrtf(dx * dx + dy * dy);
        if (dist > sp.perception_range) continue;
        float err = fabsf(angle_diff(atan2f(dy, dx), rp[2]));
        if (!(err <= sp.perception_fov || err >= kPi - sp.perception_fov)) continue;
        if (ray_blocked_by_boxes(sp, rp[0], rp[1], qp[0], qp[1])) continue;
        bool occluded = false;
        float d2 = fmaxf(dx * dx + dy * dy, 1e-8f);
        for (int o = 0; o < sp.R && !occluded; ++o) {
          if (o == r || o == q) continue;
          const float* pp = w.r_pose + g.er(o) * 3;
          float f = ((pp[0] - rp[0]) * dx + (pp[1] - rp[1]) * dy) / d2;
          if (!(f > .02f && f < .98f)) continue;
          float cx = rp[0] + f * dx - pp[0], cy = rp[1] + f * dy - pp[1];
          occluded = sqrtf(cx * cx + cy * cy) <= robot_radius_of(g.param(o, RP_LENGTH), g.param(o, RP_WIDTH));
        }
        if (!occluded && dist < best) {
          best = dist;
          best_q = q;
        }
      }
      U4 u = rng.draw((uint32_t)e, tick, RNG_OPPONENT, (uint32_t)r);
      U4 u2 = rng.draw((uint32_t)e, tick, RNG_OPPONENT, (uint32_t)(r + 64));
      if (best_q >= 0 && u01(u.x) >= sp.perception_dropout) {
        const float* qp = w.r_pose + g.er(best_q) * 3;
        float rs = 1.f + best / 8.f;
        float cx = qp[0] + normal_from(u.y, u.z) * sp.position_noise * rs;
        float cy = qp[1] + normal_from(u.w, u2.x) * sp.position_noise * rs;
        float ch = qp[2] + normal_from(u2.y, u2.z) * fminf(.05f, sp.position_noise);
        bool prior = w.o_valid[er] && w.o_age[er] < 1.f;
        float elapsed = fmaxf(w.o_age[er], sp.dt);
        float vx = prior ? ov[0] + .5f * (cx - op[0]) / elapsed : 0.f;
        float vy = prior ? ov[1] + .5f * (cy - op[1]) / elapsed : 0.f;
        float vw = prior ? ov[2] + .5f * angle_diff(ch, op[2]) / elapsed : 0.f;
        U4 u3 = rng.draw((uint32_t)e, tick, RNG_OPPONENT, (uint32_t)(r + 128));
        op[0] = cx;
        op[1] = cy;
        op[2] = ch;
        ov[0] = vx + normal_from(u3.x, u3.y) * sp.velocity_noise;
        ov[1] = vy + normal_from(u3.z, u3.w) * sp.velocity_noise;
        ov[2] = vw + normal_from(u2.w, u.x) * sp.velocity_noise;
        float* os = w.o_size + er * 3;
        os[0] = g.param(best_q, RP_LENGTH);
        os[1] = g.param(best_q, RP_WIDTH);
        os[2] = g.param(best_q, RP_ACCEL) / 10.f;
        w.o_age[er] = 0.f;
        w.o_valid[er] = 1;
      }
    }
    if (w.o_valid[er] && w.o_age[er] > 1.f) w.o_valid[er] = 0;
  }
  BARRIER();
}

// ---------------------------------------------------------------------------
// 137-feature observation for robot r (frc_defense/_tensor_3v3_observation.py:775-896).
// ---------------------------------------------------------------------------
AD_HD void observe_robot(G& g, int r, const int32_t* possession) {
  World& w = g.w;
  const SimParams& sp = g.sp;
  const size_t er = g.er(r);
  float* o = w.obs + er * kObsDim;
  const float* p = g.ppose(r);
  const float* v = g.rvel(r);
  const int team = sp.team[r];
  const float speed = g.param(r, RP_SPEED), omega = g.param(r, RP_OMEGA);
  const float spd = fmaxf(speed, .1f);
  const float FL = sp.field_length, FW = sp.field_width;
  int n = 0;
  // base 35: own pose/vel, opponent track, validity/age, hub radius, field, sizes, features
  o[n++] = p[0]; o[n++] = p[1]; o[n++] = p[2];
  o[n++] = v[0]; o[n++] = v[1]; o[n++] = v[2];
  const float* op = w.o_pose + er * 3;
  const float* ov = w.o_vel + er * 3;
  const float* os = w.o_size + er * 3;
  o[n++] = op[0]; o[n++] = op[1]; o[n++] = op[2];
  o[n++] = ov[0]; o[n++] = ov[1]; o[n++] = ov[2];
  o[n++] = w.o_valid[er] ? 1.f : 0.f;
  o[n++] = clampf(w.o_age[er], 0.f, 1.f);
  o[n++] = .595f;
  o[n++] = FL; o[n++] = FW;
  o[n++] = g.param(r, RP_LENGTH); o[n++] = g.param(r, RP_WIDTH); o[n++] = g.param(r, RP_ACCEL) / 10.f;
  o[n++] = os[0]; o[n++] = os[1]; o[n++] = os[2];
  // four nearest field features (x, y, signed radius): solids then bumps
  {
    float fd[4] = {kInf, kInf, kInf, kInf};
    float fv[12] = {0};
    for (int set = 0; set < 2; ++set) {
      int count = set == 0 ? sp.num_boxes : sp.num_bumps;
      for (int b = 0; b < count; ++b) {
        const Box& bx = set == 0 ? sp.boxes[b] : sp.bumps[b];
        float rad = sqrtf(bx.hx * bx.hx + bx.hy * bx.hy) * (set == 0 ? 1.f : -1.f);
        float d = sqr(bx.cx - p[0]) + sqr(bx.cy - p[1]);
        int k = 4;
        while (k > 0 && d < fd[k - 1]) --k;
        if (k < 4) {
          for (int m = 3; m > k; --m) {
            fd[m] = fd[m - 1];
            fv[m * 3] = fv[(m - 1) * 3];
            fv[m * 3 + 1] = fv[(m - 1) * 3 + 1];
            fv[m * 3 + 2] = fv[(m - 1) * 3 + 2];
          }
          fd[k] = d;
          fv[k * 3] = bx.cx;
          fv[k * 3 + 1] = bx.cy;
          fv[k * 3 + 2] = rad;
        }
      }
    }
    for (int k = 0; k < 12; ++k) o[n++] = fv[k];
  }
  // route (3)
  {
    const float* path = w.p_path + er * kPathPoints * 2;
    int len = w.p_len[er];
    if (len > 1) {
      float cost = 0.f;
      for (int k = 0; k < len - 1 && k < kPathPoints - 1; ++k)
        cost += sqrtf(sqr(path[(k + 1) * 2] - path[k * 2]) + sqr(path[(k + 1) * 2 + 1] - path[k * 2 + 1]));
      o[n++] = (path[2] - p[0]) / FL;
      o[n++] = (path[3] - p[1]) / FW;
      o[n++] = cost / sqrtf(FL * FL + FW * FW);
    } else {
      o[n++] = 0.f; o[n++] = 0.f; o[n++] = 0.f;
    }
  }
  // local FUEL tracks (4 x 5): nearest tracked pieces by plain distance
  Top4 top;
  top.init();
  for (int i = 0; i < sp.P; ++i) {
    size_t k = g.erp(r, i);
    if (!w.t_mask[k]) continue;
    top.push(sqrtf(sqr(g.tx(r, i) - p[0]) + sqr(g.ty(r, i) - p[1])), i);
  }
  float cpx[4], cpy[4];
  bool cv[4];
  for (int k = 0; k < 4; ++k) {
    cv[k] = top.c[k] < kInf;
    int i = top.i[k];
    cpx[k] = g.tx(r, i);
    cpy[k] = g.ty(r, i);
    o[n++] = (cpx[k] - p[0]) / FL;
    o[n++] = (cpy[k] - p[1]) / FW;
    o[n++] = g.tvx(r, i) / spd;
    o[n++] = g.tvy(r, i) / spd;
    o[n++] = cv[k] ? 1.f : 0.f;
  }
  // two nearest teammates (2 x 10)
  {
    int t0 = -1, t1 = -1;
    float d0 = kInf, d1 = kInf;
    for (int q = 0; q < sp.R; ++q) {
      if (q == r || sp.team[q] != team) continue;
      const float* qp = g.ppose(q);
      float d = sqrtf(sqr(qp[0] - p[0]) + sqr(qp[1] - p[1]));
      if (d < d0) {
        d1 = d0; t1 = t0; d0 = d; t0 = q;
      } else if (d < d1) {
        d1 = d; t1 = q;
      }
    }
    int ids[2] = {t0, t1};
    for (int k = 0; k < 2; ++k) {
      int q = ids[k];
      if (q < 0) {
        for (int m = 0; m < 8; ++m) o[n++] = 0.f;
        o[n++] = 1.f; o[n++] = 1.f;
        continue;
      }
      const float* qp = g.ppose(q);
      const float* qv = g.rvel(q);
      o[n++] = (qp[0] - p[0]) / FL;
      o[n++] = (qp[1] - p[1]) / FW;
      o[n++] = qv[0] / spd;
      o[n++] = qv[1] / spd;
      o[n++] = sinf(qp[2]);
      o[n++] = cosf(qp[2]);
      int cap = 1;
      for (int m = 0; m < sp.R; ++m) cap = sp.capacity[m] > cap ? sp.capacity[m] : cap;
      o[n++] = sp.teammate_coordination ? (float)possession[q] / (float)cap : 0.f;
      o[n++] = sp.teammate_coordination ? (sp.mode[q] == MODE_NN ? 1.f : 0.f) : 0.f;
      o[n++] = 1.f; o[n++] = 1.f;
    }
  }
  // possession (2)
  int cap = 1;
  for (int m = 0; m < sp.R; ++m) cap = sp.capacity[m] > cap ? sp.capacity[m] : cap;
  float own = (float)possession[r] / (float)cap;
  {
    float mates = 0.f;
    for (int q = 0; q < sp.R; ++q)
      if (q != r && sp.team[q] == team) mates += (float)possession[q];
    o[n++] = own;
    o[n++] = sp.teammate_coordination ? mates / (2.f * cap) : 0.f;
  }
  // match (9)
  o[n++] = g.elapsed() / 160.f;
  o[n++] = w.g_hub[(size_t)g.e * 2] ? 1.f : 0.f;
  o[n++] = w.g_hub[(size_t)g.e * 2 + 1] ? 1.f : 0.f;
  o[n++] = (float)w.g_scores[(size_t)g.e * 4 + 2] / (float)sp.P;
  o[n++] = (float)w.g_scores[(size_t)g.e * 4 + 3] / (float)sp.P;
  for (int t = 0; t < 2; ++t) {
    o[n++] = (sp.hub_x[t] - p[0]) / FL;
    o[n++] = (sp.hub_y[t] - p[1]) / FW;
  }
  // candidates (4 x 10)
  for (int k = 0; k < 4; ++k) {
    float own_eta = cv[k] ? top.c[k] / spd : 0.f;
    float enemy_eta = sqrtf(sqr(cpx[k] - op[0]) + sqr(cpy[k] - op[1])) / spd;
    float to_score = sqrtf(sqr(cpx[k] - sp.hub_x[team]) + sqr(cpy[k] - sp.hub_y[team])) / spd;
    float zone = floorf(clampf(cpx[k] / FL * 6.f, 0.f, 5.f)) / 6.f;
    zone = fminf(fmaxf(floorf(cpx[k] / FL * 6.f), 0.f), 5.f) / 6.f;
    float risk = cv[k] ? 1.f / (1.f + expf(-(own_eta - enemy_eta) * 2.f)) : 0.f;
    o[n++] = (cpx[k] - p[0]) / FL;
    o[n++] = (cpy[k] - p[1]) / FW;
    o[n++] = own_eta / 20.f;
    o[n++] = enemy_eta / 20.f;
    o[n++] = to_score / 20.f;
    o[n++] = risk;
    o[n++] = zone;
    o[n++] = own;
    o[n++] = 1.f - own;
    o[n++] = cv[k] ? 1.f : 0.f;
  }
  // action mask (8)
  bool mask[8];
  for (int k = 0; k < 4; ++k) mask[k] = cv[k] && possession[r] < sp.capacity[r];
  mask[4] = possession[r] > 0;
  mask[5] = w.o_valid[er] || sp.role[r] == 1;
  mask[6] = mask[7] = true;
  for (int k = 0; k < 8; ++k) o[n++] = mask[k] ? 1.f : 0.f;
  // fixed physical scaling of the first 35 features (frc_defense/observation.py:24-46)
  if (sp.normalize_obs) {
    o[0] /= FL; o[1] /= FW; o[2] /= kPi;
    o[3] /= fmaxf(speed, .1f); o[4] /= fmaxf(speed, .1f); o[5] /= fmaxf(omega, .1f);
    o[6] /= FL; o[7] /= FW; o[8] /= kPi;
    o[9] /= fmaxf(speed, .1f); o[10] /= fmaxf(speed, .1f); o[11] /= fmaxf(omega, .1f);
    o[12] /= FL; o[13] /= FW; o[14] /= fmaxf(FL, FW);
    o[15] /= 16.54f; o[16] /= 8.07f;
    const int cols[4] = {23, 26, 29, 32};
    for (int k = 0; k < 4; ++k) {
      o[cols[k]] /= FL;
      o[cols[k] + 1] /= FW;
    }
  }
}

}  // namespace ad
