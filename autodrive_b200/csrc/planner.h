// Grid route planner for one (environment, robot) row.
//
// Reference behaviour (frc_defense/tensor_adstar.py:1108-1468): footprint-
// inflated occupancy at the measured chassis heading, teammate/opponent
// chassis inflation, blocked start/goal projection to a nearby free cell,
// 8-connected cost-to-go by Bellman value iteration with corner cutting blocked
// and a bump traversal penalty, greedy descent extraction (<= 72 points),
// PathPlanner line-of-sight simplification with cubic Bezier corner smoothing
// (tensor_adstar.py:772-1037; handles shortened until the curve stays on free
// cells), equal-arc resampling to 72 points and a curvature/braking speed
// profile.
//
// On the GPU one CTA owns one route with the whole grid (occupancy + one value
// buffer: 5 bytes per cell, 67 KB for the 0.1 m grid of 166 x 81 cells) in
// shared memory; directional Bellman line sweeps run until a sweep changes no
// cell (block-wide vote) or the sweep budget is spent.
#pragma once

#include "game.h"

namespace ad {

// Opt-in per-phase cycle accounting of a plan (sim_bench --phases): thread 0
// adds the clock64() time since the previous mark to bucket k; the marks sit
// after CTA barriers (or inside the final serial section, which thread 0 runs).
constexpr int kPlanPhases = 8;
#if defined(__CUDA_ARCH__)
#define PLAN_MARK(ps, k)                                           \
  do {                                                             \
    if ((ps).prof && threadIdx.x == 0) {                           \
      const unsigned long long t_ = clock64();                     \
      (ps).prof[(k)] += t_ - (ps).prof[kPlanPhases];               \
      (ps).prof[kPlanPhases] = t_;                                 \
    }                                                              \
  } while (0)
#else
#define PLAN_MARK(ps, k) ((void)0)
#endif

struct PlanScratch {
  uint8_t* blocked;   // [nx*ny]
  uint16_t* moves;    // [nx*ny]: per cell, bit k = move k allowed (k < 8), bit 8 = on a bump, bit 9 = blocked
  float* value;       // [nx*ny]
  float* path;        // [plan_lattice_cap * 2]: lattice route of the greedy descent
  float* tmp;         // [4 + plan_lattice_cap * 2]: resolved goal, then the simplified corners
  int* misc;          // [8]
  unsigned long long* best;  // [2] packed endpoint-projection minima
  unsigned long long* prof;  // [kPlanPhases + 1] cycle buckets and the last mark, or null
};

// Lattice points the descent may walk: four times the grid's half perimeter
// (a shortest 8-connected route is far shorter), at least kPathPoints.
AD_HD int plan_lattice_cap(const SimParams& sp) {
  const int c = 4 * (sp.plan_nx + sp.plan_ny);
  return c > kPathPoints ? c : kPathPoints;
}

AD_HD int cell_index(const SimParams& sp, int ix, int iy) { return ix * sp.plan_ny + iy; }
AD_HD float cell_x(const SimParams& sp, int ix) { return ((float)ix + .5f) * sp.plan_res; }
AD_HD float cell_y(const SimParams& sp, int iy) { return ((float)iy + .5f) * sp.plan_res; }

AD_HD bool cell_on_bump(const SimParams& sp, float x, float y) {
  for (int b = 0; b < sp.num_bumps; ++b) {
    const Box& bx = sp.bumps[b];
    if (fabsf(x - bx.cx) <= bx.hx && fabsf(y - bx.cy) <= bx.hy) return true;
  }
  return false;
}

// Segment sampled at half-cell spacing crosses no blocked cell.
AD_HD bool grid_line_clear(const SimParams& sp, const uint8_t* blocked, float x0, float y0, float x1, float y1) {
  float dx = x1 - x0, dy = y1 - y0;
  int steps = (int)ceilf(fmaxf(fabsf(dx), fabsf(dy)) / (sp.plan_res * .5f));
  steps = steps < 1 ? 1 : steps;
  for (int k = 1; k <= steps; ++k) {
    float f = (float)k / (float)steps;
    int ix = clampi((int)floorf((x0 + dx * f) / sp.plan_res), 0, sp.plan_nx - 1);
    int iy = clampi((int)floorf((y0 + dy * f) / sp.plan_res), 0, sp.plan_ny - 1);
    if (blocked[cell_index(sp, ix, iy)]) return false;
  }
  return true;
}


AD_HD bool grid_point_blocked(const SimParams& sp, const uint8_t* blocked, float x, float y) {
  const int ix = clampi((int)floorf(x / sp.plan_res), 0, sp.plan_nx - 1);
  const int iy = clampi((int)floorf(y / sp.plan_res), 0, sp.plan_ny - 1);
  return blocked[cell_index(sp, ix, iy)] != 0;
}

// Resample the n-point chain pt(0..n-1) to kPathPoints points evenly spaced by
// arc length (the segment after a station on ties); returns whether every
// resampled point lies on a free cell.
template <typename PointFn>
AD_HD bool resample_route(const SimParams& sp, const uint8_t* blocked, int n, PointFn pt, float* out) {
  float total = 0.f, ax, ay, bx, by;
  pt(0, ax, ay);
  for (int k = 1; k < n; ++k) {
    pt(k, bx, by);
    total += sqrtf(sqr(bx - ax) + sqr(by - ay));
    ax = bx;
    ay = by;
  }
  pt(0, ax, ay);
  int k = n > 1 ? 1 : 0;
  pt(k, bx, by);
  float sa = 0.f, sb = sqrtf(sqr(bx - ax) + sqr(by - ay));
  bool clear = true;
  for (int q = 0; q < kPathPoints; ++q) {
    const float target = total * (float)q / (float)(kPathPoints - 1);
    while (k < n - 1 && sb <= target) {
      ax = bx;
      ay = by;
      sa = sb;
      pt(++k, bx, by);
      sb += sqrtf(sqr(bx - ax) + sqr(by - ay));
    }
    const float f = clampf((target - sa) / fmaxf(sb - sa, 1e-8f), 0.f, 1.f);
    out[q * 2] = ax + (bx - ax) * f;
    out[q * 2 + 1] = ay + (by - ay) * f;
    clear = clear && !grid_point_blocked(sp, blocked, out[q * 2], out[q * 2 + 1]);
  }
  return clear;
}

// PathPlanner-style corner poses of the simplified polyline s[0..m-1]: the
// start, for every corner an incoming pose 80 % along the incoming leg and an
// outgoing pose 20 % along the outgoing leg (each with its leg's heading),
// and the end; 2m - 2 poses. (ux, uy) is the unit heading (+x for a
// zero-length leg).
AD_HD void corner_pose(const float* s, int m, int k, float& x, float& y, float& ux, float& uy) {
  const int count = 2 * m - 2;
  int a, b;
  float f;
  if (k == 0) {
    a = 0, b = 1, f = 0.f;
  } else if (k >= count - 1) {
    a = m - 2, b = m - 1, f = 1.f;
  } else {
    const int c = (k + 1) / 2;
    if (k & 1) a = c - 1, b = c, f = .8f;
    else a = c, b = c + 1, f = .2f;
  }
  const float dx = s[b * 2] - s[a * 2], dy = s[b * 2 + 1] - s[a * 2 + 1];
  x = s[a * 2] + f * dx;
  y = s[a * 2 + 1] + f * dy;
  const float n = sqrtf(dx * dx + dy * dy);
  ux = n > 0.f ? dx / n : 1.f;
  uy = n > 0.f ? dy / n : 0.f;
}

// Point idx of the sampled cubic Bezier chain through the corner poses (pose
// 0, then 8 samples per segment, t = 1/8 .. 1), handles `factor` x segment
// length along the pose headings.
AD_HD void bezier_chain_point(const float* s, int m, float factor, int idx, float& x, float& y) {
  float x0, y0, ux0, uy0, x3, y3, ux3, uy3;
  if (idx == 0) {
    corner_pose(s, m, 0, x, y, ux0, uy0);
    return;
  }
  const int seg = (idx - 1) / 8, j = (idx - 1) % 8 + 1;
  corner_pose(s, m, seg, x0, y0, ux0, uy0);
  corner_pose(s, m, seg + 1, x3, y3, ux3, uy3);
  const float d = sqrtf(sqr(x3 - x0) + sqr(y3 - y0)) * factor;
  const float x1 = x0 + ux0 * d, y1 = y0 + uy0 * d;
  const float x2 = x3 - ux3 * d, y2 = y3 - uy3 * d;
  const float t = (float)j / 8.f, u = 1.f - t;
  const float w0 = u * u * u, w1 = 3.f * u * u * t, w2 = 3.f * u * t * t, w3 = t * t * t;
  x = w0 * x0 + w1 * x1 + w2 * x2 + w3 * x3;
  y = w0 * y0 + w1 * y1 + w2 * y2 + w3 * y3;
}

struct PlanRequest {
  float sx, sy, gx, gy, heading, length, width, speed, lat_mu, accel;
  // perceived robot obstacles (x, y, radius), radius <= 0 disables a slot
  float obst[kMaxRobots * 3];
  int num_obst;
};

// Plan one route. Writes the persistent route state of row (e, r).
AD_HD void plan_route(World& w, const SimParams& sp, int e, int r, const PlanRequest& q, PlanScratch& ps) {
  const int nx = sp.plan_nx, ny = sp.plan_ny, nc = nx * ny;
  const size_t er = (size_t)e * sp.R + r;
  // trench alignment hint: crossing a trench x-line from inside a clear opening
  bool trench = false;
  float heading = q.heading;
  {
    float lane_low = 0.f, lane_high = sp.field_width;
    bool have = false;
    float trench_x[2];
    int tcount = 0;
    // trench supports are the solid boxes whose y is not the field centre
    for (int b = 0; b < sp.num_boxes; ++b) {
      const Box& bx = sp.boxes[b];
      bool support = fabsf(bx.cy - sp.field_width * .5f) > 1.5f && bx.hy < .3f && bx.hx > .5f;
      if (!support) continue;
      if (bx.cy < sp.field_width * .5f) lane_low = fmaxf(lane_low, bx.cy - bx.hy);
      else lane_high = have ? fminf(lane_high, bx.cy + bx.hy) : bx.cy + bx.hy;
      have = true;
      bool seen = false;
      for (int k = 0; k < tcount; ++k) seen = seen || fabsf(trench_x[k] - bx.cx) < 1e-3f;
      if (!seen && tcount < 2) trench_x[tcount++] = bx.cx;
    }
    if (have) {
      float lo = fminf(q.sx, q.gx), hi = fmaxf(q.sx, q.gx);
      bool crosses = false;
      for (int k = 0; k < tcount; ++k) crosses = crosses || (trench_x[k] >= lo && trench_x[k] <= hi);
      float hw = q.width * .5f;
      bool opening = (q.sy >= hw && q.sy <= lane_low - hw) || (q.sy >= lane_high + hw && q.sy <= sp.field_width - hw);
      trench = crosses && opening;
      if (trench) heading = q.gx >= q.sx ? 0.f : kPi;
    }
  }
  // occupancy at the measured heading
  const float ch = cosf(q.heading), sh = sinf(q.heading);
  const float ac = fabsf(ch), as = fabsf(sh);
  const float ex = (q.length * ac + q.width * as) * .5f, ey = (q.length * as + q.width * ac) * .5f;
  const float mover = .5f * fminf(q.length, q.width);
  PAR_FOR(c, nc) {
    int ix = c / ny, iy = c % ny;
    float x = cell_x(sp, ix), y = cell_y(sp, iy);
    bool b = x < ex || x > sp.field_length - ex || y < ey || y > sp.field_width - ey;
    for (int k = 0; k < q.num_obst && !b; ++k) {
      float rr = q.obst[k * 3 + 2];
      if (!(rr > 0.f)) continue;
      float cl = mover + rr;
      b = sqr(x - q.obst[k * 3]) + sqr(y - q.obst[k * 3 + 1]) <= cl * cl;
    }
    ps.blocked[c] = b ? 1 : 0;
  }
  BARRIER();
  // solid boxes: each box tests only the cells of its inflated bounding
  // rectangle (one cell of margin; the exact per-cell test decides) and
  // marks the ones its rotated footprint covers, instead of every cell
  // testing every box
  for (int k = 0; k < sp.num_boxes; ++k) {
    const Box& bx = sp.boxes[k];
    const float sf = q.length * .5f + bx.hx * ac + bx.hy * as;
    const float sl = q.width * .5f + bx.hx * as + bx.hy * ac;
    const int ix0 = clampi((int)floorf((bx.cx - bx.hx - ex) / sp.plan_res) - 1, 0, nx - 1);
    const int ix1 = clampi((int)floorf((bx.cx + bx.hx + ex) / sp.plan_res) + 1, 0, nx - 1);
    const int iy0 = clampi((int)floorf((bx.cy - bx.hy - ey) / sp.plan_res) - 1, 0, ny - 1);
    const int iy1 = clampi((int)floorf((bx.cy + bx.hy + ey) / sp.plan_res) + 1, 0, ny - 1);
    const int span = iy1 - iy0 + 1;
    PAR_FOR(u, (ix1 - ix0 + 1) * span) {
      const int ix = ix0 + u / span, iy = iy0 + u % span;
      const float dx = cell_x(sp, ix) - bx.cx, dy = cell_y(sp, iy) - bx.cy;
      if (fabsf(dx) > bx.hx + ex || fabsf(dy) > bx.hy + ey) continue;
      const float fwd = dx * ch + dy * sh, lat = -dx * sh + dy * ch;
      if (fabsf(fwd) <= sf && fabsf(lat) <= sl) ps.blocked[cell_index(sp, ix, iy)] = 1;
    }
  }
  BARRIER();
  PLAN_MARK(ps, 0);   // occupancy grid
  // project blocked endpoints to the nearest free cell: a block-wide minimum
  // of packed (squared distance, cell index) keys, i.e. the nearest free cell
  // with ties to the lower index (the serial scan's choice)
  float pts[4] = {q.sx, q.sy, q.gx, q.gy};
  bool need[2];
  for (int k = 0; k < 2; ++k) {
    const int ix = clampi((int)floorf(pts[k * 2] / sp.plan_res), 0, nx - 1);
    const int iy = clampi((int)floorf(pts[k * 2 + 1] / sp.plan_res), 0, ny - 1);
    need[k] = ps.blocked[cell_index(sp, ix, iy)] != 0;
  }
  SERIAL_BEGIN
  ps.best[0] = ps.best[1] = ~0ull;
  SERIAL_END
  BARRIER();
  if (need[0] || need[1]) {
    PAR_FOR(c, nc) {
      if (ps.blocked[c]) continue;
      const float cx = cell_x(sp, c / ny), cy = cell_y(sp, c % ny);
      for (int k = 0; k < 2; ++k) {
        if (!need[k]) continue;
        const float d = sqr(cx - pts[k * 2]) + sqr(cy - pts[k * 2 + 1]);
        const unsigned long long key = ((unsigned long long)float_bits(d) << 32) | (unsigned)c;
#if defined(__CUDA_ARCH__)
        atomicMin(&ps.best[k], key);
#else
        if (key < ps.best[k]) ps.best[k] = key;
#endif
      }
    }
  }
  BARRIER();
  SERIAL_BEGIN
  for (int k = 0; k < 2; ++k) {
    if (!need[k] || ps.best[k] == ~0ull) continue;
    const int bc = (int)(ps.best[k] & 0xffffffffull);
    pts[k * 2] = cell_x(sp, bc / ny);
    pts[k * 2 + 1] = cell_y(sp, bc % ny);
  }
  ps.misc[0] = clampi((int)floorf(pts[0] / sp.plan_res), 0, nx - 1);
  ps.misc[1] = clampi((int)floorf(pts[1] / sp.plan_res), 0, ny - 1);
  ps.misc[2] = clampi((int)floorf(pts[2] / sp.plan_res), 0, nx - 1);
  ps.misc[3] = clampi((int)floorf(pts[3] / sp.plan_res), 0, ny - 1);
  ps.blocked[cell_index(sp, ps.misc[0], ps.misc[1])] = 0;
  ps.blocked[cell_index(sp, ps.misc[2], ps.misc[3])] = 0;
  ps.path[0] = pts[0];
  ps.path[1] = pts[1];
  ps.tmp[0] = pts[2];
  ps.tmp[1] = pts[3];
  SERIAL_END
  BARRIER();
  PLAN_MARK(ps, 1);   // endpoint projection
  const int gcell = cell_index(sp, ps.misc[2], ps.misc[3]);
  const int dxs[8] = {1, -1, 0, 0, 1, 1, -1, -1};
  const int dys[8] = {0, 0, 1, -1, 1, -1, 1, -1};
  // per-cell move table, built once per plan for the sweeps: a move is
  // allowed into an in-bounds free cell, diagonally only when both corner
  // cells are free; a blocked target would never lower a value (it keeps
  // 1e6 while every value starts at 1e6 and only decreases), so leaving it
  // out changes nothing
  PAR_FOR(c, nc) {
    ps.value[c] = c == gcell ? 0.f : 1.e6f;
    const int ix = c / ny, iy = c % ny;
    // the 3 x 3 neighbourhood's free flags, read once (outside the grid: not free)
    bool fr[3][3];
    for (int a = 0; a < 3; ++a)
      for (int b = 0; b < 3; ++b) {
        const int jx = ix + a - 1, jy = iy + b - 1;
        fr[a][b] = jx >= 0 && jx < nx && jy >= 0 && jy < ny && !ps.blocked[cell_index(sp, jx, jy)];
      }
    unsigned m = fr[1][1] ? 0u : 512u;
    for (int k = 0; k < 8; ++k) {
      const int a = dxs[k] + 1, b = dys[k] + 1;
      if (!fr[a][b]) continue;
      if (k >= 4 && (!fr[a][1] || !fr[1][b])) continue;
      m |= 1u << k;
    }
    if (cell_on_bump(sp, cell_x(sp, ix), cell_y(sp, iy))) m |= 256u;
    ps.moves[c] = (uint16_t)m;
  }
  BARRIER();
  PLAN_MARK(ps, 2);   // move table, value initialisation
  // Bellman value iteration by directional line sweeps (the fast sweeping
  // method, Zhao, Math. Comp. 2005): a line sweep walks one grid line and
  // updates its cells in place, so a value crosses a whole line in one sweep
  // instead of one cell per Jacobi sweep. Pass k runs, at the same time, every
  // row (x line, nx cells) in direction +x (k even) or -x (k odd) and every
  // column (y line, ny cells) in direction +y and then -y: the rows are about
  // twice as long as the columns, so the two thread groups finish together.
  // Values only decrease (on the GPU a cell updated by its row and its column
  // takes the smaller value through an atomic minimum) and each is the cost of
  // an actual path, so the iteration stops at the unique fixed point
  // v(c) = min_k v(n_k) + w_k (the Jacobi solution) once a pass changes no
  // cell, in any update order: the GPU (racing reads of neighbouring lines)
  // and the serial host twin return the same values.
  volatile float* vv = ps.value;
  int offs[8];   // cell index step of move k
  for (int k = 0; k < 8; ++k) offs[k] = dxs[k] * ny + dys[k];
  auto sweep_line = [&](bool along_x, int line, bool reverse) -> int {
    const int len = along_x ? nx : ny;
    // the neighbour just behind in sweep order was updated by this thread in
    // the previous step: its value comes from a register (a smaller value
    // written there meanwhile by the crossing line only delays convergence)
    const int behind = along_x ? (reverse ? 0 : 1) : (reverse ? 2 : 3);
    int changed = 0;
    float prev = 1.e6f;
    for (int step = 0; step < len; ++step) {
      const int t = reverse ? len - 1 - step : step;
      const int ix = along_x ? t : line, iy = along_x ? line : t;
      const int c = cell_index(sp, ix, iy);
      const unsigned m = ps.moves[c];
      if (m & 512u) {   // blocked: never updated, holds 1e6
        prev = 1.e6f;
        continue;
      }
      const float bc = (m & 256u) ? 1.f + sp.bump_cost : 1.f;
      const float wd = mul_rn(1.41421356237f, bc);
      const float cur = vv[c];
      // all eight candidates without branches: a move that is not allowed
      // reads the cell itself and contributes +inf, so every load can issue
      // at once; the minimum is the same as over the allowed moves alone
      float cand[8];
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
      for (int k = 0; k < 8; ++k) {
        const bool ok = (m >> k) & 1u;
        const float v = vv[ok ? c + offs[k] : c];
        cand[k] = ok ? (k == behind ? prev : v) + (k >= 4 ? wd : bc) : kInf;
      }
      float best = cur;
#if defined(__CUDA_ARCH__)
#pragma unroll
#endif
      for (int k = 0; k < 8; ++k) best = fminf(best, cand[k]);
      if (best < cur) {
#if defined(__CUDA_ARCH__)
        atomicMin(reinterpret_cast<int*>(ps.value) + c, __float_as_int(best));   // values are >= 0
#else
        ps.value[c] = best;
#endif
        changed = 1;
      }
      prev = best;
    }
    return changed;
  };
  int sweeps_run = 0;
  bool converged = false;
  for (int sweep = 0; sweep < sp.plan_sweeps; ++sweep) {
    const bool reverse = (sweep & 1) != 0;
    int changed = 0;
    PAR_FOR(item, ny + nx) {
      if (item < ny) {
        changed |= sweep_line(true, item, reverse);
      } else {
        changed |= sweep_line(false, item - ny, false);
        changed |= sweep_line(false, item - ny, true);
      }
    }
#if defined(__CUDA_ARCH__)
    const int any = __syncthreads_or(changed);
#else
    const int any = changed;
#endif
    sweeps_run = sweep + 1;
    if (!any) {
      converged = true;
      break;
    }
  }
  PLAN_MARK(ps, 3);   // value iteration sweeps
  SERIAL_BEGIN
  // passes used; negative when the budget ran out before a pass changed nothing
  w.p_sweeps[er] = converged ? sweeps_run : -sweeps_run;
  // greedy descent
  int px = ps.misc[0], py = ps.misc[1];
  const int gx = ps.misc[2], gy = ps.misc[3];
  int len = 1;
  const int cap = plan_lattice_cap(sp);
  for (int k = 1; k < cap; ++k) {
    if (px == gx && py == gy) break;
    float best = 1.e6f;
    int bk = -1;
    for (int m = 0; m < 8; ++m) {
      int jx = px + dxs[m], jy = py + dys[m];
      if (jx < 0 || jx >= nx || jy < 0 || jy >= ny) continue;
      if (m >= 4 && (ps.blocked[cell_index(sp, jx, py)] || ps.blocked[cell_index(sp, px, jy)])) continue;
      if (ps.blocked[cell_index(sp, jx, jy)]) continue;
      float v = ps.value[cell_index(sp, jx, jy)];
      if (v < best) {
        best = v;
        bk = m;
      }
    }
    if (bk < 0 || !(best < ps.value[cell_index(sp, px, py)] - 1e-5f)) break;
    px += dxs[bk];
    py += dys[bk];
    ps.path[len * 2] = cell_x(sp, px);
    ps.path[len * 2 + 1] = cell_y(sp, py);
    len++;
  }
  // snap the final point onto the resolved goal when the goal cell was reached
  if (len > 1 && px == gx && py == gy) {
    ps.path[(len - 1) * 2] = ps.tmp[0];
    ps.path[(len - 1) * 2 + 1] = ps.tmp[1];
  }
  ps.misc[6] = len;
  SERIAL_END
  BARRIER();
  PLAN_MARK(ps, 4);   // greedy descent
  // line-of-sight simplification (PathPlanner): a lattice point is kept only
  // when the last kept point cannot see the point after it. Round by round:
  // every thread tests the sight line from the current anchor to one later
  // lattice point, the first blocked one (index j) makes point j-1 the next
  // kept point and anchor; the serial rule's result, in as many rounds as
  // there are corners
  float* simp = ps.tmp + 4;  // [plan_lattice_cap * 2]
  const int len = ps.misc[6];
  SERIAL_BEGIN
  simp[0] = ps.path[0];
  simp[1] = ps.path[1];
  ps.misc[5] = 0;   // anchor
  ps.misc[7] = 1;   // kept points
  SERIAL_END
  BARRIER();
  if (len > 1) {
    while (true) {
      const int anchor = ps.misc[5];
      SERIAL_BEGIN
      ps.misc[4] = len;
      SERIAL_END
      BARRIER();
      const float ax = ps.path[anchor * 2], ay = ps.path[anchor * 2 + 1];
      PAR_FOR(j0, len - anchor - 2) {
        const int j = anchor + 2 + j0;
        if (!grid_line_clear(sp, ps.blocked, ax, ay, ps.path[j * 2], ps.path[j * 2 + 1])) {
#if defined(__CUDA_ARCH__)
          atomicMin(&ps.misc[4], j);
#else
          if (j < ps.misc[4]) ps.misc[4] = j;
#endif
        }
      }
      BARRIER();
      const int fail = ps.misc[4];
      BARRIER();
      if (fail >= len) break;
      SERIAL_BEGIN
      const int m = ps.misc[7];
      simp[m * 2] = ps.path[(fail - 1) * 2];
      simp[m * 2 + 1] = ps.path[(fail - 1) * 2 + 1];
      ps.misc[7] = m + 1;
      ps.misc[5] = fail - 1;
      SERIAL_END
      BARRIER();
    }
    SERIAL_BEGIN
    const int m = ps.misc[7];
    simp[m * 2] = ps.path[(len - 1) * 2];
    simp[m * 2 + 1] = ps.path[(len - 1) * 2 + 1];
    ps.misc[7] = m + 1;
    SERIAL_END
    BARRIER();
  }
  PLAN_MARK(ps, 5);   // line-of-sight simplification
  SERIAL_BEGIN
  const int m = ps.misc[7];
  // smoothed route: cubic Bezier corners with the longest handle (0.4, 0.28,
  // 0.18, 0.1, 0 x segment length) whose samples and kPathPoints-point
  // equal-arc resampling stay on free cells; else the simplified polyline,
  // else the lattice route, each resampled the same way
  float* dst = w.p_path + er * kPathPoints * 2;
  if (len > 1) {
    const float* src = ps.path;
    auto lattice = [&](int k, float& x, float& y) { x = src[k * 2]; y = src[k * 2 + 1]; };
    auto polyline = [&](int k, float& x, float& y) { x = simp[k * 2]; y = simp[k * 2 + 1]; };
    bool done = false;
    const float factors[5] = {.4f, .28f, .18f, .1f, 0.f};
    const int samples = 1 + (2 * m - 3) * 8;
    for (int fi = 0; fi < 5 && !done; ++fi) {
      const float factor = factors[fi];
      auto curve = [&](int k, float& x, float& y) { bezier_chain_point(simp, m, factor, k, x, y); };
      bool clear = true;
      for (int k = 0; k < samples && clear; ++k) {
        float x, y;
        curve(k, x, y);
        clear = !grid_point_blocked(sp, ps.blocked, x, y);
      }
      if (clear) done = resample_route(sp, ps.blocked, samples, curve, dst);
    }
    if (!done) done = resample_route(sp, ps.blocked, m, polyline, dst);
    if (!done) resample_route(sp, ps.blocked, len, lattice, dst);
  } else {
    for (int k = 0; k < kPathPoints; ++k) {
      dst[k * 2] = ps.path[0];
      dst[k * 2 + 1] = ps.path[1];
    }
  }
  // a one-cell route from start==goal still counts as a single point
  w.p_len[er] = len > 1 ? kPathPoints : 1;
  PLAN_MARK(ps, 6);   // smoothing and resampling
  // speed profile: curvature caps then backward braking envelope
  float* prof = w.p_profile + er * kPathPoints;
  const float mu = fmaxf(q.lat_mu, .1f), acc = fmaxf(q.accel, .2f), vcap = fmaxf(q.speed, .1f);
  const int L = w.p_len[er];
  float station[kPathPoints];
  station[0] = 0.f;
  for (int k = 0; k < kPathPoints - 1; ++k)
    station[k + 1] = station[k] + sqrtf(sqr(dst[(k + 1) * 2] - dst[k * 2]) + sqr(dst[(k + 1) * 2 + 1] - dst[k * 2 + 1]));
  for (int k = 0; k < kPathPoints; ++k) {
    float cap = vcap;
    if (k > 0 && k < kPathPoints - 1) {
      float ax = dst[k * 2] - dst[(k - 1) * 2], ay = dst[k * 2 + 1] - dst[(k - 1) * 2 + 1];
      float bx = dst[(k + 1) * 2] - dst[k * 2], by = dst[(k + 1) * 2 + 1] - dst[k * 2 + 1];
      float la = sqrtf(ax * ax + ay * ay), lb = sqrtf(bx * bx + by * by);
      float ua = 1.f / fmaxf(la, 1e-6f), ub = 1.f / fmaxf(lb, 1e-6f);
      float crs = ax * ua * by * ub - ay * ua * bx * ub, dt2 = ax * ua * bx * ub + ay * ua * by * ub;
      float turn = fabsf(atan2f(crs, dt2));
      float arc = fmaxf(.5f * (la + lb), 1e-4f);
      float curv = turn / arc;
      if (curv > 1e-6f) cap = fminf(vcap, fminf(sqrtf(mu * kG / curv), sp.steer_rate_limit / curv));
    }
    if (k == L - 1) cap = 0.f;
    prof[k] = cap;
  }
  // backward braking envelope v_k = min over j >= k of sqrt(cap_j^2 + 2 a (s_j - s_k)),
  // as the recursion v_k^2 = min(cap_k^2, v_{k+1}^2 + 2 a (s_{k+1} - s_k))
  for (int k = L; k < kPathPoints; ++k) ps.tmp[k] = kInf;
  float next2 = kInf;
  for (int k = L - 1; k >= 0; --k) {
    float v2 = prof[k] * prof[k];
    if (k < L - 1) v2 = fminf(v2, next2 + 2.f * acc * fmaxf(station[k + 1] - station[k], 0.f));
    next2 = v2;
    ps.tmp[k] = sqrtf(v2);
  }
  for (int k = 0; k < kPathPoints; ++k) prof[k] = ps.tmp[k] < kInf ? ps.tmp[k] : vcap;
  w.p_progress[er] = 0.f;
  w.p_goal[er * 2] = dst[(L - 1) * 2];
  w.p_goal[er * 2 + 1] = dst[(L - 1) * 2 + 1];
  w.p_start[er * 2] = ps.path[0];
  w.p_start[er * 2 + 1] = ps.path[1];
  w.p_heading[er] = heading;
  w.p_trench[er] = trench ? 1 : 0;
  PLAN_MARK(ps, 7);   // speed profile and route state
  SERIAL_END
  BARRIER();
}

// Build the planner request of row (e, r) from the controller state.
AD_HD PlanRequest make_plan_request(World& w, const SimParams& sp, int e, int r) {
  G g{w, sp, e};
  PlanRequest q;
  const float* p = g.ppose(r);
  q.sx = p[0];
  q.sy = p[1];
  q.gx = w.c_target[g.er(r) * 2];
  q.gy = w.c_target[g.er(r) * 2 + 1];
  q.heading = p[2];
  bool extended = sp.kind[r] == 1 || w.g_rlatch[g.er(r) * kLatches + RL_INTAKE_COLLECTING];
  q.length = g.param(r, RP_LENGTH) + (extended ? .6096f : 0.f);
  q.width = g.param(r, RP_WIDTH);
  q.speed = g.param(r, RP_SPEED);
  q.lat_mu = g.param(r, RP_LATERAL_MU);
  q.accel = g.param(r, RP_ACCEL);
  // known teammates (estimated poses) plus the anonymous opponent track
  q.num_obst = 0;
  for (int m = 0; m < sp.R; ++m) {
    if (sp.team[m] != sp.team[r] || m == r) continue;
    const float* mp = g.ppose(m);
    q.obst[q.num_obst * 3] = mp[0];
    q.obst[q.num_obst * 3 + 1] = mp[1];
    q.obst[q.num_obst * 3 + 2] = .5f * fminf(g.param(m, RP_LENGTH), g.param(m, RP_WIDTH));
    q.num_obst++;
  }
  const size_t er = g.er(r);
  const float* os = w.o_size + er * 3;
  if (w.o_valid[er] && os[0] > 0.f && os[1] > 0.f && q.num_obst < kMaxRobots) {
    q.obst[q.num_obst * 3] = w.o_pose[er * 3];
    q.obst[q.num_obst * 3 + 1] = w.o_pose[er * 3 + 1];
    q.obst[q.num_obst * 3 + 2] = .5f * fminf(os[0], os[1]);
    q.num_obst++;
  }
  return q;
}

}  // namespace ad
