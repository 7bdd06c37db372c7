// Robot and FUEL physics for one environment, written once for host and GPU.
//
// Robot model (reference: frc_defense/tensor_physics.py:585-697): four-module
// swerve with 90-degree module optimisation, steering dynamics, a motor model
// with back-EMF, per-controller and robot supply limits, battery sag, a
// per-wheel friction circle, acceleration caps and bump pitch/load transfer.
// Contacts (frc_defense/tensor_physics_collision.py): rectangle SAT between
// robots with rigid impulses and Coulomb friction, field walls, circular
// obstacles and oriented-box vs field-box contacts.
//
// FUEL model (frc_defense/fuel_physics.py:384-587): 3D compliant spheres with a
// backward-Euler spring-damper normal impulse, Coulomb friction including the
// sphere's rotational inertia, rolling resistance, bump terrain, walls, field
// boxes, reciprocal chassis impulses and sleeping. Pair contacts use a Jacobi
// update where each sphere owns the computation of the impulses acting on it,
// so the accumulation needs no atomics and is reproducible run to run.
#pragma once

#include "world.h"

namespace ad {

constexpr int kMaxGridCells = 4096;
constexpr int kRedSlots = 32;       // warps per CTA (max 1024 threads)

// Per-environment working set. On the GPU it lives in dynamic shared memory
// for the whole controller tick; on the host it is a per-thread scratch.
struct TickShared {
  // robots
  float pose[kMaxRobots * 3];
  float vel[kMaxRobots * 3];
  float param[kMaxRobots * kNumRobotParams];
  float ms[kMaxRobots * 20];
  float current[kMaxRobots];
  float cmd[kMaxRobots * 3];
  float mu3[3];
  uint8_t rflag[kMaxRobots * 4];
  uint8_t eflag[2];
  uint8_t pad0[2];
  int32_t safety[kMaxRobots * 4];
  int32_t substep_index;
  double phys_time;
  // pair scratch (Jacobi robot contacts)
  float pq_move[kMaxPairs * 4];
  float pq_dv[kMaxPairs * 6];
  float pq_jn[kMaxPairs], pq_jt[kMaxPairs];
  float pq_n[kMaxPairs * 2];
  uint8_t pq_valid[kMaxPairs];
  uint8_t pad1;
  // fuel
  float fpos[3][kMaxPieces];
  float fvel[3][kMaxPieces];
  float fang[3][kMaxPieces];
  float dv[3][kMaxPieces];
  float dw[3][kMaxPieces];
  float clock[kMaxPieces];
  float support[kMaxPieces];
  uint8_t sleep[kMaxPieces];
  uint8_t freem[kMaxPieces];
  uint8_t degree[kMaxPieces];
  uint8_t pad2[kMaxPieces % 4 == 0 ? 4 : 4 - kMaxPieces % 4];
  int16_t cell[kMaxPieces];
  int16_t slot[kMaxPieces];
  int16_t sorted[kMaxPieces];
  int16_t work[kMaxPieces];                     // spheres that need pair contacts this substep
  uint8_t listed[kMaxPieces];                   // sphere is on `work`
  int32_t nwork;
  uint32_t cmask;                               // robots with a chassis-FUEL contact this substep
  alignas(16) int32_t cell_start[kMaxGridCells + 4];
  alignas(16) uint32_t awake_bits[kMaxGridCells / 32 + 4];  // grid cells holding an awake sphere
  float rtrig[kMaxRobots * 4];                  // per robot: cos, sin, contact reach^2, unused
  alignas(16) float red[kRedSlots * 20];
  float red_out[20];
  float scal[8];
  // phase accounting (PHASE_MARK): [0] thread 0's timeline, [1] the FUEL warps' leader
  unsigned long long prof_last[2];
  unsigned long long prof[18];
  int32_t prof_on;
};

// ----------------------------------------------------------------------------
// CTA reductions. On the GPU each thread passes its partial values; on the
// host the single caller already holds the total.
// ----------------------------------------------------------------------------
template <int M>
AD_HD void cta_sum(TickShared& s, float (&v)[M]) {
#if defined(__CUDA_ARCH__)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int k = 0; k < M; ++k) {
    float x = v[k];
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) s.red[warp * 20 + k] = x;
  }
  __syncthreads();
  if (threadIdx.x < M) {
    float t = 0.f;
    for (int w = 0; w < warps; ++w) t += s.red[w * 20 + threadIdx.x];
    s.red_out[threadIdx.x] = t;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < M; ++k) v[k] = s.red_out[k];
  __syncthreads();
#else
  (void)s;
  (void)v;
#endif
}

// Max over a thread group (warp-aligned); the group barrier replaces __syncthreads.
template <int M>
AD_HD void group_max(TickShared& s, float (&v)[M], const Group& g) {
#if defined(__CUDA_ARCH__)
  const int lane = threadIdx.x & 31, warp = g.rank >> 5;
  const int warps = (g.size + 31) >> 5;
#pragma unroll
  for (int k = 0; k < M; ++k) {
    float x = v[k];
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    if (lane == 0) s.red[warp * 20 + k] = x;
  }
  group_sync(g);
  if (g.rank < M) {
    float t = -kInf;
    for (int w = 0; w < warps; ++w) t = fmaxf(t, s.red[w * 20 + g.rank]);
    s.red_out[g.rank] = t;
  }
  group_sync(g);
#pragma unroll
  for (int k = 0; k < M; ++k) v[k] = s.red_out[k];
  group_sync(g);
#else
  (void)s;
  (void)v;
  (void)g;
#endif
}

// cta_sum restricted to the robots in `mask` (entries 3r..3r+2); the other
// entries are left as they are (the caller's are zero).
AD_HD void cta_sum_robots(TickShared& s, float (&v)[18], uint32_t mask) {
#if defined(__CUDA_ARCH__)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int k = 0; k < 18; ++k) {
    if (!((mask >> (k / 3)) & 1u)) continue;
    float x = v[k];
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) s.red[warp * 20 + k] = x;
  }
  __syncthreads();
  if (threadIdx.x < 18 && ((mask >> (threadIdx.x / 3)) & 1u)) {
    float t = 0.f;
    for (int w = 0; w < warps; ++w) t += s.red[w * 20 + threadIdx.x];
    s.red_out[threadIdx.x] = t;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 18; ++k)
    if ((mask >> (k / 3)) & 1u) v[k] = s.red_out[k];
  __syncthreads();
#else
  (void)s;
  (void)v;
  (void)mask;
#endif
}

template <int M>
AD_HD void cta_max(TickShared& s, float (&v)[M]) {
#if defined(__CUDA_ARCH__)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = (blockDim.x + 31) >> 5;
#pragma unroll
  for (int k = 0; k < M; ++k) {
    float x = v[k];
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    if (lane == 0) s.red[warp * 20 + k] = x;
  }
  __syncthreads();
  if (threadIdx.x < M) {
    float t = -kInf;
    for (int w = 0; w < warps; ++w) t = fmaxf(t, s.red[w * 20 + threadIdx.x]);
    s.red_out[threadIdx.x] = t;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < M; ++k) v[k] = s.red_out[k];
  __syncthreads();
#else
  (void)s;
  (void)v;
#endif
}

// ----------------------------------------------------------------------------
// Robot helpers
// ----------------------------------------------------------------------------
AD_HD float rparam(const TickShared& s, int r, int k) { return s.param[r * kNumRobotParams + k]; }
AD_HD float robot_inertia(const TickShared& s, int r) {
  float L = rparam(s, r, RP_LENGTH), W = rparam(s, r, RP_WIDTH), m = rparam(s, r, RP_MASS);
  return m * (L * L + W * W) / 12.f * rparam(s, r, RP_YAW_INERTIA);
}

// Yaw-rate target with a stopping envelope and rate feedback
// (frc_defense/tensor_physics.py:28-46).
AD_HD float swerve_heading_rate(float error, float omega_limit, float alpha, float current_rate,
                                float control_dt, bool use_rate) {
  if (control_dt > 0.f) omega_limit = fminf(omega_limit, .6f / fmaxf(control_dt, 1e-6f));
  float max_rate = sqrtf(fmaxf(2.f * alpha * fabsf(error), 0.f));
  float desired = sgnf(error) * fminf(omega_limit, max_rate);
  if (!use_rate) return desired;
  return clampf(desired - 1.5f * (current_rate - desired), -omega_limit, omega_limit);
}

// Terrain under a point: height of the highest containing bump and its grade
// along x. Returns whether the point lies on a bump.
AD_HD bool bump_height(const SimParams& sp, float x, float y, float& height, float& grade) {
  const float panel = 0.0127f;                    // 0.5 in
  const float rise = 0.16543f - 0.0127f;          // 6.513 in - 0.5 in
  height = 0.f;
  grade = 0.f;
  bool on = false;
  float best = -1.f;
  for (int b = 0; b < sp.num_bumps; ++b) {
    const Box& bx = sp.bumps[b];
    float dx = x - bx.cx;
    float hx = fmaxf(bx.hx, 1e-6f);
    if (fabsf(dx) <= hx && fabsf(y - bx.cy) <= bx.hy) {
      on = true;
      float h = panel + rise * (1.f - fabsf(dx) / hx);
      if (h > best) {
        best = h;
        height = h;
        grade = -sgnf(dx) * rise / hx;
      }
    }
  }
  return on;
}

// One swerve drivetrain update for robot r over duration h
// (frc_defense/tensor_physics.py:585-697).
AD_HD void swerve_robot(TickShared& s, const SimParams& sp, int r, float h) {
  float* pose = s.pose + r * 3;
  float* vel = s.vel + r * 3;
  float* ms = s.ms + r * 20;
  const float L = rparam(s, r, RP_LENGTH), W = rparam(s, r, RP_WIDTH), m = rparam(s, r, RP_MASS);
  const float speed_limit = rparam(s, r, RP_SPEED), accel_limit = rparam(s, r, RP_ACCEL);
  const float omega_limit = rparam(s, r, RP_OMEGA), alpha = rparam(s, r, RP_ALPHA);
  const float ratio = rparam(s, r, RP_DRIVE_RATIO);
  const float drive_limit = rparam(s, r, RP_DRIVE_CURRENT);
  const float supply_limit = rparam(s, r, RP_DRIVE_SUPPLY);
  const float robot_supply = rparam(s, r, RP_ROBOT_SUPPLY);
  const float batt_r = rparam(s, r, RP_BATTERY_R);
  const float lat_mu = rparam(s, r, RP_LATERAL_MU);
  const float ground_mu = s.mu3[1];
  const float th = pose[2];
  const float c = cosf(th), sn = sinf(th);
  const float mxs[4] = {-sp.module_x, sp.module_x, -sp.module_x, sp.module_x};
  const float mys[4] = {-sp.module_y, -sp.module_y, sp.module_y, sp.module_y};
  float wheel_h[4], wheel_g[4];
  bool on_bump[4];
  for (int k = 0; k < 4; ++k) {
    float wx = pose[0] + c * mxs[k] - sn * mys[k];
    float wy = pose[1] + sn * mxs[k] + c * mys[k];
    on_bump[k] = bump_height(sp, wx, wy, wheel_h[k], wheel_g[k]);
  }
  const float front = .5f * (wheel_h[1] + wheel_h[3]);
  const float rear = .5f * (wheel_h[0] + wheel_h[2]);
  const float pitch = atan2f(front - rear, L);
  const float cg = 0.30f;
  float normal[4];
  for (int k = 0; k < 4; ++k)
    normal[k] = fmaxf(m * kG * cosf(pitch) / 4.f -
                      m * kG * cg * sinf(pitch) * sgnf(mxs[k]) / (2.f * fmaxf(L, 1e-6f)), 0.f);
  // commanded chassis velocity in the body frame
  const float* cmd = s.cmd + r * 3;
  float bvx = c * cmd[0] + sn * cmd[1];
  float bvy = -sn * cmd[0] + c * cmd[1];
  float omega = clampf(cmd[2], -omega_limit, omega_limit);
  float nrm = fmaxf(sqrtf(bvx * bvx + bvy * bvy), 1e-8f);
  float scale = fminf(speed_limit / nrm, 1.f);
  bvx *= scale;
  bvy *= scale;
  float tdx[4], tdy[4], target[4];
  float tmax = 0.f;
  for (int k = 0; k < 4; ++k) {
    tdx[k] = bvx - omega * mys[k];
    tdy[k] = bvy + omega * mxs[k];
    target[k] = sqrtf(tdx[k] * tdx[k] + tdy[k] * tdy[k]);
    tmax = fmaxf(tmax, target[k]);
  }
  const float desat = fminf(speed_limit / fmaxf(tmax, 1e-8f), 1.f);
  float steer_current[4];
  float steer_sum = 0.f;
  for (int k = 0; k < 4; ++k) {
    target[k] *= desat;
    float angle = atan2f(tdy[k], tdx[k]);
    float delta = wrap_angle(angle - ms[MS_ANGLE * 4 + k]);
    if (fabsf(delta) > kPi / 2) {
      angle += kPi;
      target[k] = -target[k];
    }
    angle = wrap_angle(angle);
    delta = wrap_angle(angle - ms[MS_ANGLE * 4 + k]);
    target[k] *= fmaxf(cosf(delta), 0.f);
    float steer_target = clampf(8.f * delta, -sp.steer_rate_limit, sp.steer_rate_limit);
    float se = steer_target - ms[MS_STEER_RATE * 4 + k];
    steer_current[k] = fminf(2.f * fabsf(se), sp.steer_current_limit);
    steer_sum += steer_current[k];
    float rate = clampf(ms[MS_STEER_RATE * 4 + k] + sgnf(se) * sp.steer_acceleration * steer_current[k] /
                            fmaxf(sp.steer_current_limit, 1e-6f) * h,
                        -sp.steer_rate_limit, sp.steer_rate_limit);
    ms[MS_STEER_RATE * 4 + k] = rate;
    ms[MS_ANGLE * 4 + k] = wrap_angle(ms[MS_ANGLE * 4 + k] + rate * h);
  }
  const float res = sp.nominal_voltage / sp.stall_current;
  const float stall = sp.free_speed_rpm * kTwoPi / 60.f;
  const float kv = stall / (sp.nominal_voltage - res * sp.free_current);
  const float kt = sp.stall_torque / sp.stall_current;
  const float bus = fmaxf(sp.battery_voltage - s.current[r] * batt_r, 0.f);
  float amps[4], supply[4], actual[4];
  float supply_sum = 0.f;
  for (int k = 0; k < 4; ++k) {
    float motor_target = target[k] / sp.wheel_radius * ratio;
    actual[k] = ms[MS_DRIVE_SPEED * 4 + k] / sp.wheel_radius * ratio;
    float duty = clampf(motor_target / stall + .8f * (motor_target - actual[k]) / stall, -1.f, 1.f);
    float a = clampf((duty * bus - actual[k] / kv) / res, -drive_limit, drive_limit);
    float sup = fabsf(duty * a);
    a *= fminf(supply_limit / fmaxf(sup, 1e-6f), 1.f);
    sup = fabsf(duty * a);
    amps[k] = a;
    supply[k] = sup;
    supply_sum += sup;
  }
  const float budget = fmaxf(robot_supply - steer_sum, 0.f);
  const float cap = fminf(budget / fmaxf(supply_sum, 1e-6f), 1.f);
  const float bvx0 = c * vel[0] + sn * vel[1];
  const float bvy0 = -sn * vel[0] + c * vel[1];
  float fxd = 0.f, fyd = 0.f, fxl = 0.f, fyl = 0.f, torque_z = 0.f, sup_total = 0.f, roll_n = 0.f;
  for (int k = 0; k < 4; ++k) {
    amps[k] *= cap;
    supply[k] *= cap;
    sup_total += supply[k];
    float torque = kt * (amps[k] - sp.free_current * sgnf(actual[k]));
    float force = torque * ratio * sp.motor_efficiency / sp.wheel_radius;
    float long_lim = ground_mu * normal[k];
    force = fmaxf(fminf(force, long_lim), -long_lim);
    float ma = ms[MS_ANGLE * 4 + k];
    float cma = cosf(ma), sma = sinf(ma);
    float mvx = bvx0 - vel[2] * mys[k];
    float mvy = bvy0 + vel[2] * mxs[k];
    float lat_v = -mvx * sma + mvy * cma;
    float lat_lim = lat_mu * normal[k];
    float lat_f = fminf(fmaxf(-lat_v * m / (4.f * h), -lat_lim), lat_lim);
    float comb = sqrtf(sqr(force / fmaxf(long_lim, 1e-8f)) + sqr(lat_f / fmaxf(lat_lim, 1e-8f)));
    float fs = fmaxf(comb, 1.f);
    force /= fs;
    lat_f /= fs;
    ms[MS_CURRENT * 4 + k] = amps[k];
    ms[MS_SUPPLY * 4 + k] = supply[k];
    float fx_d = force * cma, fy_d = force * sma;
    float fx_l = -lat_f * sma, fy_l = lat_f * cma;
    fxd += fx_d;
    fyd += fy_d;
    fxl += fx_l;
    fyl += fy_l;
    torque_z += mxs[k] * (fy_d + fy_l) - mys[k] * (fx_d + fx_l);
    if (on_bump[k]) roll_n += 0.0125f * normal[k];
  }
  s.current[r] = sup_total + steer_sum;
  float dax = fxd / m, day = fyd / m;
  float dscale = fminf(accel_limit / fmaxf(sqrtf(dax * dax + day * day), 1e-8f), 1.f);
  float ax = dax * dscale + fxl / m;
  float ay = day * dscale + fyl / m;
  float inertia = robot_inertia(s, r);
  float az = torque_z / inertia;
  float vx = vel[0] + (c * ax - sn * ay) * h;
  float vy = vel[1] + (sn * ax + c * ay) * h;
  float mean_grade = .25f * (wheel_g[0] + wheel_g[1] + wheel_g[2] + wheel_g[3]);
  float rolling_accel = roll_n / m;
  vx = vx + (-kG * mean_grade - rolling_accel * sgnf(vx)) * h;
  float vn = fmaxf(sqrtf(vx * vx + vy * vy), 1e-8f);
  float vs = fminf(speed_limit / vn, 1.f);
  vx *= vs;
  vy *= vs;
  float w = clampf(vel[2] + clampf(az, -alpha, alpha) * h, -omega_limit, omega_limit);
  vel[0] = vx;
  vel[1] = vy;
  vel[2] = w;
  float bx = c * vx + sn * vy, by = -sn * vx + c * vy;
  for (int k = 0; k < 4; ++k) {
    float ma = ms[MS_ANGLE * 4 + k];
    ms[MS_DRIVE_SPEED * 4 + k] = (bx - w * mys[k]) * cosf(ma) + (by + w * mxs[k]) * sinf(ma);
  }
}

#if defined(__CUDA_ARCH__)
// The four values one per module lane of a robot (lanes base..base+3) summed
// in module order, as the serial routine adds them.
__device__ __forceinline__ float module_sum(float v, int base) {
  const float a = __shfl_sync(0xffffffffu, v, base);
  const float b = __shfl_sync(0xffffffffu, v, base + 1);
  const float c = __shfl_sync(0xffffffffu, v, base + 2);
  const float d = __shfl_sync(0xffffffffu, v, base + 3);
  return ((a + b) + c) + d;
}

__device__ __forceinline__ float module_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

// swerve_robot with the four modules of each robot on four lanes of one warp
// (lane = 4 * robot + module; all 32 lanes call it, lanes past 4R only take
// part in the shuffles). Per-module arithmetic is that of swerve_robot and
// cross-module sums are added in module order.
__device__ void swerve_robot_lanes(TickShared& s, const SimParams& sp, float h) {
  const int lane = threadIdx.x & 31;
  const bool active = lane < 4 * sp.R;
  const int r = active ? (lane >> 2) : 0;
  const int k = lane & 3;
  const int base = lane & ~3;
  float* pose = s.pose + r * 3;
  float* vel = s.vel + r * 3;
  float* ms = s.ms + r * 20;
  const float L = rparam(s, r, RP_LENGTH), m = rparam(s, r, RP_MASS);
  const float speed_limit = rparam(s, r, RP_SPEED), accel_limit = rparam(s, r, RP_ACCEL);
  const float omega_limit = rparam(s, r, RP_OMEGA), alpha = rparam(s, r, RP_ALPHA);
  const float ratio = rparam(s, r, RP_DRIVE_RATIO);
  const float drive_limit = rparam(s, r, RP_DRIVE_CURRENT);
  const float supply_limit = rparam(s, r, RP_DRIVE_SUPPLY);
  const float robot_supply = rparam(s, r, RP_ROBOT_SUPPLY);
  const float batt_r = rparam(s, r, RP_BATTERY_R);
  const float lat_mu = rparam(s, r, RP_LATERAL_MU);
  const float ground_mu = s.mu3[1];
  const float th = pose[2];
  const float c = cosf(th), sn = sinf(th);
  const float mx = (k & 1) ? sp.module_x : -sp.module_x;
  const float my = (k & 2) ? sp.module_y : -sp.module_y;
  float wheel_h, wheel_g;
  const bool on_bump = bump_height(sp, pose[0] + c * mx - sn * my, pose[1] + sn * mx + c * my, wheel_h, wheel_g);
  const float h0 = __shfl_sync(0xffffffffu, wheel_h, base), h1 = __shfl_sync(0xffffffffu, wheel_h, base + 1);
  const float h2 = __shfl_sync(0xffffffffu, wheel_h, base + 2), h3 = __shfl_sync(0xffffffffu, wheel_h, base + 3);
  const float front = .5f * (h1 + h3);
  const float rear = .5f * (h0 + h2);
  const float pitch = atan2f(front - rear, L);
  const float cg = 0.30f;
  const float normal = fmaxf(m * kG * cosf(pitch) / 4.f -
                             m * kG * cg * sinf(pitch) * sgnf(mx) / (2.f * fmaxf(L, 1e-6f)), 0.f);
  const float* cmd = s.cmd + r * 3;
  float bvx = c * cmd[0] + sn * cmd[1];
  float bvy = -sn * cmd[0] + c * cmd[1];
  float omega = clampf(cmd[2], -omega_limit, omega_limit);
  float nrm = fmaxf(sqrtf(bvx * bvx + bvy * bvy), 1e-8f);
  float scale = fminf(speed_limit / nrm, 1.f);
  bvx *= scale;
  bvy *= scale;
  const float tdx = bvx - omega * my;
  const float tdy = bvy + omega * mx;
  float target = sqrtf(tdx * tdx + tdy * tdy);
  const float tmax = module_max(target);
  const float desat = fminf(speed_limit / fmaxf(tmax, 1e-8f), 1.f);
  target *= desat;
  float angle = atan2f(tdy, tdx);
  float delta = wrap_angle(angle - ms[MS_ANGLE * 4 + k]);
  if (fabsf(delta) > kPi / 2) {
    angle += kPi;
    target = -target;
  }
  angle = wrap_angle(angle);
  delta = wrap_angle(angle - ms[MS_ANGLE * 4 + k]);
  target *= fmaxf(cosf(delta), 0.f);
  const float steer_target = clampf(8.f * delta, -sp.steer_rate_limit, sp.steer_rate_limit);
  const float se = steer_target - ms[MS_STEER_RATE * 4 + k];
  const float steer_current = fminf(2.f * fabsf(se), sp.steer_current_limit);
  const float rate = clampf(ms[MS_STEER_RATE * 4 + k] + sgnf(se) * sp.steer_acceleration * steer_current /
                                fmaxf(sp.steer_current_limit, 1e-6f) * h,
                            -sp.steer_rate_limit, sp.steer_rate_limit);
  const float new_angle = wrap_angle(ms[MS_ANGLE * 4 + k] + rate * h);
  const float steer_sum = module_sum(steer_current, base);
  const float res = sp.nominal_voltage / sp.stall_current;
  const float stall = sp.free_speed_rpm * kTwoPi / 60.f;
  const float kv = stall / (sp.nominal_voltage - res * sp.free_current);
  const float kt = sp.stall_torque / sp.stall_current;
  const float bus = fmaxf(sp.battery_voltage - s.current[r] * batt_r, 0.f);
  const float motor_target = target / sp.wheel_radius * ratio;
  const float actual = ms[MS_DRIVE_SPEED * 4 + k] / sp.wheel_radius * ratio;
  const float duty = clampf(motor_target / stall + .8f * (motor_target - actual) / stall, -1.f, 1.f);
  float amps = clampf((duty * bus - actual / kv) / res, -drive_limit, drive_limit);
  float sup = fabsf(duty * amps);
  amps *= fminf(supply_limit / fmaxf(sup, 1e-6f), 1.f);
  float supply = fabsf(duty * amps);
  const float supply_sum = module_sum(supply, base);
  const float budget = fmaxf(robot_supply - steer_sum, 0.f);
  const float cap = fminf(budget / fmaxf(supply_sum, 1e-6f), 1.f);
  const float bvx0 = c * vel[0] + sn * vel[1];
  const float bvy0 = -sn * vel[0] + c * vel[1];
  const float vel2 = vel[2];
  amps *= cap;
  supply *= cap;
  const float torque = kt * (amps - sp.free_current * sgnf(actual));
  float force = torque * ratio * sp.motor_efficiency / sp.wheel_radius;
  const float long_lim = ground_mu * normal;
  force = fmaxf(fminf(force, long_lim), -long_lim);
  const float ma = new_angle;
  const float cma = cosf(ma), sma = sinf(ma);
  const float mvx = bvx0 - vel2 * my;
  const float mvy = bvy0 + vel2 * mx;
  const float lat_v = -mvx * sma + mvy * cma;
  const float lat_lim = lat_mu * normal;
  float lat_f = fminf(fmaxf(-lat_v * m / (4.f * h), -lat_lim), lat_lim);
  const float comb = sqrtf(sqr(force / fmaxf(long_lim, 1e-8f)) + sqr(lat_f / fmaxf(lat_lim, 1e-8f)));
  const float fs = fmaxf(comb, 1.f);
  force /= fs;
  lat_f /= fs;
  const float fx_d = force * cma, fy_d = force * sma;
  const float fx_l = -lat_f * sma, fy_l = lat_f * cma;
  const float fxd = module_sum(fx_d, base), fyd = module_sum(fy_d, base);
  const float fxl = module_sum(fx_l, base), fyl = module_sum(fy_l, base);
  const float torque_z = module_sum(mx * (fy_d + fy_l) - my * (fx_d + fx_l), base);
  const float sup_total = module_sum(supply, base);
  const float roll_n = module_sum(on_bump ? 0.0125f * normal : 0.f, base);
  const float g0 = __shfl_sync(0xffffffffu, wheel_g, base), g1 = __shfl_sync(0xffffffffu, wheel_g, base + 1);
  const float g2 = __shfl_sync(0xffffffffu, wheel_g, base + 2), g3 = __shfl_sync(0xffffffffu, wheel_g, base + 3);
  // every lane of the robot has read what it needs from vel/current/ms above
  __syncwarp();
  if (active) {
    ms[MS_STEER_RATE * 4 + k] = rate;
    ms[MS_ANGLE * 4 + k] = new_angle;
    ms[MS_CURRENT * 4 + k] = amps;
    ms[MS_SUPPLY * 4 + k] = supply;
  }
  const float dax = fxd / m, day = fyd / m;
  const float dscale = fminf(accel_limit / fmaxf(sqrtf(dax * dax + day * day), 1e-8f), 1.f);
  const float ax = dax * dscale + fxl / m;
  const float ay = day * dscale + fyl / m;
  const float inertia = robot_inertia(s, r);
  const float az = torque_z / inertia;
  float vx = vel[0] + (c * ax - sn * ay) * h;
  float vy = vel[1] + (sn * ax + c * ay) * h;
  const float mean_grade = .25f * (g0 + g1 + g2 + g3);
  const float rolling_accel = roll_n / m;
  vx = vx + (-kG * mean_grade - rolling_accel * sgnf(vx)) * h;
  const float vn = fmaxf(sqrtf(vx * vx + vy * vy), 1e-8f);
  const float vs = fminf(speed_limit / vn, 1.f);
  vx *= vs;
  vy *= vs;
  const float w = clampf(vel2 + clampf(az, -alpha, alpha) * h, -omega_limit, omega_limit);
  __syncwarp();
  if (active && k == 0) {
    s.current[r] = sup_total + steer_sum;
    vel[0] = vx;
    vel[1] = vy;
    vel[2] = w;
  }
  const float bx = c * vx + sn * vy, by = -sn * vx + c * vy;
  if (active) ms[MS_DRIVE_SPEED * 4 + k] = (bx - w * my) * cosf(ma) + (by + w * mx) * sinf(ma);
  __syncwarp();
}
#endif

// Rigid impulse with Coulomb friction against a fixed surface at a contact
// point (frc_defense/tensor_physics_collision.py:195-218).
AD_HD void static_contact_impulse(TickShared& s, int r, float px, float py, float nx, float ny,
                                  float friction) {
  float* pose = s.pose + r * 3;
  float* vel = s.vel + r * 3;
  const float m = rparam(s, r, RP_MASS);
  const float I = fmaxf(robot_inertia(s, r), 1e-8f);
  const float lx = px - pose[0], ly = py - pose[1];
  const float armx = -ly, army = lx;
  float cvx = vel[0] + vel[2] * armx, cvy = vel[1] + vel[2] * army;
  float vn = cvx * nx + cvy * ny;
  float inv = 1.f / m;
  float rn = cross2(lx, ly, nx, ny);
  float eff = inv + rn * rn / I;
  float jn = vn < 0.f ? -1.05f * vn / fmaxf(eff, 1e-8f) : 0.f;
  vel[0] += jn * nx * inv;
  vel[1] += jn * ny * inv;
  vel[2] += cross2(lx, ly, jn * nx, jn * ny) / I;
  float tx = -ny, ty = nx;
  cvx = vel[0] + vel[2] * armx;
  cvy = vel[1] + vel[2] * army;
  float vt = cvx * tx + cvy * ty;
  float rt = cross2(lx, ly, tx, ty);
  float efft = inv + rt * rt / I;
  float jt = fminf(fmaxf(-vt / fmaxf(efft, 1e-8f), -friction * jn), friction * jn);
  vel[0] += jt * tx * inv;
  vel[1] += jt * ty * inv;
  vel[2] += cross2(lx, ly, jt * tx, jt * ty) / I;
}

// Sequential x-min, x-max, y-min, y-max wall contacts
// (frc_defense/tensor_physics_collision.py:220-248).
AD_HD bool walls_robot(TickShared& s, const SimParams& sp, int r) {
  bool moved = false;
  float* pose = s.pose + r * 3;
  const float c = cosf(pose[2]), sn = sinf(pose[2]);
  const float hl = .5f * rparam(s, r, RP_LENGTH), hw = .5f * rparam(s, r, RP_WIDTH);
  const float hx = fabsf(c) * hl + fabsf(sn) * hw, hy = fabsf(sn) * hl + fabsf(c) * hw;
  const float ux = c, uy = sn, vx = -sn, vy = c;
  for (int wall = 0; wall < 4; ++wall) {
    int axis = wall >> 1;
    float sign = (wall & 1) ? -1.f : 1.f;
    float pen;
    if (wall == 0) pen = hx - pose[0];
    else if (wall == 1) pen = pose[0] + hx - sp.field_length;
    else if (wall == 2) pen = hy - pose[1];
    else pen = pose[1] + hy - sp.field_width;
    if (!(pen > 0.f)) continue;
    float nx = axis == 0 ? sign : 0.f, ny = axis == 1 ? sign : 0.f;
    pose[0] += nx * (pen + 1e-4f);
    pose[1] += ny * (pen + 1e-4f);
    float twx = -nx, twy = -ny;
    float px = pose[0] + sgnf(twx * ux + twy * uy) * ux * hl + sgnf(twx * vx + twy * vy) * vx * hw;
    float py = pose[1] + sgnf(twx * ux + twy * uy) * uy * hl + sgnf(twx * vx + twy * vy) * vy * hw;
    static_contact_impulse(s, r, px, py, nx, ny, s.mu3[2]);
    s.rflag[r * 4 + RF_WALL_X + axis] = 1;
    moved = true;
  }
  return moved;
}

// Most-penetrating oriented-robot vs axis-aligned field box contact
// (frc_defense/tensor_physics_collision.py:289-376).
AD_HD bool field_collision_robot(TickShared& s, const SimParams& sp, int r) {
  if (sp.num_boxes == 0) return false;
  float* pose = s.pose + r * 3;
  const float* vel = s.vel + r * 3;
  const float c = cosf(pose[2]), sn = sinf(pose[2]);
  const float ac = fabsf(c), as = fabsf(sn);
  const float hl = .5f * rparam(s, r, RP_LENGTH), hw = .5f * rparam(s, r, RP_WIDTH);
  const float ax[4] = {1.f, 0.f, c, -sn};
  const float ay[4] = {0.f, 1.f, sn, c};
  const float rr[4] = {ac * hl + as * hw, as * hl + ac * hw, hl, hw};
  float best_depth = -1.f;
  int best = -1;
  float best_pen[4], best_signed[4];
  for (int b = 0; b < sp.num_boxes; ++b) {
    const Box& bx = sp.boxes[b];
    // AABB broadphase
    if (fabsf(pose[0] - bx.cx) > rr[0] + bx.hx + 1e-6f || fabsf(pose[1] - bx.cy) > rr[1] + bx.hy + 1e-6f)
      continue;
    float dx = pose[0] - bx.cx, dy = pose[1] - bx.cy;
    float br[4] = {bx.hx, bx.hy, bx.hx * ac + bx.hy * as, bx.hx * as + bx.hy * ac};
    float pen[4], sg[4];
    float mn = kInf;
    for (int k = 0; k < 4; ++k) {
      sg[k] = ax[k] * dx + ay[k] * dy;
      pen[k] = rr[k] + br[k] - fabsf(sg[k]);
      mn = fminf(mn, pen[k]);
    }
    if (mn >= 0.f && mn > best_depth) {
      best_depth = mn;
      best = b;
      for (int k = 0; k < 4; ++k) {
        best_pen[k] = pen[k];
        best_signed[k] = sg[k];
      }
    }
  }
  if (best < 0) return false;
  const Box& bx = sp.boxes[best];
  float cnx[4], cny[4];
  int axis = -1;
  float best_app = kInf;
  int argmin = 0;
  for (int k = 0; k < 4; ++k) {
    float sg = best_signed[k] >= 0.f ? 1.f : -1.f;
    cnx[k] = ax[k] * sg;
    cny[k] = ay[k] * sg;
    if (best_pen[k] < best_pen[argmin]) argmin = k;
    bool tied = best_pen[k] <= best_depth + 1e-6f && best_pen[k] >= 0.f;
    float app = cnx[k] * vel[0] + cny[k] * vel[1];
    if (tied && app < best_app) {
      best_app = app;
      axis = k;
    }
  }
  if (!(best_app < -1e-6f)) axis = argmin;
  const float nx = cnx[axis], ny = cny[axis];
  const float depth = fmaxf(best_depth, 0.f);
  pose[0] += nx * (depth + 1e-4f);
  pose[1] += ny * (depth + 1e-4f);
  const float ux = c, uy = sn, vx = -sn, vy = c;
  const float tx = -ny, ty = nx;
  float robot_n = fabsf(nx * ux + ny * uy) * hl + fabsf(nx * vx + ny * vy) * hw;
  float box_n = fabsf(nx) * bx.hx + fabsf(ny) * bx.hy;
  float ncoord = .5f * ((nx * pose[0] + ny * pose[1]) - robot_n + (nx * bx.cx + ny * bx.cy) + box_n);
  float robot_t = fabsf(tx * ux + ty * uy) * hl + fabsf(tx * vx + ty * vy) * hw;
  float box_t = fabsf(tx) * bx.hx + fabsf(ty) * bx.hy;
  float rc = tx * pose[0] + ty * pose[1];
  float bc = tx * bx.cx + ty * bx.cy;
  float lo = fmaxf(rc - robot_t, bc - box_t), hi = fminf(rc + robot_t, bc + box_t);
  float tcoord = .5f * (lo + hi);
  float px = nx * ncoord + tx * tcoord, py = ny * ncoord + ty * tcoord;
  static_contact_impulse(s, r, px, py, nx, ny, s.mu3[2]);
  s.rflag[r * 4 + RF_FIELD_CONTACT] = 1;
  s.eflag[0] = 1;  // world robot_contact includes static contacts (reference semantics)
  return true;
}

// Robot pair q: SAT overlap, position correction split by inverse mass, and
// normal+friction impulses computed from the pre-contact velocities
// (frc_defense/tensor_physics_collision.py:88-168). Writes per-pair deltas.
AD_HD void robot_pair_compute(TickShared& s, const SimParams& sp, int q) {
  const int i = sp.pair_i[q], j = sp.pair_j[q];
  const float* pi = s.pose + i * 3;
  const float* pj = s.pose + j * 3;
  {
    // disjoint circumscribed circles: the rectangles cannot overlap (the SAT
    // below would find a separating axis), so skip it
    const float ddx = pj[0] - pi[0], ddy = pj[1] - pi[1];
    const float reach = .5f * (sqrtf(sqr(rparam(s, i, RP_LENGTH)) + sqr(rparam(s, i, RP_WIDTH))) +
                               sqrtf(sqr(rparam(s, j, RP_LENGTH)) + sqr(rparam(s, j, RP_WIDTH))));
    if (ddx * ddx + ddy * ddy > reach * reach * 1.0002f + 1e-6f) {
      s.pq_valid[q] = 0;
      for (int k = 0; k < 6; ++k) s.pq_dv[q * 6 + k] = 0.f;
      for (int k = 0; k < 4; ++k) s.pq_move[q * 4 + k] = 0.f;
      s.pq_jn[q] = 0.f;
      s.pq_jt[q] = 0.f;
      return;
    }
  }
  const float ci = cosf(pi[2]), si = sinf(pi[2]), cj = cosf(pj[2]), sj = sinf(pj[2]);
  const float axx[4] = {ci, -si, cj, -sj};
  const float axy[4] = {si, ci, sj, cj};
  const float hil = .5f * rparam(s, i, RP_LENGTH), hiw = .5f * rparam(s, i, RP_WIDTH);
  const float hjl = .5f * rparam(s, j, RP_LENGTH), hjw = .5f * rparam(s, j, RP_WIDTH);
  const float dx = pj[0] - pi[0], dy = pj[1] - pi[1];
  float depth = kInf, sgn = 1.f;
  int k_best = 0;
  for (int k = 0; k < 4; ++k) {
    float pu = fabsf(axx[k] * ci + axy[k] * si), pv = fabsf(axx[k] * -si + axy[k] * ci);
    float qu = fabsf(axx[k] * cj + axy[k] * sj), qv = fabsf(axx[k] * -sj + axy[k] * cj);
    float rad = pu * hil + pv * hiw + qu * hjl + qv * hjw;
    float sd = axx[k] * dx + axy[k] * dy;
    float ov = rad - fabsf(sd);
    if (ov < depth) {
      depth = ov;
      k_best = k;
      sgn = sd >= 0.f ? 1.f : -1.f;
    }
  }
  const bool valid = depth > 0.f;
  s.pq_valid[q] = valid ? 1 : 0;
  for (int k = 0; k < 6; ++k) s.pq_dv[q * 6 + k] = 0.f;
  for (int k = 0; k < 4; ++k) s.pq_move[q * 4 + k] = 0.f;
  s.pq_jn[q] = 0.f;
  s.pq_jt[q] = 0.f;
  if (!valid) return;
  const float nx = axx[k_best] * sgn, ny = axy[k_best] * sgn;
  s.pq_n[q * 2] = nx;
  s.pq_n[q * 2 + 1] = ny;
  const float mi = rparam(s, i, RP_MASS), mj = rparam(s, j, RP_MASS);
  const float inv_i = 1.f / mi, inv_j = 1.f / mj;
  const float total = fmaxf(inv_i + inv_j, 1e-8f);
  const float corr = fmaxf(depth, 0.f) + 1e-4f;
  s.pq_move[q * 4 + 0] = -nx * corr * inv_i / total;
  s.pq_move[q * 4 + 1] = -ny * corr * inv_i / total;
  s.pq_move[q * 4 + 2] = nx * corr * inv_j / total;
  s.pq_move[q * 4 + 3] = ny * corr * inv_j / total;
  // contact point midway between the bumper support points (pre-correction poses)
  float sxi = pi[0] + sgnf(nx * ci + ny * si) * ci * hil + sgnf(nx * -si + ny * ci) * -si * hiw;
  float syi = pi[1] + sgnf(nx * ci + ny * si) * si * hil + sgnf(nx * -si + ny * ci) * ci * hiw;
  float sxj = pj[0] - sgnf(nx * cj + ny * sj) * cj * hjl - sgnf(nx * -sj + ny * cj) * -sj * hjw;
  float syj = pj[1] - sgnf(nx * cj + ny * sj) * sj * hjl - sgnf(nx * -sj + ny * cj) * cj * hjw;
  float cpx = .5f * (sxi + sxj), cpy = .5f * (syi + syj);
  float rix = cpx - pi[0], riy = cpy - pi[1], rjx = cpx - pj[0], rjy = cpy - pj[1];
  const float* vi = s.vel + i * 3;
  const float* vj = s.vel + j * 3;
  float vcix = vi[0] + vi[2] * -riy, vciy = vi[1] + vi[2] * rix;
  float vcjx = vj[0] + vj[2] * -rjy, vcjy = vj[1] + vj[2] * rjx;
  float relx = vcjx - vcix, rely = vcjy - vciy;
  float vn = relx * nx + rely * ny;
  float Ii = fmaxf(robot_inertia(s, i), 1e-8f), Ij = fmaxf(robot_inertia(s, j), 1e-8f);
  float rni = cross2(rix, riy, nx, ny), rnj = cross2(rjx, rjy, nx, ny);
  float eff = total + rni * rni / Ii + rnj * rnj / Ij;
  float jn = vn < 0.f ? -(1.05f * vn) / fmaxf(eff, 1e-8f) : 0.f;
  float tx = -ny, ty = nx;
  float vt, rti, rtj, efft, jt, mu;
  if (sp.R == 2) {
    // two-robot variant: normal impulse first, friction from updated velocities,
    // bumper friction used directly (frc_defense/tensor_physics_collision.py:33-86)
    float dvix = -jn * nx * inv_i, dviy = -jn * ny * inv_i, dwi = -jn * rni / Ii;
    float dvjx = jn * nx * inv_j, dvjy = jn * ny * inv_j, dwj = jn * rnj / Ij;
    float ui0 = vi[0] + dvix, ui1 = vi[1] + dviy, ui2 = vi[2] + dwi;
    float uj0 = vj[0] + dvjx, uj1 = vj[1] + dvjy, uj2 = vj[2] + dwj;
    float ax2 = (uj0 + uj2 * -rjy) - (ui0 + ui2 * -riy);
    float ay2 = (uj1 + uj2 * rjx) - (ui1 + ui2 * rix);
    vt = ax2 * tx + ay2 * ty;
    mu = s.mu3[0];
    rti = cross2(rix, riy, tx, ty);
    rtj = cross2(rjx, rjy, tx, ty);
    efft = total + rti * rti / Ii + rtj * rtj / Ij;
    jt = fminf(fmaxf(-vt / fmaxf(efft, 1e-8f), -mu * jn), mu * jn);
  } else {
    vt = relx * tx + rely * ty;
    rti = cross2(rix, riy, tx, ty);
    rtj = cross2(rjx, rjy, tx, ty);
    efft = total + rti * rti / Ii + rtj * rtj / Ij;
    mu = sqrtf(fmaxf(s.mu3[0], 0.f));
    jt = fminf(fmaxf(-vt / fmaxf(efft, 1e-8f), -mu * jn), mu * jn);
  }
  float impx = jn * nx + jt * tx, impy = jn * ny + jt * ty;
  s.pq_dv[q * 6 + 0] = -impx * inv_i;
  s.pq_dv[q * 6 + 1] = -impy * inv_i;
  s.pq_dv[q * 6 + 2] = -(jn * rni + jt * rti) / Ii;
  s.pq_dv[q * 6 + 3] = impx * inv_j;
  s.pq_dv[q * 6 + 4] = impy * inv_j;
  s.pq_dv[q * 6 + 5] = (jn * rnj + jt * rtj) / Ij;
  s.pq_jn[q] = jn;
  s.pq_jt[q] = jt;
}

// Sum every pair's delta into robot r in pair order (deterministic).
AD_HD void robot_pair_apply(TickShared& s, const SimParams& sp, int r) {
  float mx = 0.f, my = 0.f, vx = 0.f, vy = 0.f, w = 0.f;
  bool touched = false, opp = false;
  for (int q = 0; q < sp.Q; ++q) {
    if (!s.pq_valid[q]) continue;
    if (sp.pair_i[q] == r) {
      mx += s.pq_move[q * 4 + 0];
      my += s.pq_move[q * 4 + 1];
      vx += s.pq_dv[q * 6 + 0];
      vy += s.pq_dv[q * 6 + 1];
      w += s.pq_dv[q * 6 + 2];
      touched = true;
    } else if (sp.pair_j[q] == r) {
      mx += s.pq_move[q * 4 + 2];
      my += s.pq_move[q * 4 + 3];
      vx += s.pq_dv[q * 6 + 3];
      vy += s.pq_dv[q * 6 + 4];
      w += s.pq_dv[q * 6 + 5];
      touched = true;
    }
    if (sp.team[sp.pair_i[q]] != sp.team[sp.pair_j[q]]) opp = true;
  }
  s.pose[r * 3 + 0] += mx;
  s.pose[r * 3 + 1] += my;
  s.vel[r * 3 + 0] += vx;
  s.vel[r * 3 + 1] += vy;
  s.vel[r * 3 + 2] += w;
  if (touched) s.rflag[r * 4 + RF_ROBOT_CONTACT] = 1;
  (void)opp;
}

// Solver-originated contact evidence per robot pair (six-robot roster only,
// frc_defense/tensor_physics_collision.py:170-193).
AD_HD void record_pair_events(TickShared& s, const SimParams& sp, World& w, int env, float h) {
  if (sp.R != 6) return;
  const int end_sub = s.substep_index + 1;
  const float end_time = (float)(s.phys_time + (double)h);
  for (int q = 0; q < sp.Q; ++q) {
    bool valid = s.pq_valid[q];
    int32_t* cnt = w.pair_count + ((size_t)env * sp.Q + q) * 2;
    int32_t* sub = w.pair_substep + ((size_t)env * sp.Q + q) * 2;
    float* tm = w.pair_time + ((size_t)env * sp.Q + q) * 2;
    float* imp = w.pair_impulse + ((size_t)env * sp.Q + q) * 4;
    if (!valid) continue;
    if (cnt[0] == 0) {
      sub[0] = end_sub;
      tm[0] = end_time;
    }
    if (sub[1] != end_sub) {
      sub[1] = end_sub;
      tm[1] = end_time;
      cnt[0] += 1;
    }
    cnt[1] += 1;
    float jn = s.pq_jn[q], jt = s.pq_jt[q];
    float nx = s.pq_n[q * 2], ny = s.pq_n[q * 2 + 1];
    imp[0] += jn;
    imp[1] += jt;
    imp[2] += jn * nx + jt * -ny;
    imp[3] += jn * ny + jt * nx;
  }
}

// One robot substep: swerve, swept integration with field contacts, then up
// to contact_iterations rounds of pair/wall/field resolution. Runs on thread
// group `g` (one warp on the GPU while the FUEL warps work concurrently). A
// round that finds no robot pair in contact and moves no robot off a wall or
// field element leaves the state unchanged, so the remaining rounds (which
// would repeat it exactly) are skipped. Ends by caching each robot's heading
// trig and contact reach for the chassis-FUEL contacts.
AD_HD void robot_substep(TickShared& s, const SimParams& sp, World& w, int env, float h, const Group& g) {
#if defined(__CUDA_ARCH__)
  if (g.bar < 0 && sp.R <= 8) {
    swerve_robot_lanes(s, sp, h);
  } else {
    GFOR(r, sp.R, g) { swerve_robot(s, sp, r, h); }
  }
#else
  GFOR(r, sp.R, g) { swerve_robot(s, sp, r, h); }
#endif
  group_sync(g);
  PHASE_MARK_BY(s, 0, g.first);
  SERIAL_BEGIN
  s.eflag[0] = 0;
  s.eflag[1] = 0;
  SERIAL_END
  GFOR(r, sp.R, g) {
    for (int k = 0; k < 4; ++k) s.rflag[r * 4 + k] = 0;
    const float hs = h / (float)sp.sweep_steps;
    for (int step = 0; step < sp.sweep_steps; ++step) {
      s.pose[r * 3 + 0] += s.vel[r * 3 + 0] * hs;
      s.pose[r * 3 + 1] += s.vel[r * 3 + 1] * hs;
      s.pose[r * 3 + 2] = wrap_angle(s.pose[r * 3 + 2] + s.vel[r * 3 + 2] * hs);
      field_collision_robot(s, sp, r);
    }
  }
  group_sync(g);
  PHASE_MARK_BY(s, 1, g.first);
  for (int it = 0; it < sp.contact_iterations; ++it) {
    GFOR(q, sp.Q, g) { robot_pair_compute(s, sp, q); }
    group_sync(g);
    bool any = false;
    for (int q = 0; q < sp.Q; ++q) any = any || s.pq_valid[q];
    if (any) {
      SERIAL_BEGIN
      bool opp = false;
      for (int q = 0; q < sp.Q; ++q)
        if (s.pq_valid[q] && sp.team[sp.pair_i[q]] != sp.team[sp.pair_j[q]]) opp = true;
      s.eflag[0] = 1;
      if (opp) s.eflag[1] = 1;
      record_pair_events(s, sp, w, env, h);
      SERIAL_END
    }
    bool moved = false;
    GFOR(r, sp.R, g) {
      if (any) robot_pair_apply(s, sp, r);
      moved = walls_robot(s, sp, r) || moved;
      moved = field_collision_robot(s, sp, r) || moved;
    }
    group_sync(g);
    moved = group_any(g, moved);
    if (!any && !moved) break;
  }
  PHASE_MARK_BY(s, 2, g.first);
  GFOR(r, sp.R, g) {
    s.safety[r * 4 + 0] += 1;
    s.safety[r * 4 + 1] += s.rflag[r * 4 + RF_ROBOT_CONTACT] ? 1 : 0;
    s.safety[r * 4 + 2] += s.rflag[r * 4 + RF_FIELD_CONTACT] ? 1 : 0;
    s.safety[r * 4 + 3] += (s.rflag[r * 4 + RF_WALL_X] | s.rflag[r * 4 + RF_WALL_Y]) ? 1 : 0;
    const float th = s.pose[r * 3 + 2];
    s.rtrig[r * 4 + 0] = cosf(th);
    s.rtrig[r * 4 + 1] = sinf(th);
    const float reach = .5f * sqrtf(sqr(rparam(s, r, RP_LENGTH)) + sqr(rparam(s, r, RP_WIDTH))) + sp.fr;
    s.rtrig[r * 4 + 2] = reach * reach;
  }
  SERIAL_BEGIN
  s.substep_index += 1;
  s.phys_time += (double)h;
  SERIAL_END
  group_sync(g);
  PHASE_MARK_BY(s, 3, g.first);
}

// ----------------------------------------------------------------------------
// FUEL
// ----------------------------------------------------------------------------

// Backward-Euler spring-damper normal impulse plus capped Coulomb friction
// (frc_defense/fuel_physics.py:384-400). Returns the impulse on the first body.
AD_HD V3 fuel_impulse(const SimParams& sp, V3 n, float depth, V3 rel, float inv_mass, float h,
                      float tangent_inv, float damping) {
  float vn = dot3(rel, n);
  float jn = fmaxf(h * (sp.fk * depth - damping * vn) /
                       (1.f + h * damping * inv_mass + h * h * sp.fk * inv_mass),
                   0.f);
  if (depth >= 2.f * sp.fr * sp.max_comp) jn = fmaxf(jn, fmaxf(-vn / inv_mass, 0.f));
  V3 t = V3{rel.x - vn * n.x, rel.y - vn * n.y, rel.z - vn * n.z};
  float speed = norm3(t);
  float jt = fminf(speed / tangent_inv, sp.fmu * jn);
  float inv_s = 1.f / fmaxf(speed, 1e-12f);
  return V3{jn * n.x - jt * t.x * inv_s, jn * n.y - jt * t.y * inv_s, jn * n.z - jt * t.z * inv_s};
}

AD_HD void box_normal2(float lx, float ly, float hx, float hy, float& nx, float& ny, float& signed_d) {
  float cx = fminf(fmaxf(lx, -hx), hx), cy = fminf(fmaxf(ly, -hy), hy);
  float dx = lx - cx, dy = ly - cy;
  float d = sqrtf(dx * dx + dy * dy);
  if (d > 1e-12f) {
    nx = dx / d;
    ny = dy / d;
    signed_d = d;
  } else {
    float gx = hx - fabsf(lx), gy = hy - fabsf(ly);
    if (gx <= gy) {
      nx = lx >= 0.f ? 1.f : -1.f;
      ny = 0.f;
      signed_d = -gx;
    } else {
      nx = 0.f;
      ny = ly >= 0.f ? 1.f : -1.f;
      signed_d = -gy;
    }
  }
}

AD_HD int fuel_cell_of(const SimParams& sp, float x, float y) {
  int cx = clampi((int)floorf(x / sp.grid_cell), 0, sp.grid_nx - 1);
  int cy = clampi((int)floorf(y / sp.grid_cell), 0, sp.grid_ny - 1);
  return cy * sp.grid_nx + cx;
}

// Exclusive scan of cell_start[0..n) in place; cell_start[n] = total.
// Exclusive scan of cell_start[0..n) by a thread group; cell_start[n] = total.
// On the GPU each warp owns a 128-cell-aligned segment and reads it as int4
// (lane-consecutive, no bank conflicts): pass 1 sums the segment, pass 2 scans
// it with a running carry that starts at the sum of the earlier segments.
AD_HD void group_exclusive_scan(TickShared& s, int n, const Group& g) {
#if defined(__CUDA_ARCH__)
  const int lane = threadIdx.x & 31, warp = g.rank >> 5, warps = g.size >> 5;
  const int seg = ((n + warps - 1) / warps + 127) & ~127;
  const int b = warp * seg, e = min(b + seg, n);
  int4* cs4 = reinterpret_cast<int4*>(s.cell_start);
  int* wsum = reinterpret_cast<int*>(s.red);
  int tot = 0;
  for (int c = b + lane * 4; c < e; c += 128) {
    const int4 v = cs4[c >> 2];
    tot += v.x + (c + 1 < e ? v.y : 0) + (c + 2 < e ? v.z : 0) + (c + 3 < e ? v.w : 0);
  }
  for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
  if (lane == 0) wsum[warp] = tot;
  group_sync(g);
  int carry = 0, all = 0;
  for (int w2 = 0; w2 < warps; ++w2) {
    const int t = wsum[w2];
    if (w2 < warp) carry += t;
    all += t;
  }
  for (int c0 = b; c0 < b + seg; c0 += 128) {  // uniform trip count: every lane shuffles
    const int c = c0 + lane * 4;
    int4 v = make_int4(0, 0, 0, 0);
    if (c < e) {
      v = cs4[c >> 2];
      if (c + 1 >= e) v.y = 0;
      if (c + 2 >= e) v.z = 0;
      if (c + 3 >= e) v.w = 0;
    }
    const int lsum = v.x + v.y + v.z + v.w;
    int incl = lsum;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int base = carry + incl - lsum;
    if (c < e) {
      const int4 out = make_int4(base, base + v.x, base + v.x + v.y, base + v.x + v.y + v.z);
      if (c + 3 < e) {
        cs4[c >> 2] = out;
      } else {
        s.cell_start[c] = out.x;
        if (c + 1 < e) s.cell_start[c + 1] = out.y;
        if (c + 2 < e) s.cell_start[c + 2] = out.z;
      }
    }
    carry += __shfl_sync(0xffffffffu, incl, 31);
    if (c0 + 128 >= e) break;
  }
  if (g.rank == 0) s.cell_start[n] = all;
  group_sync(g);
#else
  (void)g;
  int acc = 0;
  for (int k = 0; k < n; ++k) {
    int t = s.cell_start[k];
    s.cell_start[k] = acc;
    acc += t;
  }
  s.cell_start[n] = acc;
#endif
}

AD_HD int atomic_inc_cell(TickShared& s, int cell) {
#if defined(__CUDA_ARCH__)
  return atomicAdd(&s.cell_start[cell], 1);
#else
  return s.cell_start[cell]++;
#endif
}

AD_HD void mark_awake_cell(TickShared& s, int cell) {
#if defined(__CUDA_ARCH__)
  atomicOr(&s.awake_bits[cell >> 5], 1u << (cell & 31));
#else
  s.awake_bits[cell >> 5] |= 1u << (cell & 31);
#endif
}

AD_HD bool cell_awake(const TickShared& s, int cell) { return (s.awake_bits[cell >> 5] >> (cell & 31)) & 1u; }

// Append sphere i to the work list when `take` (warp-aggregated on the GPU:
// one shared atomic per warp). Every lane of the warp must call it.
AD_HD void push_work(TickShared& s, int i, bool take) {
#if defined(__CUDA_ARCH__)
  const unsigned m = __ballot_sync(0xffffffffu, take);
  if (!m) return;
  const int lane = threadIdx.x & 31;
  const int leader = __ffs(m) - 1;
  int base = 0;
  if (lane == leader) base = atomicAdd(&s.nwork, __popc(m));
  base = __shfl_sync(0xffffffffu, base, leader);
  if (take) s.work[base + __popc(m & ((1u << lane) - 1u))] = (int16_t)i;
#else
  if (take) s.work[s.nwork++] = (int16_t)i;
#endif
}

// A sleeping sphere only receives impulses from awake neighbours: it needs the
// pair scan iff it is awake or one of its 3x3 cells holds an awake sphere.
AD_HD bool needs_pair_scan(const TickShared& s, const SimParams& sp, int i) {
  if (!s.sleep[i]) return true;
  // the cell index of fuel_cell_of, without an integer division
  const int cx = clampi((int)floorf(s.fpos[0][i] / sp.grid_cell), 0, sp.grid_nx - 1);
  const int cy = clampi((int)floorf(s.fpos[1][i] / sp.grid_cell), 0, sp.grid_ny - 1);
  for (int oy = -1; oy <= 1; ++oy) {
    const int yy = cy + oy;
    if (yy < 0 || yy >= sp.grid_ny) continue;
    for (int ox = -1; ox <= 1; ++ox) {
      const int xx = cx + ox;
      if (xx >= 0 && xx < sp.grid_nx && cell_awake(s, yy * sp.grid_nx + xx)) return true;
    }
  }
  return false;
}

AD_HD void static_contact_fuel(TickShared& s, const SimParams& sp, int i, V3 n, float depth, bool valid,
                               float h) {
  if (!(valid && depth > 0.f && !s.sleep[i])) return;
  const float I = .4f * sp.fm * sp.fr * sp.fr;
  V3 arm = V3{-sp.fr * n.x, -sp.fr * n.y, -sp.fr * n.z};
  V3 w = V3{s.fang[0][i], s.fang[1][i], s.fang[2][i]};
  V3 v = V3{s.fvel[0][i], s.fvel[1][i], s.fvel[2][i]};
  V3 wa = cross3(w, arm);
  V3 rel = V3{v.x + wa.x, v.y + wa.y, v.z + wa.z};
  V3 imp = fuel_impulse(sp, n, depth, rel, 1.f / sp.fm, h, 1.f / sp.fm + 2.5f / sp.fm, sp.fc);
  s.fvel[0][i] = v.x + imp.x / sp.fm;
  s.fvel[1][i] = v.y + imp.y / sp.fm;
  s.fvel[2][i] = v.z + imp.z / sp.fm;
  V3 dw = cross3(arm, imp);
  w = V3{w.x + dw.x / I, w.y + dw.y / I, w.z + dw.z / I};
  if (sp.froll > 0.f) {
    float mag = norm3(w);
    float loss = sp.froll * norm3(imp) * sp.fr / I;
    float k = fmaxf(1.f - loss / fmaxf(mag, 1e-12f), 0.f);
    w = V3{w.x * k, w.y * k, w.z * k};
  }
  s.fang[0][i] = w.x;
  s.fang[1][i] = w.y;
  s.fang[2][i] = w.z;
}

// One FUEL substep for the pieces marked free in s.freem
// (frc_defense/fuel_physics.py:513-587).
// FUEL phases that read no robot state (wake, integrate, grid, pair contacts,
// Jacobi apply), run by thread group `g`.
AD_HD void fuel_pre(TickShared& s, const SimParams& sp, float h, const Group& g) {
  const int P = sp.P;
  const float r2 = 2.f * sp.fr;
  // wake, gravity, explicit position update
  GFOR(i, P, g) {
    if (s.freem[i]) {
      float vx = s.fvel[0][i], vy = s.fvel[1][i], vz = s.fvel[2][i];
      float wn = sqrtf(sqr(s.fang[0][i]) + sqr(s.fang[1][i]) + sqr(s.fang[2][i]));
      if (sqrtf(vx * vx + vy * vy + vz * vz) >= sp.sleep_speed || wn >= sp.sleep_ang) s.sleep[i] = 0;
      if (!s.sleep[i]) {
        vz -= sp.fg * h;
        s.fvel[2][i] = vz;
        s.fpos[0][i] += vx * h;
        s.fpos[1][i] += vy * h;
        s.fpos[2][i] += vz * h;
      }
    }
  }
  // uniform XY grid (counting sort)
  const int ncell = sp.grid_nx * sp.grid_ny;
#if defined(__CUDA_ARCH__)
  {
    int4* cs = reinterpret_cast<int4*>(s.cell_start);
    int4* ab = reinterpret_cast<int4*>(s.awake_bits);
    const int4 z = make_int4(0, 0, 0, 0);
    GFOR(c, (ncell + 1 + 3) / 4, g) { cs[c] = z; }
    GFOR(c, (ncell / 32 + 1 + 3) / 4, g) { ab[c] = z; }
  }
#else
  GFOR(c, ncell + 1, g) { s.cell_start[c] = 0; }
  GFOR(c, ncell / 32 + 1, g) { s.awake_bits[c] = 0u; }
#endif
  if (g.rank == 0) {
    s.nwork = 0;
    s.cmask = 0u;
  }
  group_sync(g);
  PHASE_MARK_BY(s, 4, g.first);
  GFOR(i, P, g) {
    if (s.freem[i]) {
      int c = fuel_cell_of(sp, s.fpos[0][i], s.fpos[1][i]);
      s.cell[i] = (int16_t)c;
      s.slot[i] = (int16_t)atomic_inc_cell(s, c);
      if (!s.sleep[i]) mark_awake_cell(s, c);
    }
  }
  group_sync(g);
  PHASE_MARK_BY(s, 14, g.first);
  group_exclusive_scan(s, ncell, g);
  PHASE_MARK_BY(s, 15, g.first);
  for (int b0 = 0; b0 < P; b0 += g.size) {  // uniform trip count (warp-aggregated push)
    const int i = b0 + g.rank;
    bool listed = false;
    if (i < P) {
      if (s.freem[i]) {
        s.sorted[s.cell_start[(int)s.cell[i]] + (int)s.slot[i]] = (int16_t)i;
        listed = needs_pair_scan(s, sp, i);
      }
      s.listed[i] = listed ? 1 : 0;
    }
    push_work(s, i, listed);
  }
  group_sync(g);
  PHASE_MARK_BY(s, 5, g.first);
  float local_max[2] = {0.f, 0.f};
  const float I = .4f * sp.fm * sp.fr * sp.fr;
  // Jacobi pair contacts over the work list, each sphere computing the
  // impulses that act on it (spheres off the list receive none this substep)
  const int nwork = s.nwork;
  GFOR(k, nwork, g) {
    const int i = s.work[k];
    float dvx = 0.f, dvy = 0.f, dvz = 0.f, dwx = 0.f, dwy = 0.f, dwz = 0.f;
    int deg = 0;
    {
      const float px = s.fpos[0][i], py = s.fpos[1][i], pz = s.fpos[2][i];
      // candidate cells: those overlapping [p - r2, p + r2] in x and y (any
      // contact lies there; the cell index is monotone in the coordinate; a
      // 0.1 mm margin absorbs rounding); the cells of a row are consecutive in
      // the sorted order
      const float inv_cell = 1.f / sp.grid_cell, reach = r2 + 1e-4f;
      const int x0 = clampi((int)floorf((px - reach) * inv_cell), 0, sp.grid_nx - 1);
      const int x1 = clampi((int)floorf((px + reach) * inv_cell), 0, sp.grid_nx - 1);
      const int y0 = clampi((int)floorf((py - reach) * inv_cell), 0, sp.grid_ny - 1);
      const int y1 = clampi((int)floorf((py + reach) * inv_cell), 0, sp.grid_ny - 1);
      const bool sleep_i = s.sleep[i];
      const V3 vi = V3{s.fvel[0][i], s.fvel[1][i], s.fvel[2][i]};
      const V3 wi = V3{s.fang[0][i], s.fang[1][i], s.fang[2][i]};
      for (int yy = y0; yy <= y1; ++yy) {
        const int row = yy * sp.grid_nx;
        if (sleep_i) {  // a sleeping sphere only interacts with awake ones
          bool awake_row = false;
          for (int xx = x0; xx <= x1; ++xx) awake_row = awake_row || cell_awake(s, row + xx);
          if (!awake_row) continue;
        }
        {
          const int m_end = s.cell_start[row + x1 + 1];
          for (int m = s.cell_start[row + x0]; m < m_end; ++m) {
            int j = s.sorted[m];
            if (j == i || (sleep_i && s.sleep[j])) continue;
            float dx = px - s.fpos[0][j], dy = py - s.fpos[1][j], dz = pz - s.fpos[2][j];
            float d2 = dx * dx + dy * dy + dz * dz;
            if (d2 >= r2 * r2) continue;
            float d = sqrtf(d2);
            V3 n = d < 1e-12f ? V3{(j > i) ? 1.f : -1.f, 0.f, 0.f} : V3{dx / d, dy / d, dz / d};
            V3 ri = V3{-.5f * d * n.x, -.5f * d * n.y, -.5f * d * n.z};
            V3 rj = V3{.5f * d * n.x, .5f * d * n.y, .5f * d * n.z};
            V3 wj = V3{s.fang[0][j], s.fang[1][j], s.fang[2][j]};
            V3 a = cross3(wi, ri), b = cross3(wj, rj);
            V3 rel = V3{vi.x + a.x - s.fvel[0][j] - b.x, vi.y + a.y - s.fvel[1][j] - b.y,
                        vi.z + a.z - s.fvel[2][j] - b.z};
            float tinv = 2.f / sp.fm + 2.f * sqr(.5f * d) / I;
            V3 imp = fuel_impulse(sp, n, r2 - d, rel, 2.f / sp.fm, h, tinv, sp.pair_damping);
            dvx += imp.x / sp.fm;
            dvy += imp.y / sp.fm;
            dvz += imp.z / sp.fm;
            V3 tq = cross3(ri, imp);
            dwx += tq.x / I;
            dwy += tq.y / I;
            dwz += tq.z / I;
            ++deg;
          }
        }
      }
    }
    s.dv[0][i] = dvx;
    s.dv[1][i] = dvy;
    s.dv[2][i] = dvz;
    s.dw[0][i] = dwx;
    s.dw[1][i] = dwy;
    s.dw[2][i] = dwz;
    s.degree[i] = (uint8_t)(deg > 255 ? 255 : deg);
    local_max[0] = fmaxf(local_max[0], sqrtf(dvx * dvx + dvy * dvy + dvz * dvz));
    local_max[1] = fmaxf(local_max[1], (float)deg);
  }
  group_sync(g);
  PHASE_MARK_BY(s, 17, g.first);
  group_max<2>(s, local_max, g);
  PHASE_MARK_BY(s, 6, g.first);
  // crowded piles share one Jacobi response scale per world
  const float scale = local_max[1] > 4.f ? fminf(.08f / fmaxf(local_max[0], .08f), 1.f) : 1.f;
  GFOR(k, nwork, g) {
    const int i = s.work[k];
    {
      s.fvel[0][i] += s.dv[0][i] * scale;
      s.fvel[1][i] += s.dv[1][i] * scale;
      s.fvel[2][i] += s.dv[2][i] * scale;
      s.fang[0][i] += s.dw[0][i] * scale;
      s.fang[1][i] += s.dw[1][i] * scale;
      s.fang[2][i] += s.dw[2][i] * scale;
      if (s.degree[i]) s.sleep[i] = 0;
    }
  }
  group_sync(g);
  PHASE_MARK_BY(s, 7, g.first);
}

// ---- island sleep (frc_defense/fuel_physics_sleep.py) ------------------------
// Free spheres that touch (centre distance <= 2r) form islands (union-find,
// roots linked towards the smaller index). An island is stable when one of
// its spheres rests on its support and every sphere is quiet (speed and spin
// under the sleep thresholds, no robot chassis within r + 2 mm below the
// chassis top); a stable island's clock is its members' minimum clock plus
// the substep, an unstable island's is zero, and the whole island sleeps once
// the clock reaches sleep_time. A sleeping island touched by an awake sphere
// merges with it and wakes as a whole. The partition and the per-island
// minimum / flags do not depend on the order of unions, so the GPU and the
// serial host twin decide the same.
AD_HD int uf_find(int* parent, int i) {
#if defined(__CUDA_ARCH__)
  volatile int* p = parent;
  while (true) {
    const int q = p[i];
    if (q == i) return i;
    const int gq = p[q];
    if (gq != q) p[i] = gq;   // path halving: only ever points to an ancestor
    i = q;
  }
#else
  while (parent[i] != i) {
    parent[i] = parent[parent[i]];
    i = parent[i];
  }
  return i;
#endif
}

AD_HD void uf_unite(int* parent, int a, int b) {
  while (true) {
    a = uf_find(parent, a);
    b = uf_find(parent, b);
    if (a == b) return;
    if (a < b) {
      const int t = a;
      a = b;
      b = t;
    }
#if defined(__CUDA_ARCH__)
    if (atomicCAS(&parent[a], a, b) == a) return;
#else
    parent[a] = b;
    return;
#endif
  }
}

AD_HD void island_sleep(TickShared& s, const SimParams& sp, float h) {
  const int P = sp.P;
  // the Jacobi scratch (dv) is dead until the next substep's pair phase
  int* parent = reinterpret_cast<int*>(s.dv[0]);
  int* flags = reinterpret_cast<int*>(s.dv[1]);          // bit 0: a member is not quiet, bit 1: supported
  uint32_t* minclk = reinterpret_cast<uint32_t*>(s.dv[2]);
  const float r2 = 2.f * sp.fr;
  PAR_FOR(i, P) {
    parent[i] = i;
    flags[i] = 0;
    minclk[i] = 0x7f7fffffu;   // FLT_MAX; clocks are non-negative, so their bits order like the values
  }
  BARRIER();
  PAR_FOR(i, P) {
    if (!s.freem[i]) continue;
    const float px = s.fpos[0][i], py = s.fpos[1][i], pz = s.fpos[2][i];
    const float inv_cell = 1.f / sp.grid_cell, reach = r2 + 1e-4f;
    const int x0 = clampi((int)floorf((px - reach) * inv_cell), 0, sp.grid_nx - 1);
    const int x1 = clampi((int)floorf((px + reach) * inv_cell), 0, sp.grid_nx - 1);
    const int y0 = clampi((int)floorf((py - reach) * inv_cell), 0, sp.grid_ny - 1);
    const int y1 = clampi((int)floorf((py + reach) * inv_cell), 0, sp.grid_ny - 1);
    for (int yy = y0; yy <= y1; ++yy) {
      const int row = yy * sp.grid_nx;
      const int m_end = s.cell_start[row + x1 + 1];
      for (int m = s.cell_start[row + x0]; m < m_end; ++m) {
        const int j = s.sorted[m];
        if (j <= i) continue;
        const float d2 = sqr(px - s.fpos[0][j]) + sqr(py - s.fpos[1][j]) + sqr(pz - s.fpos[2][j]);
        if (d2 <= r2 * r2) uf_unite(parent, i, j);
      }
    }
  }
  BARRIER();
  PAR_FOR(i, P) {
    if (!s.freem[i]) continue;
    const bool on_floor = s.fpos[2][i] < s.support[i] + sp.fr + .005f;
    const float svz = s.fvel[2][i] - ((on_floor && !s.sleep[i]) ? sp.fg * h : 0.f);
    const float sv = sqrtf(sqr(s.fvel[0][i]) + sqr(s.fvel[1][i]) + svz * svz);
    const float wn = sqrtf(sqr(s.fang[0][i]) + sqr(s.fang[1][i]) + sqr(s.fang[2][i]));
    bool quiet = sv < sp.sleep_speed && wn < sp.sleep_ang;
    for (int r = 0; r < sp.R && quiet; ++r) {
      const float dx = s.fpos[0][i] - s.pose[r * 3], dy = s.fpos[1][i] - s.pose[r * 3 + 1];
      const float co = s.rtrig[r * 4 + 0], si = s.rtrig[r * 4 + 1];
      float nx, ny, dist;
      box_normal2(co * dx + si * dy, -si * dx + co * dy, .5f * rparam(s, r, RP_LENGTH),
                  .5f * rparam(s, r, RP_WIDTH), nx, ny, dist);
      if (dist <= sp.fr + .002f && s.fpos[2][i] < sp.robot_height + sp.fr) quiet = false;
    }
    const int root = uf_find(parent, i);
    const int bits = (quiet ? 0 : 1) | (on_floor ? 2 : 0);
#if defined(__CUDA_ARCH__)
    if (bits) atomicOr(&flags[root], bits);
    atomicMin(&minclk[root], float_bits(s.clock[i]));
#else
    flags[root] |= bits;
    const uint32_t cb = float_bits(s.clock[i]);
    if (cb < minclk[root]) minclk[root] = cb;
#endif
  }
  BARRIER();
  PAR_FOR(i, P) {
    if (!s.freem[i]) continue;
    const int root = uf_find(parent, i);
    const int f = flags[root];
    const bool stable = (f & 2) && !(f & 1);
    const float elapsed = stable ? float_from_bits(minclk[root]) + h : 0.f;
    const bool asleep = stable && elapsed >= sp.sleep_time;
    s.clock[i] = elapsed;
    s.sleep[i] = asleep ? 1 : 0;
    if (asleep) {
      for (int k = 0; k < 3; ++k) {
        s.fvel[k][i] = 0.f;
        s.fang[k][i] = 0.f;
      }
    }
  }
  BARRIER();
}

// FUEL phases coupled to the robots (chassis contacts with reciprocal robot
// impulses), then terrain / walls / field boxes and sleep; whole CTA.
AD_HD void fuel_post(TickShared& s, const SimParams& sp, float h) {
  const int P = sp.P;
  const float I = .4f * sp.fm * sp.fr * sp.fr;
  float racc[18];
  for (int k = 0; k < 18; ++k) racc[k] = 0.f;
  uint32_t cmask = 0u;
  for (int b0 = 0; b0 < P; b0 += AD_NT) {  // uniform trip count (warp-aggregated push)
    const int i = b0 + AD_TID;
    bool take = false;
    if (i < P && s.freem[i]) {
      for (int r = 0; r < sp.R; ++r) {
        const float* rp = s.pose + r * 3;
        const float* rv = s.vel + r * 3;
        float dx = s.fpos[0][i] - rp[0], dy = s.fpos[1][i] - rp[1];
        if (dx * dx + dy * dy > s.rtrig[r * 4 + 2]) continue;
        const float co = s.rtrig[r * 4 + 0], si = s.rtrig[r * 4 + 1];
        float lx = co * dx + si * dy, ly = -si * dx + co * dy;
        float hl = .5f * rparam(s, r, RP_LENGTH), hw = .5f * rparam(s, r, RP_WIDTH);
        float n2x, n2y, dist;
        box_normal2(lx, ly, hl, hw, n2x, n2y, dist);
        bool valid = dist < sp.fr && s.fpos[2][i] < sp.robot_height + sp.fr;
        if (!valid) continue;
        V3 n = V3{co * n2x - si * n2y, si * n2x + co * n2y, 0.f};
        float armx = s.fpos[0][i] - sp.fr * n.x - rp[0];
        float army = s.fpos[1][i] - sp.fr * n.y - rp[1];
        float rvx = rv[0] + rv[2] * -army, rvy = rv[1] + rv[2] * armx;
        V3 w = V3{s.fang[0][i], s.fang[1][i], s.fang[2][i]};
        V3 arm3 = V3{-sp.fr * n.x, -sp.fr * n.y, 0.f};
        V3 wa = cross3(w, arm3);
        V3 rel = V3{s.fvel[0][i] + wa.x - rvx, s.fvel[1][i] + wa.y - rvy, s.fvel[2][i] + wa.z};
        float mr = rparam(s, r, RP_MASS);
        float Ir = robot_inertia(s, r);
        float cr = armx * n.y - army * n.x;
        float inv = 1.f / sp.fm + 1.f / mr + cr * cr / Ir;
        float rn = dot3(rel, n);
        V3 t = V3{rel.x - rn * n.x, rel.y - rn * n.y, rel.z};
        float tn = fmaxf(norm3(t), 1e-12f);
        float rt = armx * (t.y / tn) - army * (t.x / tn);
        float inv_t = 3.5f / sp.fm + 1.f / mr + rt * rt / Ir;
        V3 imp = fuel_impulse(sp, n, sp.fr - dist, rel, inv, h, inv_t, sp.fc);
        s.fvel[0][i] += imp.x / sp.fm;
        s.fvel[1][i] += imp.y / sp.fm;
        s.fvel[2][i] += imp.z / sp.fm;
        V3 tq = cross3(arm3, imp);
        s.fang[0][i] += tq.x / I;
        s.fang[1][i] += tq.y / I;
        s.fang[2][i] += tq.z / I;
        racc[r * 3 + 0] -= imp.x / mr;
        racc[r * 3 + 1] -= imp.y / mr;
        racc[r * 3 + 2] -= (armx * imp.y - army * imp.x) / Ir;
        cmask |= 1u << r;
        s.sleep[i] = 0;
        if (!s.listed[i]) {
          s.listed[i] = 1;
          take = true;
        }
      }
    }
    push_work(s, i, take);
  }
#if defined(__CUDA_ARCH__)
  cmask = __reduce_or_sync(0xffffffffu, cmask);
  if ((threadIdx.x & 31) == 0 && cmask) atomicOr(&s.cmask, cmask);
#else
  s.cmask = cmask;
#endif
  BARRIER();
  PHASE_MARK(s, 16);
  cmask = s.cmask;
  if (cmask) cta_sum_robots(s, racc, cmask);
  PHASE_MARK(s, 8);
  SERIAL_BEGIN
  for (int r = 0; r < sp.R; ++r) {
    if (!((cmask >> r) & 1u)) continue;
    s.vel[r * 3 + 0] += racc[r * 3 + 0];
    s.vel[r * 3 + 1] += racc[r * 3 + 1];
    s.vel[r * 3 + 2] += racc[r * 3 + 2];
  }
  SERIAL_END
  // terrain, floor, walls, field boxes, sleep, for the awake spheres (all of
  // them are on the work list: awake at binning, or woken by a chassis contact)
  const int nwork = s.nwork;
  PAR_FOR(k, nwork) {
    const int i = s.work[k];
    // a sleeping sphere has zero velocity and takes no static impulse; it
    // stays asleep (its sleep clock is irrelevant once asleep)
    if (!s.sleep[i]) {
      float height, grade;
      bool on = bump_height(sp, s.fpos[0][i], s.fpos[1][i], height, grade);
      V3 n = V3{0.f, 0.f, 1.f};
      if (on && height > 0.f) {
        float inv = 1.f / sqrtf(grade * grade + 1.f);
        n = V3{-grade * inv, 0.f, inv};
      } else {
        height = 0.f;
      }
      s.support[i] = height;
      static_contact_fuel(s, sp, i, n, sp.fr - (s.fpos[2][i] - height) * n.z, true, h);
      static_contact_fuel(s, sp, i, V3{1.f, 0.f, 0.f}, sp.fr - s.fpos[0][i], true, h);
      static_contact_fuel(s, sp, i, V3{-1.f, 0.f, 0.f}, s.fpos[0][i] + sp.fr - sp.field_length, true, h);
      static_contact_fuel(s, sp, i, V3{0.f, 1.f, 0.f}, sp.fr - s.fpos[1][i], true, h);
      static_contact_fuel(s, sp, i, V3{0.f, -1.f, 0.f}, s.fpos[1][i] + sp.fr - sp.field_width, true, h);
      const bool low = s.fpos[2][i] < sp.robot_height + sp.fr;
      for (int b = 0; b < sp.num_boxes && low; ++b) {
        const Box& bx = sp.boxes[b];
        if (fabsf(s.fpos[0][i] - bx.cx) >= bx.hx + sp.fr || fabsf(s.fpos[1][i] - bx.cy) >= bx.hy + sp.fr) continue;
        float nx, ny, dist;
        box_normal2(s.fpos[0][i] - bx.cx, s.fpos[1][i] - bx.cy, bx.hx, bx.hy, nx, ny, dist);
        static_contact_fuel(s, sp, i, V3{nx, ny, 0.f}, sp.fr - dist, low, h);
      }
      // sleep update (per sphere; island mode decides below)
      if (!sp.sleep) {
        s.sleep[i] = 0;
      } else if (!sp.sleep_islands) {
        float sup = s.support[i];
        bool on_floor = s.fpos[2][i] < sup + sp.fr + .005f;
        float svz = s.fvel[2][i] - ((on_floor && !s.sleep[i]) ? sp.fg * h : 0.f);
        float sv = sqrtf(sqr(s.fvel[0][i]) + sqr(s.fvel[1][i]) + svz * svz);
        float wn = sqrtf(sqr(s.fang[0][i]) + sqr(s.fang[1][i]) + sqr(s.fang[2][i]));
        bool quiet = sv < sp.sleep_speed && wn < sp.sleep_ang && on_floor;
        s.clock[i] = quiet ? s.clock[i] + h : 0.f;
        s.sleep[i] = (quiet && s.clock[i] >= sp.sleep_time) ? 1 : 0;
        if (s.sleep[i]) {
          for (int k = 0; k < 3; ++k) {
            s.fvel[k][i] = 0.f;
            s.fang[k][i] = 0.f;
          }
        }
      }
    }
  }
  BARRIER();
  if (sp.sleep && sp.sleep_islands) island_sleep(s, sp, h);
  PHASE_MARK(s, 9);
}

// One physics substep of robots and FUEL. On the GPU (FUEL on, 256-thread
// CTA) warp 0 advances the robots while the remaining warps run the FUEL
// phases that do not read robot state; both groups meet at a CTA barrier
// before the chassis contacts. Every value is produced by the same
// operations in the same order as the serial host sequence.
AD_HD void physics_substep(TickShared& s, const SimParams& sp, World& w, int env, float h) {
#if defined(__CUDA_ARCH__)
  if (sp.fuel_physics && blockDim.x == 256) {
    if (threadIdx.x < 32) {
      robot_substep(s, sp, w, env, h, Group{(int)threadIdx.x, 32, 0, -1});
    } else {
      if (s.prof_on && threadIdx.x == 32) s.prof_last[1] = clock64();
      fuel_pre(s, sp, h, Group{(int)threadIdx.x - 32, 224, 32, 1});
    }
    __syncthreads();
    PHASE_MARK_BY(s, 12, 0);
    PHASE_MARK_BY(s, 13, 32);
    fuel_post(s, sp, h);
    return;
  }
#endif
  robot_substep(s, sp, w, env, h, group_all());
  if (sp.fuel_physics) {
    fuel_pre(s, sp, h, group_all());
    fuel_post(s, sp, h);
  }
}

// Analytic terrain contact height for a ground-spawned sphere
// (frc_defense/fuel_physics.py:180-196).
AD_HD float fuel_spawn_height(const SimParams& sp, float x, float y) {
  const float panel = 0.0127f, rise = 0.16543f - 0.0127f;
  float h = sp.fr;
  for (int b = 0; b < sp.num_bumps; ++b) {
    const Box& bx = sp.bumps[b];
    float dx = x - bx.cx;
    if (fabsf(dx) <= bx.hx && fabsf(y - bx.cy) <= bx.hy) {
      float terrain = panel + rise * (1.f - fabsf(dx) / bx.hx);
      float slope = -sgnf(dx) * rise / bx.hx;
      h = fmaxf(h, terrain + sp.fr * sqrtf(1.f + slope * slope));
    }
  }
  return h;
}

}  // namespace ad
