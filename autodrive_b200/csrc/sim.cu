// Simulation kernels (sm_100a) and their host twins.
//
// Per controller tick the environment runs three stages:
//   control   one CTA per environment; strategic action -> navigation target
//   plan      one CTA per (environment, robot) row on replanning ticks; the
//             whole planning grid stays in shared memory
//   tick      one CTA per environment; command synthesis, every physics
//             substep of robots and FUEL with the state resident in shared
//             memory, odometry, match clock, FUEL actions, perception, rewards
//   sense     one CTA per (environment, robot) row on sensor ticks of the 3v3
//             environment: stereo lenses, angular clustering, stereo fusion
//             and anonymous track association (sense.h)
// plus an optional observe stage (one CTA per environment) that writes the
// 137-feature observation rows.
//
// The host twins run the same __host__ __device__ routines serially per
// environment across OpenMP threads; CPU tests and CPU training use them.
#include "sim.h"
#include "smem_opt_in.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>
#include <thread>

namespace ad {

// ---------------------------------------------------------------------------
// Environment-level routines shared by kernel and host
// ---------------------------------------------------------------------------
AD_HD void count_possession(const World& w, const SimParams& sp, int e, int32_t* poss) {
#if defined(__CUDA_ARCH__)
  if (threadIdx.x < kMaxRobots) poss[threadIdx.x] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < sp.P; i += blockDim.x) {
    int o = w.f_owner[(size_t)e * sp.P + i];
    if (w.f_active[(size_t)e * sp.P + i] && o >= 0 && o < sp.R) atomicAdd(&poss[o], 1);
  }
  __syncthreads();
#else
  for (int r = 0; r < kMaxRobots; ++r) poss[r] = 0;
  for (int i = 0; i < sp.P; ++i) {
    int o = w.f_owner[(size_t)e * sp.P + i];
    if (w.f_active[(size_t)e * sp.P + i] && o >= 0 && o < sp.R) poss[o]++;
  }
#endif
}

AD_HD void control_env(World& w, const SimParams& sp, int e, const int32_t* actions, int32_t* poss,
                        ControlScan& cs) {
  count_possession(w, sp, e, poss);
  G g{w, sp, e};
  PAR_FOR(r, sp.R) {
    if (sp.mode[r] == MODE_DET && sp.role[r] == 0) raster_prepare(g, r);
  }
#if defined(__CUDA_ARCH__)
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int r = warp; r < sp.R; r += nw)
      if (sp.mode[r] != MODE_NONE) control_scan_tracks(g, r, poss, cs, lane, 32);
    __syncthreads();
    for (int r = warp; r < sp.R; r += nw)
      if (sp.mode[r] != MODE_NONE) control_scan_yields(g, r, cs, cs, lane, 32);
    __syncthreads();
  }
#else
  for (int r = 0; r < sp.R; ++r)
    if (sp.mode[r] != MODE_NONE) {
      control_scan_tracks(g, r, poss, cs, 0, 1);
      control_scan_yields(g, r, cs, cs, 0, 1);
    }
#endif
  PAR_FOR(r, sp.R) {
    if (sp.mode[r] != MODE_NONE) control_robot(g, r, actions, poss, cs);
  }
  BARRIER();
  // contour tracing of the robots that collect inside a cluster
#if defined(__CUDA_ARCH__)
  {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int r = warp; r < sp.R; r += nw)
      if (sp.mode[r] != MODE_NONE && cs.edge[r]) control_scan_cloud(g, r, cs, lane, 32);
  }
#else
  for (int r = 0; r < sp.R; ++r)
    if (sp.mode[r] != MODE_NONE && cs.edge[r]) control_scan_cloud(g, r, cs, 0, 1);
#endif
  BARRIER();
  PAR_FOR(r, sp.R) {
    if (sp.mode[r] != MODE_NONE) control_edge_finish(g, r, cs);
  }
  BARRIER();
  SERIAL_BEGIN
  w.g_steps[(size_t)e * 2 + 1] += 1;  // planner tick counter
  SERIAL_END
  BARRIER();
}

AD_HD void observe_env(World& w, const SimParams& sp, int e, int32_t* poss) {
  count_possession(w, sp, e, poss);
  G g{w, sp, e};
  PAR_FOR(r, sp.R) { observe_robot(g, r, poss); }
  BARRIER();
}

AD_HD void load_robots(TickShared& s, const World& w, const SimParams& sp, int e) {
  PAR_FOR(k, sp.R * 3) {
    s.pose[k] = w.r_pose[(size_t)e * sp.R * 3 + k];
    s.vel[k] = w.r_vel[(size_t)e * sp.R * 3 + k];
    s.cmd[k] = w.c_command[(size_t)e * sp.R * 3 + k];
  }
  PAR_FOR(k, sp.R * kNumRobotParams) { s.param[k] = w.r_param[(size_t)e * sp.R * kNumRobotParams + k]; }
  PAR_FOR(k, sp.R * 20) { s.ms[k] = w.m_state[(size_t)e * sp.R * 20 + k]; }
  PAR_FOR(k, sp.R * 4) {
    s.rflag[k] = w.r_flags[(size_t)e * sp.R * 4 + k];
    s.safety[k] = w.r_safety[(size_t)e * sp.R * 4 + k];
  }
  PAR_FOR(k, sp.R) { s.current[k] = w.r_current[(size_t)e * sp.R + k]; }
  SERIAL_BEGIN
  for (int k = 0; k < 3; ++k) s.mu3[k] = w.e_mu[(size_t)e * 3 + k];
  s.eflag[0] = w.e_flags[(size_t)e * 2];
  s.eflag[1] = w.e_flags[(size_t)e * 2 + 1];
  s.substep_index = w.e_substep[e];
  s.phys_time = w.e_phys_time[e];
  SERIAL_END
}

AD_HD void store_robots(const TickShared& s, World& w, const SimParams& sp, int e) {
  PAR_FOR(k, sp.R * 3) {
    w.r_pose[(size_t)e * sp.R * 3 + k] = s.pose[k];
    w.r_vel[(size_t)e * sp.R * 3 + k] = s.vel[k];
  }
  PAR_FOR(k, sp.R * 20) { w.m_state[(size_t)e * sp.R * 20 + k] = s.ms[k]; }
  PAR_FOR(k, sp.R * 4) {
    w.r_flags[(size_t)e * sp.R * 4 + k] = s.rflag[k];
    w.r_safety[(size_t)e * sp.R * 4 + k] = s.safety[k];
  }
  PAR_FOR(k, sp.R) { w.r_current[(size_t)e * sp.R + k] = s.current[k]; }
  SERIAL_BEGIN
  w.e_flags[(size_t)e * 2] = s.eflag[0];
  w.e_flags[(size_t)e * 2 + 1] = s.eflag[1];
  w.e_substep[e] = s.substep_index;
  w.e_phys_time[e] = s.phys_time;
  SERIAL_END
}

AD_HD void load_fuel(TickShared& s, const World& w, const SimParams& sp, int e) {
  const size_t b3 = (size_t)e * 3 * sp.P, b1 = (size_t)e * sp.P;
  PAR_FOR(i, sp.P) {
    for (int k = 0; k < 3; ++k) {
      s.fpos[k][i] = w.f_pos[b3 + (size_t)k * sp.P + i];
      s.fvel[k][i] = w.f_vel[b3 + (size_t)k * sp.P + i];
      s.fang[k][i] = w.f_ang[b3 + (size_t)k * sp.P + i];
    }
    s.clock[i] = w.f_clock[b1 + i];
    s.sleep[i] = w.f_sleep[b1 + i];
    s.freem[i] = (w.f_active[b1 + i] && w.f_owner[b1 + i] < 0) ? 1 : 0;
  }
}

AD_HD void store_fuel(const TickShared& s, World& w, const SimParams& sp, int e) {
  const size_t b3 = (size_t)e * 3 * sp.P, b1 = (size_t)e * sp.P;
  PAR_FOR(i, sp.P) {
    for (int k = 0; k < 3; ++k) {
      w.f_pos[b3 + (size_t)k * sp.P + i] = s.fpos[k][i];
      w.f_vel[b3 + (size_t)k * sp.P + i] = s.fvel[k][i];
      w.f_ang[b3 + (size_t)k * sp.P + i] = s.fang[k][i];
    }
    w.f_clock[b1 + i] = s.clock[i];
    w.f_sleep[b1 + i] = s.sleep[i];
  }
}

// State validation (option `checks`): before a tick uses the world state,
// invalid entries are recorded as bits of the environment's status word
// e_status and made harmless, so a corrupted state is reported instead of
// being indexed with or propagated:
//   1  a FUEL owner outside [-1, robots)     -> owner cleared (free piece)
//   2  a non-finite FUEL position / velocity / spin -> piece deactivated
//   4  an active FUEL piece more than 1 m outside the field or above 20 m -> deactivated
//   8  a non-finite robot pose / velocity / command -> velocity and command
//      zeroed, a non-finite pose replaced by the field centre
constexpr int kStatusOwner = 1, kStatusFuelNonFinite = 2, kStatusFuelEscaped = 4, kStatusRobotNonFinite = 8;

AD_HD bool bad_float(float v) { return (float_bits(v) & 0x7f800000u) == 0x7f800000u; }

AD_HD void validate_state(World& w, const SimParams& sp, int e) {
  int bits = 0;
  const size_t b3 = (size_t)e * 3 * sp.P, b1 = (size_t)e * sp.P;
  PAR_FOR(i, sp.P) {
    const int o = w.f_owner[b1 + i];
    if (o < -1 || o >= sp.R) {
      w.f_owner[b1 + i] = -1;
      bits |= kStatusOwner;
    }
    if (!w.f_active[b1 + i]) continue;
    bool finite = true;
    for (int k = 0; k < 3; ++k) {
      const size_t j = b3 + (size_t)k * sp.P + i;
      finite = finite && !bad_float(w.f_pos[j]) && !bad_float(w.f_vel[j]) && !bad_float(w.f_ang[j]);
    }
    if (!finite) {
      w.f_active[b1 + i] = 0;
      w.f_owner[b1 + i] = -1;
      bits |= kStatusFuelNonFinite;
      continue;
    }
    const float x = w.f_pos[b3 + i], y = w.f_pos[b3 + sp.P + i], z = w.f_pos[b3 + 2 * sp.P + i];
    if (x < -1.f || x > sp.field_length + 1.f || y < -1.f || y > sp.field_width + 1.f || z < -1.f || z > 20.f) {
      w.f_active[b1 + i] = 0;
      w.f_owner[b1 + i] = -1;
      bits |= kStatusFuelEscaped;
    }
  }
  PAR_FOR(r, sp.R) {
    const size_t b = ((size_t)e * sp.R + r) * 3;
    bool bad_pose = false, bad_motion = false;
    for (int k = 0; k < 3; ++k) {
      bad_pose = bad_pose || bad_float(w.r_pose[b + k]);
      bad_motion = bad_motion || bad_float(w.r_vel[b + k]) || bad_float(w.c_command[b + k]);
    }
    if (bad_pose || bad_motion) {
      for (int k = 0; k < 3; ++k) {
        w.r_vel[b + k] = 0.f;
        w.c_command[b + k] = 0.f;
      }
      if (bad_pose) {
        w.r_pose[b] = .5f * sp.field_length;
        w.r_pose[b + 1] = .5f * sp.field_width;
        w.r_pose[b + 2] = 0.f;
      }
      bits |= kStatusRobotNonFinite;
    }
  }
#if defined(__CUDA_ARCH__)
  if (bits) atomicOr(&w.e_status[e], bits);
  __syncthreads();
#else
  w.e_status[e] |= bits;
#endif
}

// Full controller tick for environment e (after control / plan stages).
AD_HD void tick_env(World& w, const SimParams& sp, TickShared& s, int e, uint32_t tick, int32_t* poss,
                    int run_game) {
  G g{w, sp, e};
  const Rng rng{sp.seed0, sp.seed1};
  (void)tick;
  if (sp.checks) validate_state(w, sp, e);
  if (run_game) {
    count_possession(w, sp, e, poss);
    SERIAL_BEGIN
    synthesize_commands(g, poss);
    SERIAL_END
    BARRIER();
  }
  load_robots(s, w, sp, e);
  load_fuel(s, w, sp, e);
  BARRIER();
  // controller-frame velocity before physics (odometry trapezoid) and the
  // poses of uncontrolled robots, which stay parked
  float prior[kMaxRobots * 3];
  float parked[kMaxRobots * 3];
  for (int k = 0; k < sp.R * 3; ++k) {
    prior[k] = s.vel[k];
    parked[k] = s.pose[k];
  }
  const float h = sp.dt / (float)sp.substeps;
  PHASE_MARK(s, 10);
  for (int sub = 0; sub < sp.substeps; ++sub) {
    physics_substep(s, sp, w, e, h);
  }
  SERIAL_BEGIN
  for (int r = 0; r < sp.R; ++r) {
    if (sp.mode[r] == MODE_NONE) {
      for (int k = 0; k < 3; ++k) {
        s.pose[r * 3 + k] = parked[r * 3 + k];
        s.vel[r * 3 + k] = 0.f;
      }
    }
  }
  SERIAL_END
  BARRIER();
  store_robots(s, w, sp, e);
  BARRIER();
  if (!run_game) {
    store_fuel(s, w, sp, e);
    BARRIER();
    return;
  }
  SERIAL_BEGIN
  // wheel/gyro odometry of the policy-visible pose estimate
  for (int r = 0; r < sp.R; ++r) {
    if (sp.mode[r] == MODE_NONE) continue;
    float* est = w.est_pose + g.er(r) * 3;
    float* pol = w.policy_pose + g.er(r) * 3;
    for (int k = 0; k < 2; ++k) est[k] += .5f * (prior[r * 3 + k] + s.vel[r * 3 + k]) * sp.dt;
    float th = est[2] + .5f * (prior[r * 3 + 2] + s.vel[r * 3 + 2]) * sp.dt;
    est[2] = atan2f(sinf(th), cosf(th));
    for (int k = 0; k < 3; ++k) pol[k] = est[k];
    if (sp.mode[r] == MODE_DET && sp.role[r] == 0) raster_finish(g, r);
  }
  w.g_steps[(size_t)e * 2] += 1;
  update_match(w, sp, e);
  SERIAL_END
  BARRIER();
  const int steps = w.g_steps[(size_t)e * 2];
  // counter-based draws keyed by (episode, tick): reproducible under masks and graph replay
  const uint32_t tick_id = ((uint32_t)w.e_episode[e] << 14) ^ (uint32_t)steps;
  fuel_actions(g, s, rng, tick_id);
  invalidate_contact_tracks(g);
  perception_update(g, s, rng, tick_id, (steps % sp.perception_interval) == 0);
  SERIAL_BEGIN
  // rewards
  if (sp.R == 6) {
    float red = 0.f, blue = 0.f;
    for (int r = 0; r < sp.R; ++r) {
      float sc = (float)g.rcount(r, RC_SCORED_EVENT);
      if (sp.team[r] == 0) red += sc;
      else blue += sc;
    }
    for (int r = 0; r < sp.R; ++r) w.g_reward[g.er(r)] = sp.team[r] == 0 ? red - blue : blue - red;
  } else if (sp.counter_defense) {
    // counter-defense: the learner (slot 0) attacks; scores plus a small
    // acquisition bonus and a per-tick cost (frc_defense/tensor_defense_step.py:198-203)
    const float own = (float)g.rcount(0, RC_SCORED_EVENT);
    const float acq = (float)g.rcount(0, RC_ACQUIRED_EVENT);
    w.g_reward[g.er(0)] = own + .05f * acq - .001f;
    w.g_reward[g.er(1)] = -own;
  } else {
    // two-robot defence: the learner (slot 0) is scored against the attacker (slot 1)
    float atk = (float)g.rcount(1, RC_SCORED_EVENT);
    float acq = (float)g.rcount(1, RC_ACQUIRED_EVENT);
    const float* p0 = w.r_pose + g.er(0) * 3;
    const float* p1 = w.r_pose + g.er(1) * 3;
    const float* goal = w.c_target + g.er(1) * 2;
    float rx = goal[0] - p0[0], ry = goal[1] - p0[1];
    float rs = fmaxf(rx * rx + ry * ry, 1e-8f);
    float proj = clampf(((p1[0] - p0[0]) * rx + (p1[1] - p0[1]) * ry) / rs, 0.f, 1.f);
    float cx = p0[0] + proj * rx, cy = p0[1] + proj * ry;
    float lane = sqrtf(sqr(p1[0] - cx) + sqr(p1[1] - cy));
    float score = expf(-lane / .7f) * expf(-sqr((proj - .55f) / .35f));
    w.g_reward[g.er(0)] = -atk - .02f * acq - .001f + .01f * score;
    w.g_reward[g.er(1)] = atk;
  }
  SERIAL_END
  store_fuel(s, w, sp, e);
  BARRIER();
  PHASE_MARK(s, 11);
}

// Sensor update without physics (episode reset): fresh detections only.
AD_HD void perceive_env(World& w, const SimParams& sp, TickShared& s, int e) {
  G g{w, sp, e};
  const Rng rng{sp.seed0, sp.seed1};
  load_fuel(s, w, sp, e);
  BARRIER();
  const uint32_t tick_id = ((uint32_t)w.e_episode[e] << 14) ^ 0x3fffu;
  perception_update(g, s, rng, tick_id, true);
}

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
__global__ void control_kernel(World w, SimParams sp, const int32_t* __restrict__ actions) {
  const int e = blockIdx.x;
  if (e >= sp.n || !w.active[e]) return;
  __shared__ int32_t poss[kMaxRobots];
  __shared__ ControlScan cs;
  control_env(w, sp, e, actions, poss, cs);
}

__global__ void observe_kernel(World w, SimParams sp) {
  const int e = blockIdx.x;
  if (e >= sp.n || !w.active[e]) return;
  __shared__ int32_t poss[kMaxRobots];
  observe_env(w, sp, e, poss);
}

__device__ int g_prof_on = 0;
__device__ unsigned long long g_prof[18];
__device__ unsigned long long g_plan_prof[kPlanPhases];
__device__ unsigned long long g_sense_prof[kSensePhases];

__global__ void __launch_bounds__(256, 3) tick_kernel(World w, SimParams sp, uint32_t tick, int run_game) {
  extern __shared__ __align__(16) uint8_t smem[];
  TickShared& s = *reinterpret_cast<TickShared*>(smem);
  __shared__ int32_t poss[kMaxRobots];
  const int e = blockIdx.x;
  if (e >= sp.n || !w.active[e]) return;
  if (threadIdx.x == 0) {
    s.prof_on = g_prof_on;
    for (int k = 0; k < 18; ++k) s.prof[k] = 0ull;
    s.prof_last[0] = s.prof_last[1] = clock64();
  }
  tick_env(w, sp, s, e, tick, poss, run_game);
  if (threadIdx.x == 0 && s.prof_on)
    for (int k = 0; k < 18; ++k) atomicAdd(&g_prof[k], s.prof[k]);
}

__global__ void __launch_bounds__(512) perceive_kernel(World w, SimParams sp) {
  extern __shared__ __align__(16) uint8_t smem[];
  TickShared& s = *reinterpret_cast<TickShared*>(smem);
  const int e = blockIdx.x;
  if (e >= sp.n || !w.active[e]) return;
  perceive_env(w, sp, s, e);
}

// One CTA per (env, robot) row; rows whose environment has no sensor update
// this tick exit at once.
__global__ void __launch_bounds__(256, 2) sense_kernel(World w, SimParams sp, int force) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int row = blockIdx.x;
  const int e = row / sp.R, r = row % sp.R;
  if (e >= sp.n || !w.active[e] || sp.mode[r] == MODE_NONE) return;
  SenseScratch s;
  sense_carve(smem, sp.P, &s);
  if (threadIdx.x == 0) {
    s.misc[kSenseProfOn] = g_prof_on;
    unsigned long long* acc = reinterpret_cast<unsigned long long*>(s.misc + kSenseProfAcc);
    for (int k = 0; k < kSensePhases; ++k) acc[k] = 0ull;
    acc[kSensePhases] = clock64();
  }
  sense_row(w, sp, s, e, r, force != 0);
  if (threadIdx.x == 0 && s.misc[kSenseProfOn]) {
    const unsigned long long* acc = reinterpret_cast<const unsigned long long*>(s.misc + kSenseProfAcc);
    for (int k = 0; k < kSensePhases; ++k) atomicAdd(&g_sense_prof[k], acc[k]);
  }
}

// One CTA per (env, robot) row; rows not due for replanning exit at once.
__global__ void plan_kernel(World w, SimParams sp, int force) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int row = blockIdx.x;
  const int e = row / sp.R, r = row % sp.R;
  if (e >= sp.n || !w.active[e] || sp.mode[r] == MODE_NONE) return;
  const int ticks = w.g_steps[(size_t)e * 2 + 1];
  if (!force && (ticks % sp.replan_interval) != 0) return;
  const int nc = sp.plan_nx * sp.plan_ny;
  PlanScratch ps;
  float* f = reinterpret_cast<float*>(smem);
  const int cap = plan_lattice_cap(sp);
  ps.value = f;
  ps.path = f + nc;
  ps.tmp = ps.path + cap * 2;
  ps.misc = reinterpret_cast<int*>(ps.tmp + cap * 2 + 4);
  ps.moves = reinterpret_cast<uint16_t*>(ps.misc + 8);
  ps.blocked = reinterpret_cast<uint8_t*>(ps.moves + nc);
  __shared__ PlanRequest q;
  __shared__ unsigned long long s_best[2];
  __shared__ unsigned long long s_prof[kPlanPhases + 1];
  ps.best = s_best;
  const bool prof = g_prof_on != 0;
  ps.prof = prof ? s_prof : nullptr;
  if (threadIdx.x == 0) {
    q = make_plan_request(w, sp, e, r);
    if (prof) {
      for (int k = 0; k < kPlanPhases; ++k) s_prof[k] = 0ull;
      s_prof[kPlanPhases] = clock64();
    }
  }
  __syncthreads();
  plan_route(w, sp, e, r, q, ps);
  if (prof && threadIdx.x == 0)
    for (int k = 0; k < kPlanPhases; ++k) atomicAdd(&g_plan_prof[k], s_prof[k]);
}

// Fuel-only microbenchmark kernel: `ticks` ticks of robot + FUEL substeps
// with the state resident in shared memory between ticks.
__global__ void __launch_bounds__(256, 3) physics_kernel(World w, SimParams sp, int ticks) {
  extern __shared__ __align__(16) uint8_t smem[];
  TickShared& s = *reinterpret_cast<TickShared*>(smem);
  const int e = blockIdx.x;
  if (e >= sp.n || !w.active[e]) return;
  load_robots(s, w, sp, e);
  load_fuel(s, w, sp, e);
  __syncthreads();
  const float h = sp.dt / (float)sp.substeps;
  for (int t = 0; t < ticks; ++t)
    for (int sub = 0; sub < sp.substeps; ++sub) {
      physics_substep(s, sp, w, e, h);
    }
  __syncthreads();
  store_robots(s, w, sp, e);
  store_fuel(s, w, sp, e);
}

// ---------------------------------------------------------------------------
// Launchers
// ---------------------------------------------------------------------------
static void check(cudaError_t err, const char* what) {
  if (err != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
}

size_t tick_smem_bytes() { return sizeof(TickShared); }

void phase_profile_enable(bool on) {
  const int v = on ? 1 : 0;
  check(cudaMemcpyToSymbol(g_prof_on, &v, sizeof(int)), "phase profile flag");
}

std::vector<unsigned long long> phase_profile_read() {
  std::vector<unsigned long long> out(18, 0ull);
  check(cudaMemcpyFromSymbol(out.data(), g_prof, sizeof(unsigned long long) * 18), "phase profile read");
  std::vector<unsigned long long> zero(18, 0ull);
  check(cudaMemcpyToSymbol(g_prof, zero.data(), sizeof(unsigned long long) * 18), "phase profile reset");
  return out;
}

std::vector<unsigned long long> plan_profile_read() {
  std::vector<unsigned long long> out(kPlanPhases, 0ull);
  check(cudaMemcpyFromSymbol(out.data(), g_plan_prof, sizeof(unsigned long long) * kPlanPhases),
        "plan profile read");
  std::vector<unsigned long long> zero(kPlanPhases, 0ull);
  check(cudaMemcpyToSymbol(g_plan_prof, zero.data(), sizeof(unsigned long long) * kPlanPhases),
        "plan profile reset");
  return out;
}

std::vector<unsigned long long> sense_profile_read() {
  std::vector<unsigned long long> out(kSensePhases, 0ull);
  check(cudaMemcpyFromSymbol(out.data(), g_sense_prof, sizeof(unsigned long long) * kSensePhases),
        "sense profile read");
  std::vector<unsigned long long> zero(kSensePhases, 0ull);
  check(cudaMemcpyToSymbol(g_sense_prof, zero.data(), sizeof(unsigned long long) * kSensePhases),
        "sense profile reset");
  return out;
}

size_t plan_smem_bytes(const SimParams& sp) {
  const int nc = sp.plan_nx * sp.plan_ny;
  return (size_t)(nc + plan_lattice_cap(sp) * 4 + 4) * sizeof(float) + 8 * sizeof(int) + (size_t)nc * 3 + 16;
}

void validate_params(const SimParams& sp) {
  if (sp.R < 2 || sp.R > kMaxRobots) throw std::runtime_error("robot count must be 2..6");
  if (sp.P < 1 || sp.P > kMaxPieces) throw std::runtime_error("piece count must be 1..640");
  if (sp.grid_nx * sp.grid_ny > kMaxGridCells) throw std::runtime_error("FUEL grid exceeds 4096 cells");
  if (sp.grid_cell < 2.f * sp.fr) throw std::runtime_error("FUEL grid cell must be >= sphere diameter");
  if (sp.num_boxes > kMaxBoxes || sp.num_bumps > kMaxBumps) throw std::runtime_error("too many field boxes");
  if (sp.substeps < 1) throw std::runtime_error("substeps must be positive");
}

void launch_control(const World& w, const SimParams& sp, const int32_t* actions, cudaStream_t st) {
  control_kernel<<<sp.n, 128, 0, st>>>(w, sp, actions);
  check(cudaGetLastError(), "control_kernel");
}

void launch_plan(const World& w, const SimParams& sp, int force, cudaStream_t st) {
  size_t smem = plan_smem_bytes(sp);
  static size_t configured[dynsmem::kMaxDevices] = {};
  check(dynsmem::opt_in(plan_kernel, smem, configured), "plan_kernel smem attribute");
  plan_kernel<<<sp.n * sp.R, 256, smem, st>>>(w, sp, force);
  check(cudaGetLastError(), "plan_kernel");
}

size_t sense_smem_bytes(const SimParams& sp) { return sense_carve(nullptr, sp.P, nullptr); }

void launch_sense(const World& w, const SimParams& sp, int force, cudaStream_t st) {
  const size_t smem = sense_smem_bytes(sp);
  static size_t configured[dynsmem::kMaxDevices] = {};
  check(dynsmem::opt_in(sense_kernel, smem, configured), "sense_kernel smem attribute");
  sense_kernel<<<sp.n * sp.R, 256, smem, st>>>(w, sp, force);
  check(cudaGetLastError(), "sense_kernel");
}

void launch_tick(const World& w, const SimParams& sp, uint32_t tick, int run_game, int threads, cudaStream_t st) {
  static size_t tick_done[dynsmem::kMaxDevices] = {}, physics_done[dynsmem::kMaxDevices] = {},
                perceive_done[dynsmem::kMaxDevices] = {};
  const size_t smem = tick_smem_bytes();
  check(dynsmem::opt_in(tick_kernel, smem, tick_done), "tick_kernel smem attribute");
  check(dynsmem::opt_in(physics_kernel, smem, physics_done), "physics_kernel smem attribute");
  check(dynsmem::opt_in(perceive_kernel, smem, perceive_done), "perceive_kernel smem attribute");
  if (run_game < 0) return;
  tick_kernel<<<sp.n, threads, smem, st>>>(w, sp, tick, run_game);
  check(cudaGetLastError(), "tick_kernel");
}

void launch_physics(const World& w, const SimParams& sp, int ticks, int threads, cudaStream_t st) {
  launch_tick(w, sp, 0, 0, threads, st);  // ensures attributes; runs one physics-only tick
  physics_kernel<<<sp.n, threads, tick_smem_bytes(), st>>>(w, sp, ticks - 1 > 0 ? ticks - 1 : 0);
  check(cudaGetLastError(), "physics_kernel");
}

void launch_perceive(const World& w, const SimParams& sp, int threads, cudaStream_t st) {
  launch_tick(w, sp, 0, -1, threads, st);  // attribute setup only (run_game < 0 launches nothing)
  perceive_kernel<<<sp.n, threads, tick_smem_bytes(), st>>>(w, sp);
  check(cudaGetLastError(), "perceive_kernel");
}

void launch_observe(const World& w, const SimParams& sp, cudaStream_t st) {
  observe_kernel<<<sp.n, 64, 0, st>>>(w, sp);
  check(cudaGetLastError(), "observe_kernel");
}

// ---------------------------------------------------------------------------
// Host twins
// ---------------------------------------------------------------------------

// Run fn(worker, begin, end) over [0, n) on up to hardware_concurrency threads.
template <typename F>
static void host_parallel(int n, F fn) {
  int workers = (int)std::thread::hardware_concurrency();
  workers = workers < 1 ? 1 : (workers > 64 ? 64 : workers);
  workers = workers > n ? (n > 0 ? n : 1) : workers;
  if (workers <= 1) {
    fn(0, 0, n);
    return;
  }
  std::vector<std::thread> pool;
  int chunk = (n + workers - 1) / workers;
  for (int t = 0; t < workers; ++t) {
    int b = t * chunk, e = b + chunk > n ? n : b + chunk;
    if (b >= e) break;
    pool.emplace_back([=, &fn] { fn(t, b, e); });
  }
  for (auto& th : pool) th.join();
}
void host_control(World w, const SimParams& sp, const int32_t* actions) {
  host_parallel(sp.n, [&](int, int b, int end) {
    for (int e = b; e < end; ++e) {
      if (!w.active[e]) continue;
      int32_t poss[kMaxRobots];
      ControlScan cs;
      control_env(w, sp, e, actions, poss, cs);
    }
  });
}

void host_plan(World w, const SimParams& sp, int force) {
  const int nc = sp.plan_nx * sp.plan_ny;
  host_parallel(sp.n * sp.R, [&](int, int b, int end) {
    const int cap = plan_lattice_cap(sp);
    std::vector<float> fbuf(nc + cap * 4 + 4);
    std::vector<uint8_t> blocked(nc);
    std::vector<uint16_t> moves(nc);
    int misc[8];
    unsigned long long best[2];
    PlanScratch ps{blocked.data(), moves.data(), fbuf.data(), fbuf.data() + nc, fbuf.data() + nc + cap * 2, misc,
                   best, nullptr};
    for (int row = b; row < end; ++row) {
      const int e = row / sp.R, r = row % sp.R;
      if (!w.active[e] || sp.mode[r] == MODE_NONE) continue;
      const int ticks = w.g_steps[(size_t)e * 2 + 1];
      if (!force && (ticks % sp.replan_interval) != 0) continue;
      PlanRequest q = make_plan_request(w, sp, e, r);
      plan_route(w, sp, e, r, q, ps);
    }
  });
}

void host_sense(World w, const SimParams& sp, int force) {
  host_parallel(sp.n * sp.R, [&](int, int b, int end) {
    std::vector<uint8_t> buf(sense_smem_bytes(sp) + 16);
    SenseScratch s;
    sense_carve(buf.data(), sp.P, &s);
    for (int row = b; row < end; ++row) {
      const int e = row / sp.R, r = row % sp.R;
      if (!w.active[e] || sp.mode[r] == MODE_NONE) continue;
      sense_row(w, sp, s, e, r, force != 0);
    }
  });
}

void host_tick(World w, const SimParams& sp, uint32_t tick, int run_game) {
  host_parallel(sp.n, [&](int, int b, int end) {
    std::vector<uint8_t> buf(sizeof(TickShared) + 16);
    TickShared* s = reinterpret_cast<TickShared*>(buf.data());
    for (int e = b; e < end; ++e) {
      if (!w.active[e]) continue;
      int32_t poss[kMaxRobots];
      tick_env(w, sp, *s, e, tick, poss, run_game);
    }
  });
}

void host_physics(World w, const SimParams& sp, int ticks) {
  for (int t = 0; t < ticks; ++t) host_tick(w, sp, 0, 0);
}

void host_perceive(World w, const SimParams& sp) {
  host_parallel(sp.n, [&](int, int b, int end) {
    std::vector<uint8_t> buf(sizeof(TickShared) + 16);
    TickShared* s = reinterpret_cast<TickShared*>(buf.data());
    for (int e = b; e < end; ++e) {
      if (!w.active[e]) continue;
      perceive_env(w, sp, *s, e);
    }
  });
}

void host_observe(World w, const SimParams& sp) {
  host_parallel(sp.n, [&](int, int b, int end) {
    for (int e = b; e < end; ++e) {
      if (!w.active[e]) continue;
      int32_t poss[kMaxRobots];
      observe_env(w, sp, e, poss);
    }
  });
}

}  // namespace ad
