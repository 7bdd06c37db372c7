// Environment state schema and simulation parameters.
//
// All per-environment state lives in torch tensors owned by Python. The schema
// below is the single source of truth: Python asks the extension for the list
// of (name, dtype, shape) entries, allocates one tensor per entry, and hands
// the list back once; the extension then keeps a struct of raw pointers (the
// World) that every kernel and host routine reads.
//
// Layout rules: the environment index is always the leading dimension; FUEL
// arrays are structure-of-arrays per environment ([N][3][P] for vectors) so a
// CTA that owns one environment reads each component with coalesced loads.
#pragma once

#include "common.h"

namespace ad {

constexpr int kMaxRobots = 6;
constexpr int kMaxPairs = 15;
constexpr int kMaxPieces = 640;
constexpr int kPathPoints = 72;
constexpr int kMaxBoxes = 16;
constexpr int kMaxBumps = 4;
constexpr int kObsDim = 137;
constexpr int kNumRobotParams = 14;
constexpr int kRasterPoints = 256;   // samples of each robot's closed raster route

// Robot parameter columns in r_param.
enum RobotParam : int {
  RP_LENGTH = 0, RP_WIDTH, RP_MASS, RP_SPEED, RP_ACCEL, RP_OMEGA, RP_ALPHA,
  RP_DRIVE_RATIO, RP_DRIVE_CURRENT, RP_DRIVE_SUPPLY, RP_ROBOT_SUPPLY,
  RP_BATTERY_R, RP_LATERAL_MU, RP_YAW_INERTIA,
};

// Module state rows in m_state [N][R][5][4].
enum ModuleRow : int { MS_ANGLE = 0, MS_STEER_RATE, MS_DRIVE_SPEED, MS_CURRENT, MS_SUPPLY };

// Robot flags [N][R][4].
enum RobotFlag : int { RF_ROBOT_CONTACT = 0, RF_FIELD_CONTACT, RF_WALL_X, RF_WALL_Y };

// Per-robot game counters [N][R][6].
enum RobotCount : int {
  RC_ACQUIRED_TOTAL = 0, RC_DENIED_TOTAL, RC_ACQUIRED_EVENT, RC_SCORED_EVENT,
  RC_PASSED_EVENT, RC_DENIED_EVENT,
};

// Per-robot game timers [N][R][3].
enum RobotTimer : int { RT_NEXT_INTAKE = 0, RT_NEXT_SCORE, RT_NEXT_FERRY };

// Per-robot latches [N][R][kLatches].
constexpr int kLatches = 16;
enum RobotLatch : int {
  RL_FERRY_COMMITTED = 0, RL_SCORE_COMMITTED, RL_LAST_HUB_ZONE, RL_INTAKE_COLLECTING,
  RL_SCORE_INTENT, RL_TARGET_COLLECTING, RL_NO_TRACK_SEARCH, RL_STATIC_OPPONENT,
  RL_RASTER_SWEEP,  // the raster cursor follows this robot after the tick
};

// dtype codes shared with Python.
enum DType : int { DT_F32 = 0, DT_I32 = 1, DT_U8 = 2, DT_I8 = 3, DT_F64 = 4 };

// X(name, ctype, dtype, rank, d0, d1, d2, d3) with symbolic dims
// N envs, R robots, P pieces, Q robot pairs, K path points, O obs dim.
#define AD_WORLD_FIELDS(X)                                              \
  X(r_pose, float, DT_F32, 3, N, R, 3, 1)                               \
  X(r_vel, float, DT_F32, 3, N, R, 3, 1)                                \
  X(r_param, float, DT_F32, 3, N, R, kNumRobotParams, 1)                \
  X(e_mu, float, DT_F32, 2, N, 3, 1, 1)                                 \
  X(m_state, float, DT_F32, 4, N, R, 5, 4)                              \
  X(r_current, float, DT_F32, 2, N, R, 1, 1)                            \
  X(r_flags, uint8_t, DT_U8, 3, N, R, 4, 1)                             \
  X(e_flags, uint8_t, DT_U8, 2, N, 2, 1, 1)                             \
  X(r_safety, int32_t, DT_I32, 3, N, R, 4, 1)                           \
  X(pair_count, int32_t, DT_I32, 3, N, Q, 2, 1)                         \
  X(pair_substep, int32_t, DT_I32, 3, N, Q, 2, 1)                       \
  X(pair_time, float, DT_F32, 3, N, Q, 2, 1)                            \
  X(pair_impulse, float, DT_F32, 3, N, Q, 4, 1)                         \
  X(e_substep, int32_t, DT_I32, 1, N, 1, 1, 1)                          \
  X(e_phys_time, double, DT_F64, 1, N, 1, 1, 1)                         \
  X(f_pos, float, DT_F32, 3, N, 3, P, 1)                                \
  X(f_vel, float, DT_F32, 3, N, 3, P, 1)                                \
  X(f_ang, float, DT_F32, 3, N, 3, P, 1)                                \
  X(f_clock, float, DT_F32, 2, N, P, 1, 1)                              \
  X(f_sleep, uint8_t, DT_U8, 2, N, P, 1, 1)                             \
  X(f_active, uint8_t, DT_U8, 2, N, P, 1, 1)                            \
  X(f_owner, int8_t, DT_I8, 2, N, P, 1, 1)                              \
  X(f_zone, int8_t, DT_I8, 2, N, P, 1, 1)                               \
  X(g_time, float, DT_F32, 2, N, 2, 1, 1)                               \
  X(g_steps, int32_t, DT_I32, 2, N, 2, 1, 1)                            \
  X(g_hub, uint8_t, DT_U8, 2, N, 2, 1, 1)                               \
  X(g_scores, int32_t, DT_I32, 2, N, 4, 1, 1)                           \
  X(g_first_inactive, int32_t, DT_I32, 1, N, 1, 1, 1)                   \
  X(g_rcount, int32_t, DT_I32, 3, N, R, 6, 1)                           \
  X(g_rtime, float, DT_F32, 3, N, R, 3, 1)                              \
  X(g_rlatch, uint8_t, DT_U8, 3, N, R, 16, 1)                          \
  X(g_action, int32_t, DT_I32, 2, N, R, 1, 1)                           \
  X(g_reward, float, DT_F32, 2, N, R, 1, 1)                             \
  X(c_target, float, DT_F32, 3, N, R, 2, 1)                             \
  X(c_fuel_target, float, DT_F32, 3, N, R, 2, 1)                        \
  X(c_fuel_delta, float, DT_F32, 3, N, R, 2, 1)                         \
  X(c_target_index, int32_t, DT_I32, 2, N, R, 1, 1)                     \
  X(c_collect_heading, float, DT_F32, 2, N, R, 1, 1)                    \
  X(c_empty_ticks, int32_t, DT_I32, 2, N, R, 1, 1)                      \
  X(c_raster, int32_t, DT_I32, 2, N, R, 1, 1)  /* raster cursor + 1; 0: re-anchor */ \
  X(raster_pts, float, DT_F32, 3, R, S, 2, 1)                           \
  X(c_avoid, int32_t, DT_I32, 2, N, Q, 1, 1)                            \
  X(c_command, float, DT_F32, 3, N, R, 3, 1)                            \
  X(c_cand, int32_t, DT_I32, 3, N, R, 4, 1)                             \
  X(est_pose, float, DT_F32, 3, N, R, 3, 1)                             \
  X(policy_pose, float, DT_F32, 3, N, R, 3, 1)                          \
  X(t_pos, float, DT_F32, 4, N, R, 2, P)                                \
  X(t_vel, float, DT_F32, 4, N, R, 2, P)                                \
  X(t_age, float, DT_F32, 3, N, R, P, 1)                                \
  X(t_conf, float, DT_F32, 3, N, R, P, 1)                               \
  X(t_quality, float, DT_F32, 3, N, R, P, 1)                            \
  X(t_mask, uint8_t, DT_U8, 3, N, R, P, 1)                              \
  X(t_spatial, float, DT_F32, 4, N, R, 2, P)                            \
  X(t_angular, float, DT_F32, 3, N, R, P, 1)                            \
  X(t_merged, uint8_t, DT_U8, 3, N, R, P, 1)                            \
  X(t_visible, uint8_t, DT_U8, 3, N, R, P, 1)                           \
  X(o_pose, float, DT_F32, 3, N, R, 3, 1)                               \
  X(o_vel, float, DT_F32, 3, N, R, 3, 1)                                \
  X(o_size, float, DT_F32, 3, N, R, 3, 1)                               \
  X(o_age, float, DT_F32, 2, N, R, 1, 1)                                \
  X(o_valid, uint8_t, DT_U8, 2, N, R, 1, 1)                             \
  X(p_path, float, DT_F32, 4, N, R, K, 2)                               \
  X(p_profile, float, DT_F32, 3, N, R, K, 1)                            \
  X(p_len, int32_t, DT_I32, 2, N, R, 1, 1)                              \
  X(p_goal, float, DT_F32, 3, N, R, 2, 1)                               \
  X(p_start, float, DT_F32, 3, N, R, 2, 1)                              \
  X(p_heading, float, DT_F32, 2, N, R, 1, 1)                            \
  X(p_progress, float, DT_F32, 2, N, R, 1, 1)                           \
  X(p_trench, uint8_t, DT_U8, 2, N, R, 1, 1)                            \
  X(p_sweeps, int32_t, DT_I32, 2, N, R, 1, 1)                           \
  X(obs, float, DT_F32, 3, N, R, O, 1)                                  \
  X(e_episode, int32_t, DT_I32, 1, N, 1, 1, 1)                         \
  X(e_status, int32_t, DT_I32, 1, N, 1, 1, 1)                          \
  X(active, uint8_t, DT_U8, 1, N, 1, 1, 1)

struct World {
#define AD_DECL(name, ctype, dt, rank, a, b, c, d) ctype* name = nullptr;
  AD_WORLD_FIELDS(AD_DECL)
#undef AD_DECL
};

// Static box for collisions / geometry: centre and half extents.
struct Box { float cx, cy, hx, hy; };

// Everything that is uniform across environments. Passed by value to kernels
// (it fits in the 32 KB parameter space) and shared by the host path.
struct SimParams {
  int n = 0, R = 6, P = 504, Q = 15;
  int substeps = 64;            // physics substeps per controller tick
  int contact_iterations = 3;
  int sweep_steps = 1;          // field sweep increments per substep
  float dt = 0.02f;             // controller tick
  float field_length = 16.54f, field_width = 8.07f;
  float alliance_depth = 4.02844f;
  int num_boxes = 0, num_bumps = 0;
  Box boxes[kMaxBoxes];          // solid colliders
  Box bumps[kMaxBumps];          // bump ramps
  float hub_x[2], hub_y[2];
  int team[kMaxRobots];
  int mode[kMaxRobots];          // 0 none, 1 nn, 2 deterministic
  int role[kMaxRobots];          // 0 offense, 1 defense
  int kind[kMaxRobots];          // 0 dumper, 1 turret
  int capacity[kMaxRobots];
  float score_interval[kMaxRobots];
  int pair_i[kMaxPairs], pair_j[kMaxPairs];
  // swerve drivetrain constants
  float wheel_radius = .0508f, steer_current_limit = 20.f, steer_rate_limit = 12.f;
  float steer_acceleration = 80.f, motor_efficiency = .9f, battery_voltage = 12.6f;
  float stall_torque = 7.09f, stall_current = 366.f, free_speed_rpm = 6000.f;
  float free_current = 2.f, nominal_voltage = 12.f, module_x = .36f, module_y = .36f;
  // fuel physics
  int fuel_physics = 1;         // 0: static FUEL (no contact dynamics)
  float fr = .075f, fm = .215f, fk = 2000.f, fc = 40.f, fmu = .45f, froll = .20f, fg = 9.81f;
  float robot_height = .5f, max_comp = .5f;
  float pair_damping = 160.f;
  int sleep = 1;
  int sleep_islands = 0;         // 1: whole contact islands sleep and wake together
  float sleep_time = .5f, sleep_speed = .025f, sleep_ang = .5f;
  float grid_cell = .2f;
  int grid_nx = 83, grid_ny = 41;
  int colored_solver = 0;       // 0: Jacobi (owner computes), 1: two-colour sequential
  // game rules
  float fuel_radius_rules = .0825f;   // intake/track geometry radius
  int two_robot_schedule = 0;   // 0: 3v3 REBUILT shifts; 1: two-robot 20 s + 30 s alternation
  int counter_defense = 0;      // two-robot task: 1 = slot 0 attacks (learner), slot 1 defends (scripted)
  int opponent_kind = 0;        // two-robot attacker: 0 offense/adstar, 1 mirror, 2 cutoff,
                                // 3 velocity_intercept, 4 random
  int perception_interval = 2;
  float perception_range = 6.f, perception_fov = 1.0471976f;  // half FOV (rad)
  float perception_dropout = .02f, position_noise = .015f, velocity_noise = .05f;
  float track_timeout = 2.f, ball_diameter = .15f, stereo_baseline = .0635f;
  int stereo_tracks = 0;        // 1: anonymous stereo-cluster FUEL tracks; 0: per-piece tracks
  int sweeping = 0;             // scripted offense collects along its raster route
  int raster_lookahead = 20;    // raster route samples ahead of the cursor
  int num_depots = 0;
  Box depots[2];                // open-floor depot footprints (red, blue)
  int replan_interval = 20;
  int teammate_coordination = 0;
  int normalize_obs = 1;
  int horizon = 8000;
  int checks = 0;               // 1: validate and sanitise the world state every tick (status word e_status)
  float max_speed_nominal = 9.6f, max_omega_nominal = 16.f;
  // planner grid
  float plan_res = .3f;
  int plan_nx = 56, plan_ny = 27, plan_sweeps = 72;
  float bump_cost = .12f;
  // random numbers
  uint32_t seed0 = 0, seed1 = 0;
};

}  // namespace ad
