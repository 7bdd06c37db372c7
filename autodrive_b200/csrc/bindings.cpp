// Python bindings of the simulator extension.
//
// `schema(n, R, P)` tells Python which state tensors to allocate; `Sim` binds
// one list of those tensors to the kernels. CUDA tensors run the sm_100a
// kernels on the current torch stream; CPU tensors run the host twins. There
// is no fallback between the two: a CUDA world never runs host code.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include <string>
#include <vector>

#include "sim.h"

namespace py = pybind11;
using namespace ad;

namespace {

int64_t dim_value(const std::string& sym, int64_t N, int64_t R, int64_t P) {
  if (sym == "N") return N;
  if (sym == "R") return R;
  if (sym == "P") return P;
  if (sym == "Q") return R * (R - 1) / 2;
  if (sym == "K") return kPathPoints;
  if (sym == "O") return kObsDim;
  if (sym == "S") return kRasterPoints;
  if (sym == "kNumRobotParams") return kNumRobotParams;
  return std::stoll(sym);
}

py::list schema(int64_t N, int64_t R, int64_t P) {
  py::list out;
#define AD_SCHEMA(name, ctype, dt, rank, a, b, c, d)                                      \
  {                                                                                       \
    std::vector<int64_t> shape;                                                           \
    const char* syms[4] = {#a, #b, #c, #d};                                               \
    for (int k = 0; k < rank; ++k) shape.push_back(dim_value(syms[k], N, R, P));          \
    out.append(py::make_tuple(std::string(#name), (int)dt, shape));                       \
  }
  AD_WORLD_FIELDS(AD_SCHEMA)
#undef AD_SCHEMA
  return out;
}

template <typename T>
void set_if(const py::dict& d, const char* key, T& dst) {
  if (d.contains(key)) dst = d[key].cast<T>();
}

template <typename T>
void set_array(const py::dict& d, const char* key, T* dst, int max_len, int* count = nullptr) {
  if (!d.contains(key)) return;
  auto values = d[key].cast<std::vector<T>>();
  if ((int)values.size() > max_len) throw std::runtime_error(std::string(key) + " has too many entries");
  for (size_t k = 0; k < values.size(); ++k) dst[k] = values[k];
  if (count) *count = (int)values.size();
}

void set_boxes(const py::dict& d, const char* key, Box* dst, int max_len, int& count) {
  if (!d.contains(key)) return;
  auto rows = d[key].cast<std::vector<std::vector<float>>>();
  if ((int)rows.size() > max_len) throw std::runtime_error(std::string(key) + " has too many boxes");
  for (size_t k = 0; k < rows.size(); ++k) {
    if (rows[k].size() != 4) throw std::runtime_error("boxes are (cx, cy, hx, hy)");
    dst[k] = Box{rows[k][0], rows[k][1], rows[k][2], rows[k][3]};
  }
  count = (int)rows.size();
}

SimParams params_from_dict(const py::dict& d) {
  SimParams p;
#define I(k) set_if(d, #k, p.k);
  I(n) I(R) I(P) I(substeps) I(contact_iterations) I(sweep_steps) I(dt) I(field_length) I(field_width)
  I(alliance_depth) I(wheel_radius) I(steer_current_limit) I(steer_rate_limit) I(steer_acceleration)
  I(motor_efficiency) I(battery_voltage) I(stall_torque) I(stall_current) I(free_speed_rpm) I(free_current)
  I(nominal_voltage) I(module_x) I(module_y) I(fuel_physics) I(fr) I(fm) I(fk) I(fc) I(fmu) I(froll) I(fg)
  I(robot_height) I(max_comp) I(pair_damping) I(sleep) I(sleep_islands) I(sleep_time) I(sleep_speed) I(sleep_ang)
  I(grid_cell) I(grid_nx) I(grid_ny) I(colored_solver) I(fuel_radius_rules) I(two_robot_schedule) I(counter_defense)
  I(perception_interval) I(opponent_kind) I(perception_range) I(perception_fov) I(perception_dropout) I(position_noise)
  I(velocity_noise) I(track_timeout) I(ball_diameter) I(stereo_baseline) I(stereo_tracks) I(sweeping) I(raster_lookahead) I(replan_interval)
  I(teammate_coordination) I(normalize_obs) I(horizon) I(checks) I(max_speed_nominal) I(max_omega_nominal)
  I(plan_res) I(plan_nx) I(plan_ny) I(plan_sweeps) I(bump_cost) I(seed0) I(seed1)
#undef I
  p.Q = p.R * (p.R - 1) / 2;
  set_boxes(d, "boxes", p.boxes, kMaxBoxes, p.num_boxes);
  set_boxes(d, "bumps", p.bumps, kMaxBumps, p.num_bumps);
  set_boxes(d, "depots", p.depots, 2, p.num_depots);
  set_array(d, "hub_x", p.hub_x, 2);
  set_array(d, "hub_y", p.hub_y, 2);
  set_array(d, "team", p.team, kMaxRobots);
  set_array(d, "mode", p.mode, kMaxRobots);
  set_array(d, "role", p.role, kMaxRobots);
  set_array(d, "kind", p.kind, kMaxRobots);
  set_array(d, "capacity", p.capacity, kMaxRobots);
  set_array(d, "score_interval", p.score_interval, kMaxRobots);
  int q = 0;
  for (int i = 0; i < p.R; ++i)
    for (int j = i + 1; j < p.R; ++j) {
      p.pair_i[q] = i;
      p.pair_j[q] = j;
      ++q;
    }
  validate_params(p);
  return p;
}

struct Sim {
  World w;
  SimParams sp;
  std::vector<torch::Tensor> keep;
  bool cuda = false;
  int threads = 256;
  bool sense_in_tick = true;  // run the stereo sensor stage right after each game tick

  Sim(std::vector<torch::Tensor> tensors, py::dict params) {
    sp = params_from_dict(params);
    py::list sch = schema(sp.n, sp.R, sp.P);
    if ((size_t)py::len(sch) != tensors.size()) throw std::runtime_error("state tensor count mismatch");
    keep = tensors;
    cuda = tensors[0].is_cuda();
    size_t k = 0;
#define AD_BIND(name, ctype, dt, rank, a, b, c, d)                                                 \
    {                                                                                              \
      auto& t = tensors[k];                                                                        \
      auto entry = sch[k].cast<py::tuple>();                                                       \
      auto shape = entry[2].cast<std::vector<int64_t>>();                                          \
      if (!t.is_contiguous()) throw std::runtime_error(std::string(#name) + " must be contiguous"); \
      if (t.is_cuda() != cuda) throw std::runtime_error(std::string(#name) + " is on another device"); \
      if (t.sizes().vec() != shape) throw std::runtime_error(std::string(#name) + " has a bad shape"); \
      if (t.element_size() != (int64_t)sizeof(ctype))                                              \
        throw std::runtime_error(std::string(#name) + " has a bad dtype");                          \
      w.name = reinterpret_cast<ctype*>(t.data_ptr());                                             \
      ++k;                                                                                         \
    }
    AD_WORLD_FIELDS(AD_BIND)
#undef AD_BIND
  }

  cudaStream_t stream() const { return c10::cuda::getCurrentCUDAStream().stream(); }

  void control(c10::optional<torch::Tensor> actions) {
    const int32_t* a = nullptr;
    if (actions.has_value()) {
      auto& t = actions.value();
      if (t.scalar_type() != torch::kInt32 || !t.is_contiguous() || t.numel() != (int64_t)sp.n * sp.R ||
          t.is_cuda() != cuda)
        throw std::runtime_error("actions must be a contiguous int32 [n, R] tensor on the world device");
      a = t.data_ptr<int32_t>();
    }
    if (cuda) launch_control(w, sp, a, stream());
    else host_control(w, sp, a);
  }
  void plan(int force) {
    if (cuda) launch_plan(w, sp, force, stream());
    else host_plan(w, sp, force);
  }
  void tick(uint32_t t, int run_game) {
    if (cuda) launch_tick(w, sp, t, run_game, threads, stream());
    else host_tick(w, sp, t, run_game);
    if (run_game && sense_in_tick) sense(0);
  }
  // Stereo-cluster FUEL perception (3v3); rows without a sensor update this
  // tick return at once unless `force`.
  void sense(int force) {
    if (!sp.stereo_tracks) return;
    if (cuda) launch_sense(w, sp, force, stream());
    else host_sense(w, sp, force);
  }
  void physics(int ticks) {
    if (cuda) launch_physics(w, sp, ticks, threads, stream());
    else host_physics(w, sp, ticks);
  }
  void perceive() {
    if (cuda) launch_perceive(w, sp, threads, stream());
    else host_perceive(w, sp);
    sense(1);
  }
  void observe() {
    if (cuda) launch_observe(w, sp, stream());
    else host_observe(w, sp);
  }
  void set_seed(uint32_t s0, uint32_t s1) {
    sp.seed0 = s0;
    sp.seed1 = s1;
  }
};

}  // namespace

void register_policy_ops(py::module& m);
void register_comm_ops(py::module& m);
void register_policy_tc_ops(py::module& m);
void register_tc_gemm_ops(py::module& m);
void register_attention_ops(py::module& m);
void register_layernorm_ops(py::module& m);
void register_adstar_cpu(py::module& m);
void register_sha256_ops(py::module& m);
void register_plan_a_ops(py::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200-native FRC REBUILT simulator kernels";
  m.def("schema", &schema, "state tensor schema (name, dtype code, shape)");
  m.def("tick_smem_bytes", &tick_smem_bytes);
  m.def("phase_profile_enable", &phase_profile_enable, "turn the tick kernel's per-phase cycle counters on/off");
  m.def("phase_profile_read", &phase_profile_read,
        "read and reset the 18 per-phase cycle totals (summed over CTAs): robot swerve, robot sweep, robot "
        "contacts, robot tail, fuel integrate+clear, fuel scatter, fuel pairs, fuel apply, fuel chassis "
        "reduction, fuel static, pre-substep, post-substep, robot-warp join wait, fuel-warps join wait, "
        "fuel count, fuel scan, fuel chassis loop, fuel pairs loop (the pairs bucket then holds only its reduction)");
  m.def("sense_rank_sort_host", [](torch::Tensor keys) {
        // host twin of the sensor stage's bearing sort (both the all-pairs and bucketed paths)
        auto k = keys.detach().to(torch::kCPU, torch::kFloat32).contiguous();
        const int n = (int)k.numel();
        if (n > 2 * kMaxPieces) throw std::runtime_error("at most 2 x 640 keys");
        const int P = n / 2 + 1;
        std::vector<uint8_t> buf(sense_carve(nullptr, P, nullptr) + 16);
        SenseScratch s;
        sense_carve(buf.data(), P, &s);
        for (int b = 0; b <= kSortBuckets; ++b) s.sbucket[b] = 0;
        const float* kp = k.data_ptr<float>();
        for (int j = 0; j < n; ++j) sense_sort_add(s, j, kp[j]);
        std::vector<int16_t> order(n > 0 ? n : 1);
        sense_rank_sort(kp, n, order.data(), s);
        auto out = torch::empty({n}, torch::kInt64);
        for (int j = 0; j < n; ++j) out[j] = (int64_t)order[j];
        return out;
      }, "stable ascending order of keys in [-pi, pi] by the sensor stage's rank sort (host)");
  m.def("plan_profile_read", &plan_profile_read,
        "read and reset the plan kernel's per-phase cycle counters (grid, endpoints, move table, sweeps, "
        "descent, line of sight, smoothing, speed profile)");
  m.def("sense_profile_read", &sense_profile_read,
        "read and reset the sense kernel's 8 per-phase cycle totals (summed over rows; counted while the "
        "phase profile is enabled): load, lens visibility, lens geometry+sort, lens depth buffer, lens "
        "objects, stereo fusion, packing, association");
  m.def("plan_smem_bytes", [](py::dict d) { return plan_smem_bytes(params_from_dict(d)); });
  m.def("sense_smem_bytes", [](py::dict d) { return sense_smem_bytes(params_from_dict(d)); });
  py::class_<Sim>(m, "Sim")
      .def(py::init<std::vector<torch::Tensor>, py::dict>())
      .def("control", &Sim::control, py::arg("actions") = py::none())
      .def("plan", &Sim::plan, py::arg("force") = 0)
      .def("tick", &Sim::tick, py::arg("tick"), py::arg("run_game") = 1)
      .def("physics", &Sim::physics, py::arg("ticks"))
      .def("observe", &Sim::observe)
      .def("perceive", &Sim::perceive)
      .def("sense", &Sim::sense, py::arg("force") = 0)
      .def_readwrite("sense_in_tick", &Sim::sense_in_tick)
      .def("set_seed", &Sim::set_seed)
      .def_readwrite("threads", &Sim::threads)
      .def_property_readonly("cuda", [](const Sim& s) { return s.cuda; });
  register_policy_ops(m);
  register_comm_ops(m);
  register_policy_tc_ops(m);
  register_tc_gemm_ops(m);
  register_attention_ops(m);
  register_layernorm_ops(m);
  register_adstar_cpu(m);
  register_sha256_ops(m);
  register_plan_a_ops(m);
}
