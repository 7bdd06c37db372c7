// Host-side incremental Anytime Dynamic A* (AD*) on an 8-connected grid.
//
// Algorithm: Likhachev, Ferguson, Gordon, Stentz, Thrun, "Anytime Dynamic A*:
// An Anytime, Replanning Algorithm" (ICAPS 2005). The search runs backwards
// from the goal (like D* Lite), so a moved start or changed cell costs reuse
// the previous g/rhs values:
//   key(s)   = [rhs + eps*h, rhs] if g > rhs else [g + h, g]
//   update   rhs(s) = min over successors (c(s,s') + g(s')); re-queue s in
//            OPEN (or INCONS if already expanded in this pass)
//   improve  pop while key(top) < key(start) or rhs(start) != g(start)
//   replan   changed cells -> update their neighbours; move INCONS into OPEN,
//            re-key OPEN, clear CLOSED, then improve with the next epsilon.
// Costs: edge length (1 or sqrt 2 cells) times the mean of the two cells'
// traversal weights; diagonal moves past a blocked corner are not allowed.
// Reference behaviour: frc_defense/adstar.py:62-912 (ADStarPlanner).
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>
#include <queue>
#include <stdexcept>
#include <utility>
#include <vector>

namespace py = pybind11;

namespace {

constexpr double kInf = std::numeric_limits<double>::infinity();
constexpr int kDX[8] = {1, -1, 0, 0, 1, 1, -1, -1};
constexpr int kDY[8] = {0, 0, 1, -1, 1, -1, 1, -1};

struct Key {
  double a, b;
  bool operator<(const Key& o) const { return a < o.a || (a == o.a && b < o.b); }
};

struct KeyGreater {  // min-heap on the key
  bool operator()(const std::pair<Key, int>& x, const std::pair<Key, int>& y) const { return y.first < x.first; }
};

class ADStarCore {
 public:
  ADStarCore(int nx, int ny) : nx_(nx), ny_(ny), n_(nx * ny) {
    if (nx < 1 || ny < 1) throw std::invalid_argument("grid must be at least 1x1");
    blocked_.assign(n_, 0);
    weight_.assign(n_, 1.f);
    reset_values();
  }

  int nx() const { return nx_; }
  int ny() const { return ny_; }
  double epsilon() const { return eps_; }
  int64_t expansions() const { return expansions_; }

  // Replace occupancy and weights; cells whose cost changed are repaired
  // incrementally on the next plan() call.
  void set_grid(torch::Tensor blocked, torch::Tensor weight) {
    TORCH_CHECK(blocked.numel() == n_ && weight.numel() == n_, "grid tensors must have nx*ny entries");
    auto b = blocked.to(torch::kCPU, torch::kUInt8).contiguous();
    auto w = weight.to(torch::kCPU, torch::kFloat32).contiguous();
    const uint8_t* bp = b.data_ptr<uint8_t>();
    const float* wp = w.data_ptr<float>();
    for (int i = 0; i < n_; ++i) {
      const float wi = std::max(wp[i], 1e-3f);
      if (bp[i] != blocked_[i] || wi != weight_[i]) {
        blocked_[i] = bp[i];
        weight_[i] = wi;
        changed_.push_back(i);
      }
    }
  }

  // Plan from start to goal (cell indices). Returns the cell path (start..goal)
  // or an empty list when the goal is unreachable within the budget.
  std::vector<int> plan(int start, int goal, int64_t budget, double eps0, double eps_min, double eps_step) {
    if (start < 0 || start >= n_ || goal < 0 || goal >= n_) throw std::out_of_range("cell out of the grid");
    const bool fresh = goal != goal_;
    const bool moved = start != start_;
    start_ = start;  // keys below use the heuristic towards the new start
    if (fresh) {
      goal_ = goal;
      reset_values();
      changed_.clear();
      eps_ = eps0;
      rhs_[goal_] = 0.;
      push(goal_);
    }
    if (!changed_.empty()) {
      for (int c : changed_) {
        update_state(c);
        for (int k = 0; k < 8; ++k) {
          const int x = c % nx_ + kDX[k], y = c / nx_ + kDY[k];
          if (x >= 0 && x < nx_ && y >= 0 && y < ny_) update_state(y * nx_ + x);
        }
      }
      changed_.clear();
      eps_ = std::max(eps_, eps0 * .5);  // significant change: back off the bound a little
    }
    if (moved && !fresh) rekey();
    expansions_ = 0;
    double eps = eps_;
    std::vector<int> best;
    while (true) {
      eps_ = eps;
      // INCONS -> OPEN, clear CLOSED, re-key for the new epsilon
      for (int s : incons_) if (g_[s] != rhs_[s]) open_flag_[s] = 1;
      incons_.clear();
      std::fill(closed_.begin(), closed_.end(), 0);
      rekey();
      if (!improve(budget)) break;
      best = extract();
      if (eps <= eps_min + 1e-12 || best.empty()) break;
      eps = std::max(eps_min, eps - eps_step);
    }
    return best;
  }

  torch::Tensor g_values() const {
    auto t = torch::empty({n_}, torch::kFloat64);
    std::copy(g_.begin(), g_.end(), t.data_ptr<double>());
    return t;
  }

 private:
  int nx_, ny_, n_;
  std::vector<uint8_t> blocked_;
  std::vector<float> weight_;
  std::vector<double> g_, rhs_;
  std::vector<uint8_t> closed_, open_flag_;
  std::vector<Key> key_;
  std::vector<int> incons_, changed_;
  std::priority_queue<std::pair<Key, int>, std::vector<std::pair<Key, int>>, KeyGreater> heap_;
  int start_ = -1, goal_ = -1;
  double eps_ = 2.5;
  int64_t expansions_ = 0;

  void reset_values() {
    g_.assign(n_, kInf);
    rhs_.assign(n_, kInf);
    closed_.assign(n_, 0);
    open_flag_.assign(n_, 0);
    key_.assign(n_, Key{kInf, kInf});
    incons_.clear();
    heap_ = decltype(heap_)();
  }

  double h(int s) const {  // octile distance in cells (admissible for unit-weight moves)
    const int dx = std::abs(s % nx_ - start_ % nx_), dy = std::abs(s / nx_ - start_ / nx_);
    return (double)std::max(dx, dy) + (std::sqrt(2.) - 1.) * std::min(dx, dy);
  }

  Key key(int s) const {
    if (g_[s] > rhs_[s]) return Key{rhs_[s] + eps_ * h(s), rhs_[s]};
    return Key{g_[s] + h(s), g_[s]};
  }

  double cost(int a, int b, int k) const {
    if (blocked_[a] || blocked_[b]) return kInf;
    if (k >= 4) {  // no corner cutting
      const int ax = a % nx_, ay = a / nx_;
      if (blocked_[ay * nx_ + ax + kDX[k]] || blocked_[(ay + kDY[k]) * nx_ + ax]) return kInf;
    }
    return (k >= 4 ? std::sqrt(2.) : 1.) * .5 * ((double)weight_[a] + (double)weight_[b]);
  }

  void push(int s) {
    key_[s] = key(s);
    open_flag_[s] = 1;
    heap_.push({key_[s], s});
  }

  void rekey() {
    heap_ = decltype(heap_)();
    for (int s = 0; s < n_; ++s)
      if (open_flag_[s]) push(s);
  }

  void update_state(int s) {
    if (s != goal_) {
      double best = kInf;
      const int x = s % nx_, y = s / nx_;
      for (int k = 0; k < 8; ++k) {
        const int xx = x + kDX[k], yy = y + kDY[k];
        if (xx < 0 || xx >= nx_ || yy < 0 || yy >= ny_) continue;
        const int t = yy * nx_ + xx;
        const double c = cost(s, t, k);
        if (c < kInf) best = std::min(best, c + g_[t]);
      }
      rhs_[s] = best;
    }
    open_flag_[s] = 0;
    if (g_[s] != rhs_[s]) {
      if (!closed_[s]) push(s);
      else incons_.push_back(s);
    }
  }

  bool top(int& s, Key& k) {
    while (!heap_.empty()) {
      auto [kk, ss] = heap_.top();
      if (!open_flag_[ss] || kk.a != key_[ss].a || kk.b != key_[ss].b) {  // stale entry
        heap_.pop();
        continue;
      }
      s = ss;
      k = kk;
      return true;
    }
    return false;
  }

  bool improve(int64_t budget) {
    int s;
    Key k;
    while (top(s, k) && (k < key(start_) || rhs_[start_] != g_[start_])) {
      if (expansions_++ >= budget) return false;
      heap_.pop();
      open_flag_[s] = 0;
      const int x = s % nx_, y = s / nx_;
      if (g_[s] > rhs_[s]) {
        g_[s] = rhs_[s];
        closed_[s] = 1;
        for (int kk = 0; kk < 8; ++kk) {
          const int xx = x + kDX[kk], yy = y + kDY[kk];
          if (xx >= 0 && xx < nx_ && yy >= 0 && yy < ny_) update_state(yy * nx_ + xx);
        }
      } else {
        g_[s] = kInf;
        update_state(s);
        for (int kk = 0; kk < 8; ++kk) {
          const int xx = x + kDX[kk], yy = y + kDY[kk];
          if (xx >= 0 && xx < nx_ && yy >= 0 && yy < ny_) update_state(yy * nx_ + xx);
        }
      }
    }
    return true;
  }

  std::vector<int> extract() const {
    std::vector<int> path;
    if (!(g_[start_] < kInf) && !(rhs_[start_] < kInf)) return path;
    int s = start_;
    path.push_back(s);
    for (int guard = 0; guard < n_ && s != goal_; ++guard) {
      const int x = s % nx_, y = s / nx_;
      double best = kInf;
      int next = -1;
      for (int k = 0; k < 8; ++k) {
        const int xx = x + kDX[k], yy = y + kDY[k];
        if (xx < 0 || xx >= nx_ || yy < 0 || yy >= ny_) continue;
        const int t = yy * nx_ + xx;
        const double c = cost(s, t, k) + g_[t];
        if (c < best) {
          best = c;
          next = t;
        }
      }
      if (next < 0 || !(best < kInf)) return {};
      s = next;
      path.push_back(s);
    }
    if (s != goal_) return {};
    return path;
  }
};

}  // namespace

void register_adstar_cpu(py::module& m) {
  py::class_<ADStarCore>(m, "ADStarCore", "incremental Anytime Dynamic A* on an 8-connected grid (host)")
      .def(py::init<int, int>())
      .def_property_readonly("nx", &ADStarCore::nx)
      .def_property_readonly("ny", &ADStarCore::ny)
      .def_property_readonly("epsilon", &ADStarCore::epsilon)
      .def_property_readonly("expansions", &ADStarCore::expansions)
      .def("set_grid", &ADStarCore::set_grid)
      .def("plan", &ADStarCore::plan, py::arg("start"), py::arg("goal"), py::arg("budget") = 12000,
           py::arg("eps0") = 2.5, py::arg("eps_min") = 1.0, py::arg("eps_step") = .5)
      .def("g_values", &ADStarCore::g_values);
}
