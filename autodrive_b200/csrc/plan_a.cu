// Exact-weight shortest paths on batched pose graphs (MECO "Plan A").
//
// Graphs share one CSR topology (row_ptr [n+1], col [E]) and carry their own
// fp64 edge weights [G, E] (>= 0) and source node. One CTA per graph runs a
// frontier relaxation (Bellman-Ford restricted to nodes whose distance changed
// in the previous round) until a round changes nothing; distances are fp64
// and relaxed with a 64-bit integer atomicMin on their bit patterns, which
// orders non-negative doubles exactly. The fixed point is the exact Dijkstra
// distance (same sums, min over the same paths). Predecessors are then
// recovered from the reverse CSR: the smallest-index in-neighbour u with
// dist[u] + w(u,v) == dist[v]. The host twin is a binary-heap Dijkstra.
// Reference: frc_defense/meco_plan_a_shortest_path_hip.py,
// csrc/meco_plan_a_shortest_path_hip_kernel.cu:216-650.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <limits>
#include <queue>
#include <vector>

namespace py = pybind11;

namespace {

constexpr int kThreads = 1024;

__device__ __forceinline__ unsigned long long bits(double x) { return (unsigned long long)__double_as_longlong(x); }

__global__ void __launch_bounds__(kThreads) frontier_sssp_kernel(
    const int64_t* __restrict__ row_ptr, const int32_t* __restrict__ col, const double* __restrict__ weights,
    const int64_t* __restrict__ sources, int n, int64_t E, double* __restrict__ dist_out,
    uint8_t* __restrict__ active, int* __restrict__ rounds_out, int max_rounds) {
  const int g = blockIdx.x;
  double* dist = dist_out + (int64_t)g * n;
  uint8_t* act = active + (int64_t)g * 2 * n;   // [cur | next]
  const double* w = weights + (int64_t)g * E;
  const double inf = __longlong_as_double(0x7ff0000000000000ll);
  for (int v = threadIdx.x; v < n; v += blockDim.x) {
    dist[v] = inf;
    act[v] = 0;
    act[n + v] = 0;
  }
  __syncthreads();
  const int s = (int)sources[g];
  if (threadIdx.x == 0 && s >= 0 && s < n) {
    dist[s] = 0.;
    act[s] = 1;
  }
  __syncthreads();
  __shared__ int changed;
  int round = 0;
  uint8_t* cur = act;
  uint8_t* nxt = act + n;
  for (; round < max_rounds; ++round) {
    if (threadIdx.x == 0) changed = 0;
    __syncthreads();
    for (int u = threadIdx.x; u < n; u += blockDim.x) {
      if (!cur[u]) continue;
      cur[u] = 0;
      const double du = dist[u];
      for (int64_t e = row_ptr[u]; e < row_ptr[u + 1]; ++e) {
        const int v = col[e];
        const double cand = du + w[e];
        if (cand < dist[v]) {
          const unsigned long long old = atomicMin(reinterpret_cast<unsigned long long*>(dist + v), bits(cand));
          if (bits(cand) < old) {
            nxt[v] = 1;
            changed = 1;
          }
        }
      }
    }
    __syncthreads();
    const int any = changed;
    uint8_t* t = cur;
    cur = nxt;
    nxt = t;
    __syncthreads();
    if (!any) break;
  }
  if (threadIdx.x == 0) rounds_out[g] = round;
}

__global__ void predecessor_kernel(const int64_t* __restrict__ rrow, const int32_t* __restrict__ rcol,
                                   const int64_t* __restrict__ redge, const double* __restrict__ weights,
                                   const double* __restrict__ dist_all, int n, int64_t E,
                                   int32_t* __restrict__ pred_out) {
  const int g = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= n) return;
  const double* dist = dist_all + (int64_t)g * n;
  const double* w = weights + (int64_t)g * E;
  int best = -1;
  const double dv = dist[v];
  if (dv > 0. && dv < __longlong_as_double(0x7ff0000000000000ll)) {
    for (int64_t k = rrow[v]; k < rrow[v + 1]; ++k) {
      const int u = rcol[k];
      if (dist[u] + w[redge[k]] == dv && (best < 0 || u < best)) best = u;
    }
  }
  pred_out[(int64_t)g * n + v] = best;
}

void check_csr(const torch::Tensor& row_ptr, const torch::Tensor& col, const torch::Tensor& weights,
               const torch::Tensor& sources) {
  TORCH_CHECK(row_ptr.scalar_type() == torch::kInt64 && row_ptr.dim() == 1, "row_ptr must be int64 [n+1]");
  TORCH_CHECK(col.scalar_type() == torch::kInt32 && col.dim() == 1, "col must be int32 [E]");
  TORCH_CHECK(weights.scalar_type() == torch::kFloat64 && weights.dim() == 2 && weights.size(1) == col.numel(),
              "weights must be float64 [G, E]");
  TORCH_CHECK(sources.scalar_type() == torch::kInt64 && sources.numel() == weights.size(0), "sources: int64 [G]");
  for (auto* t : {&row_ptr, &col, &weights, &sources}) TORCH_CHECK(t->is_contiguous(), "inputs must be contiguous");
}

// Reverse CSR (host): for every node v its in-neighbours u and the forward edge ids.
void reverse_csr(const int64_t* rp, const int32_t* c, int n, int64_t E, std::vector<int64_t>& rrow,
                 std::vector<int32_t>& rcol, std::vector<int64_t>& redge) {
  rrow.assign(n + 1, 0);
  for (int64_t e = 0; e < E; ++e) rrow[c[e] + 1]++;
  for (int v = 0; v < n; ++v) rrow[v + 1] += rrow[v];
  rcol.resize(E);
  redge.resize(E);
  std::vector<int64_t> fill(rrow.begin(), rrow.end() - 1);
  for (int u = 0; u < n; ++u)
    for (int64_t e = rp[u]; e < rp[u + 1]; ++e) {
      const int64_t k = fill[c[e]]++;
      rcol[k] = u;
      redge[k] = e;
    }
}

std::vector<torch::Tensor> shortest_paths(torch::Tensor row_ptr, torch::Tensor col, torch::Tensor weights,
                                          torch::Tensor sources, int64_t max_rounds) {
  check_csr(row_ptr, col, weights, sources);
  const int n = (int)row_ptr.numel() - 1;
  const int64_t E = col.numel();
  const int64_t G = weights.size(0);
  auto dist = torch::empty({G, n}, weights.options());
  auto pred = torch::empty({G, n}, weights.options().dtype(torch::kInt32));
  auto rounds = torch::zeros({G}, weights.options().dtype(torch::kInt32));
  if (G == 0 || n == 0) return {dist, pred, rounds};
  // reverse topology on the host (shared by every graph)
  auto rp_h = row_ptr.cpu();
  auto c_h = col.cpu();
  TORCH_CHECK(rp_h[0].item<int64_t>() == 0 && rp_h[n].item<int64_t>() == E, "row_ptr must span [0, E]");
  TORCH_CHECK(c_h.numel() == 0 || (c_h.min().item<int32_t>() >= 0 && c_h.max().item<int32_t>() < n),
              "col entries must be node ids");
  std::vector<int64_t> rrow, redge;
  std::vector<int32_t> rcol;
  reverse_csr(rp_h.data_ptr<int64_t>(), c_h.data_ptr<int32_t>(), n, E, rrow, rcol, redge);
  if (weights.is_cuda()) {
    auto opt = weights.options();
    auto rrow_t = torch::from_blob(rrow.data(), {(int64_t)rrow.size()}, torch::kInt64).to(opt.dtype(torch::kInt64));
    auto rcol_t = torch::from_blob(rcol.data(), {(int64_t)rcol.size()}, torch::kInt32).to(opt.dtype(torch::kInt32));
    auto redge_t = torch::from_blob(redge.data(), {(int64_t)redge.size()}, torch::kInt64).to(opt.dtype(torch::kInt64));
    auto active = torch::empty({G, 2 * (int64_t)n}, opt.dtype(torch::kUInt8));
    auto st = c10::cuda::getCurrentCUDAStream().stream();
    frontier_sssp_kernel<<<(unsigned)G, kThreads, 0, st>>>(
        row_ptr.data_ptr<int64_t>(), col.data_ptr<int32_t>(), weights.data_ptr<double>(), sources.data_ptr<int64_t>(),
        n, E, dist.data_ptr<double>(), active.data_ptr<uint8_t>(), rounds.data_ptr<int32_t>(), (int)max_rounds);
    TORCH_CHECK(cudaGetLastError() == cudaSuccess, "frontier_sssp_kernel launch failed");
    dim3 grid((unsigned)((n + 255) / 256), (unsigned)G);
    predecessor_kernel<<<grid, 256, 0, st>>>(rrow_t.data_ptr<int64_t>(), rcol_t.data_ptr<int32_t>(),
                                             redge_t.data_ptr<int64_t>(), weights.data_ptr<double>(),
                                             dist.data_ptr<double>(), n, E, pred.data_ptr<int32_t>());
    TORCH_CHECK(cudaGetLastError() == cudaSuccess, "predecessor_kernel launch failed");
    return {dist, pred, rounds};
  }
  // host twin: binary-heap Dijkstra per graph, predecessors by the same tightness rule
  const int64_t* rp = row_ptr.data_ptr<int64_t>();
  const int32_t* c = col.data_ptr<int32_t>();
  const int64_t* src = sources.data_ptr<int64_t>();
  const double inf = std::numeric_limits<double>::infinity();
  for (int64_t g = 0; g < G; ++g) {
    const double* w = weights.data_ptr<double>() + g * E;
    double* d = dist.data_ptr<double>() + g * n;
    int32_t* p = pred.data_ptr<int32_t>() + g * n;
    for (int v = 0; v < n; ++v) d[v] = inf;
    using Item = std::pair<double, int>;
    std::priority_queue<Item, std::vector<Item>, std::greater<Item>> pq;
    if (src[g] >= 0 && src[g] < n) {
      d[src[g]] = 0.;
      pq.push({0., (int)src[g]});
    }
    int pops = 0;
    while (!pq.empty()) {
      auto [du, u] = pq.top();
      pq.pop();
      if (du > d[u]) continue;
      ++pops;
      for (int64_t e = rp[u]; e < rp[u + 1]; ++e) {
        const double cand = du + w[e];
        if (cand < d[c[e]]) {
          d[c[e]] = cand;
          pq.push({cand, c[e]});
        }
      }
    }
    rounds.data_ptr<int32_t>()[g] = pops;
    for (int v = 0; v < n; ++v) {
      int best = -1;
      if (d[v] > 0. && d[v] < inf)
        for (int64_t k = rrow[v]; k < rrow[v + 1]; ++k)
          if (d[rcol[k]] + w[redge[k]] == d[v] && (best < 0 || rcol[k] < best)) best = rcol[k];
      p[v] = best;
    }
  }
  return {dist, pred, rounds};
}

}  // namespace

void register_plan_a_ops(py::module& m) {
  m.def("plan_a_shortest_paths", &shortest_paths,
        "batched exact fp64 shortest paths on a shared CSR topology -> (dist [G,n], pred [G,n], rounds [G])",
        py::arg("row_ptr"), py::arg("col"), py::arg("weights"), py::arg("sources"), py::arg("max_rounds") = 1 << 20);
}
