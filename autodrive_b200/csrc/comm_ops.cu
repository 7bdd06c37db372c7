// Fused data-parallel gradient all-reduce + global-norm clip + Adam over peer
// memory (NVLink / NVSwitch), one cooperative kernel per optimizer step.
//
// Reference behaviour being replaced: DDP's NCCL all-reduce of the gradient
// bucket, clip_grad_norm_ and Adam.step (frc_defense/tensor_training_ppo.py:
// 82-85, 431-434). Here every rank's flat gradient and flat parameter buffers
// live in one cudaMalloc'd region exported with CUDA IPC, so a kernel on rank
// r can load and store the buffers of every other rank directly:
//
//   phase 0  every rank signals "gradients ready" into each peer's signal pad
//   phase 1  rank r owns shard r: it loads shard r of every rank's gradient
//            (P2P loads), averages, writes the result into its own buffer and
//            accumulates the shard's sum of squares
//   phase 2  shard sums of squares are exchanged through the pads -> global
//            norm -> clip scale (identical on every rank)
//   phase 3  Adam on shard r (moments are kept for the owned shard only) and
//            the updated parameters are stored into every rank's parameter
//            buffer (P2P stores)
//   phase 4  final barrier: no rank overwrites its gradients or reads its
//            parameters before every peer is done with them
//
// Bytes over NVLink per rank and step: (W-1)/W of the gradient in and
// (W-1)/W of the parameters out, the two-shot all-reduce volume, with the
// optimizer work divided by W. Every wait on a peer flag is bounded; on
// expiry the kernel records the phase in a status word and finishes, so a
// missing peer never hangs the GPU. No TMA, no multicast.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

namespace py = pybind11;
namespace cg = cooperative_groups;

namespace {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 512;
constexpr int kPadWords = 1024;         // per-rank signal pad (uint32 words)
// pad layout (uint32 words): [0,8) ready flags, [8,16) norm flags, [16,24) done
// flags, [32,48) shard sums of squares as float bits (indexed by rank),
// [64, 64 + kMaxCta] per-CTA partials and the clip scale (local use only)
constexpr int kFlagReady = 0, kFlagNorm = 8, kFlagDone = 16, kFlagStats = 24, kNorms = 32, kFlagBcast = 48,
              kPartials = 64;
// stats exchange: two parity areas of kMaxRanks x kMaxStats doubles at word 512 and 768
constexpr int kStatsArea = 512, kMaxStats = 16;
constexpr int kMaxCta = 296;              // 2 CTAs per SM on a 148-SM part
constexpr int kUnroll = 4;                // independent 16-byte loads in flight per thread and peer

struct Ptrs {
  float* grad[kMaxRanks];
  float* param[kMaxRanks];
  uint32_t* pad[kMaxRanks];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Signal `slot` in every rank's pad, then wait for every rank's signal in ours.
// Returns false if the wait ran out of iterations.
__device__ bool cross_rank_barrier(const Ptrs& P, int world, int rank, int slot, uint32_t epoch,
                                   long long max_iters) {
  __threadfence_system();
  for (int q = 0; q < world; ++q) st_release_sys(P.pad[q] + slot + rank, epoch);
  for (int q = 0; q < world; ++q) {
    long long it = 0;
    while (ld_acquire_sys(P.pad[rank] + slot + q) != epoch) {
      if (++it > max_iters) return false;
      __nanosleep(128);
    }
  }
  return true;
}

// out[4k..4k+3] = (1/W) sum over ranks of grad_q[base + 4k..], k in [0, nvec);
// returns this thread's sum of squares of the written values. Every thread
// issues kUnroll independent 16-byte loads per rank before using any, so
// enough remote bytes are in flight to cover the NVLink round trip. Ranks are
// visited starting at `first` (the two-shot owner starts at its next peer so
// the W owners do not all read rank 0 first); the one-shot path passes 0 so
// every rank sums in the same order and the replicas stay bitwise equal.
__device__ __forceinline__ float reduce_range(const Ptrs& P, int world, float* __restrict__ out, int64_t base,
                                              int64_t nvec, float inv_w, int first) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float acc = 0.f;
  for (int64_t k0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k0 < nvec; k0 += kUnroll * stride) {
    float4 s[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) s[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j) {
      if (j >= world) break;
      const int q = first + j < world ? first + j : first + j - world;
      float4 x[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t k = k0 + u * stride;
        x[u] = k < nvec ? __ldcg(reinterpret_cast<const float4*>(P.grad[q] + base) + k) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        s[u].x += x[u].x; s[u].y += x[u].y; s[u].z += x[u].z; s[u].w += x[u].w;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t k = k0 + u * stride;
      if (k < nvec) {
        float4 r = make_float4(s[u].x * inv_w, s[u].y * inv_w, s[u].z * inv_w, s[u].w * inv_w);
        reinterpret_cast<float4*>(out)[k] = r;
        acc += r.x * r.x + r.y * r.y + r.z * r.z + r.w * r.w;
      }
    }
  }
  return acc;
}

__global__ void __launch_bounds__(kThreads) fused_allreduce_adam_kernel(
    Ptrs P, int world, int rank, int64_t n_padded, float* __restrict__ m, float* __restrict__ v,
    uint32_t epoch, float lr, float b1, float b2, float eps, float wd, float bias1, float bias2, float max_norm,
    float* __restrict__ norm_out, int* __restrict__ status, long long max_iters) {
  cg::grid_group grid = cg::this_grid();
  const int64_t shard = n_padded / world;       // multiple of 4
  const int64_t lo = shard * rank;
  __shared__ bool ok_s;
  __shared__ float red[kThreads / 32];
  uint32_t* mypad = P.pad[rank];
  // phase 0: gradients ready on every rank
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    bool ok = cross_rank_barrier(P, world, rank, kFlagReady, epoch, max_iters);
    if (!ok) atomicExch(status, 1);
  }
  grid.sync();
  const bool healthy = *(volatile int*)status == 0;
  // phase 1: reduce-scatter the owned shard, sum of squares
  float acc = 0.f;
  const float inv_w = 1.f / (float)world;
  if (healthy) acc = reduce_range(P, world, P.grad[rank] + lo, lo, shard / 4, inv_w, rank + 1 < world ? rank + 1 : 0);
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    reinterpret_cast<float*>(mypad + kPartials)[blockIdx.x] = t;
  }
  grid.sync();
  // phase 2: exchange shard norms
  __shared__ float scale_s;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    float t = 0.f;
    for (int c = 0; c < (int)gridDim.x; ++c) t += reinterpret_cast<float*>(mypad + kPartials)[c];
    for (int q = 0; q < world; ++q) reinterpret_cast<float*>(P.pad[q] + kNorms)[rank] = t;
    bool ok = healthy && cross_rank_barrier(P, world, rank, kFlagNorm, epoch, max_iters);
    if (!ok && healthy) atomicExch(status, 2);
    float total = 0.f;
    for (int q = 0; q < world; ++q) total += reinterpret_cast<volatile float*>(mypad + kNorms)[q];
    const float norm = sqrtf(total);
    reinterpret_cast<float*>(mypad + kPartials)[kMaxCta] = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
    *norm_out = norm;
  }
  grid.sync();
  ok_s = *(volatile int*)status == 0;
  scale_s = reinterpret_cast<volatile float*>(mypad + kPartials)[kMaxCta];
  __syncthreads();
  // phase 3: Adam on the owned shard, all-gather parameters with peer stores
  if (ok_s) {
    const float scale = scale_s;
    const int64_t nvec = shard / 4;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nvec; k += (int64_t)gridDim.x * blockDim.x) {
      const int64_t i = lo + k * 4;
      float4 g = *reinterpret_cast<const float4*>(P.grad[rank] + i);
      float4 p = *reinterpret_cast<const float4*>(P.param[rank] + i);
      float4 mm = *reinterpret_cast<const float4*>(m + i);
      float4 vv = *reinterpret_cast<const float4*>(v + i);
      float* pg = &g.x;
      float* pp = &p.x;
      float* pm = &mm.x;
      float* pv = &vv.x;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float gi = pg[c] * scale + wd * pp[c];
        pm[c] = b1 * pm[c] + (1.f - b1) * gi;
        pv[c] = b2 * pv[c] + (1.f - b2) * gi * gi;
        pp[c] -= lr * (pm[c] / bias1) / (sqrtf(pv[c] / bias2) + eps);
      }
      *reinterpret_cast<float4*>(m + i) = mm;
      *reinterpret_cast<float4*>(v + i) = vv;
      for (int j = 1; j <= world; ++j) {   // peers from the next rank on, own buffer last
        const int q = rank + j < world ? rank + j : rank + j - world;
        *reinterpret_cast<float4*>(P.param[q] + i) = p;
      }
    }
  }
  __threadfence_system();
  grid.sync();
  // phase 4: every peer finished reading gradients and writing parameters
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    bool ok = cross_rank_barrier(P, world, rank, kFlagDone, epoch, max_iters);
    if (!ok) atomicCAS(status, 0, 4);
  }
  grid.sync();
}

// One-shot variant for small buffers (latency bound): every rank reads every
// peer's full gradient, reduces it into a local scratch buffer, computes the
// global norm itself and applies Adam to the whole buffer, so parameters never
// cross NVLink and there is no norm exchange. Two cross-rank barriers: the
// gradients are ready, and every peer has finished reading ours.
__global__ void __launch_bounds__(kThreads) oneshot_allreduce_adam_kernel(
    Ptrs P, int world, int rank, int64_t n_padded, float* __restrict__ scratch, float* __restrict__ m,
    float* __restrict__ v, uint32_t epoch, float lr, float b1, float b2, float eps, float wd, float bias1,
    float bias2, float max_norm, float* __restrict__ norm_out, int* __restrict__ status, long long max_iters) {
  cg::grid_group grid = cg::this_grid();
  __shared__ float red[kThreads / 32];
  __shared__ float scale_s;
  __shared__ bool ok_s;
  uint32_t* mypad = P.pad[rank];
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    bool ok = cross_rank_barrier(P, world, rank, kFlagReady, epoch, max_iters);
    if (!ok) atomicExch(status, 1);
  }
  grid.sync();
  const bool healthy = *(volatile int*)status == 0;
  const float inv_w = 1.f / (float)world;
  const int64_t nvec = n_padded / 4;
  float acc = 0.f;
  if (healthy) acc = reduce_range(P, world, scratch, 0, nvec, inv_w, 0);
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    reinterpret_cast<float*>(mypad + kPartials)[blockIdx.x] = t;
  }
  grid.sync();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    float total = 0.f;
    for (int c = 0; c < (int)gridDim.x; ++c) total += reinterpret_cast<float*>(mypad + kPartials)[c];
    const float norm = sqrtf(total);
    reinterpret_cast<float*>(mypad + kPartials)[kMaxCta] = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
    *norm_out = norm;
  }
  grid.sync();
  ok_s = healthy;
  scale_s = reinterpret_cast<volatile float*>(mypad + kPartials)[kMaxCta];
  __syncthreads();
  if (ok_s) {
    const float scale = scale_s;
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nvec; k += (int64_t)gridDim.x * blockDim.x) {
      float4 g = reinterpret_cast<const float4*>(scratch)[k];
      float4 p = *reinterpret_cast<const float4*>(P.param[rank] + 4 * k);
      float4 mm = reinterpret_cast<const float4*>(m)[k];
      float4 vv = reinterpret_cast<const float4*>(v)[k];
      float* pg = &g.x;
      float* pp = &p.x;
      float* pm = &mm.x;
      float* pv = &vv.x;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float gi = pg[c] * scale + wd * pp[c];
        pm[c] = b1 * pm[c] + (1.f - b1) * gi;
        pv[c] = b2 * pv[c] + (1.f - b2) * gi * gi;
        pp[c] -= lr * (pm[c] / bias1) / (sqrtf(pv[c] / bias2) + eps);
      }
      reinterpret_cast<float4*>(m)[k] = mm;
      reinterpret_cast<float4*>(v)[k] = vv;
      *reinterpret_cast<float4*>(P.param[rank] + 4 * k) = p;
    }
  }
  __threadfence_system();
  grid.sync();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    bool ok = cross_rank_barrier(P, world, rank, kFlagDone, epoch, max_iters);
    if (!ok) atomicCAS(status, 0, 4);
  }
  grid.sync();
}

// Stats all-reduce over peer memory: `nsum` values are summed and `nmax`
// values max-reduced across ranks in one single-CTA launch (one cross-rank
// barrier). Values travel as doubles through the peers' signal pads; the
// epoch's parity selects one of two areas so a peer one call behind never
// sees its inputs overwritten.
__global__ void peer_stats_kernel(Ptrs P, int world, int rank, const double* __restrict__ in,
                                  double* __restrict__ out, int nsum, int nmax, uint32_t epoch,
                                  int* __restrict__ status, long long max_iters) {
  const int nv = nsum + nmax;
  const int area = kStatsArea + (int)(epoch & 1u) * (kMaxRanks * kMaxStats * 2);
  if ((int)threadIdx.x < nv) {
    const double x = in[threadIdx.x];
    for (int q = 0; q < world; ++q)
      reinterpret_cast<double*>(P.pad[q] + area)[rank * kMaxStats + threadIdx.x] = x;
  }
  __syncthreads();
  __shared__ bool ok;
  if (threadIdx.x == 0) {
    ok = cross_rank_barrier(P, world, rank, kFlagStats, epoch, max_iters);
    if (!ok) atomicCAS(status, 0, 8);
  }
  __syncthreads();
  if ((int)threadIdx.x < nv && ok) {
    const volatile double* mine = reinterpret_cast<const volatile double*>(P.pad[rank] + area);
    double acc = mine[threadIdx.x];
    for (int q = 1; q < world; ++q) {
      const double y = mine[q * kMaxStats + threadIdx.x];
      acc = (int)threadIdx.x < nsum ? acc + y : fmax(acc, y);
    }
    out[threadIdx.x] = acc;
  }
}

// Broadcast of rank `root`'s parameter buffer into every peer's parameter
// buffer with peer stores (cooperative): the root's CTAs copy, then it
// releases a flag in every pad; the other ranks wait for it.
__global__ void __launch_bounds__(kThreads) peer_broadcast_kernel(Ptrs P, int world, int rank, int root,
                                                                  int64_t n_padded, uint32_t epoch,
                                                                  int* __restrict__ status, long long max_iters) {
  cg::grid_group grid = cg::this_grid();
  if (rank == root) {
    const int64_t nvec = n_padded / 4;
    const float4* src = reinterpret_cast<const float4*>(P.param[root]);
    for (int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; k < nvec; k += (int64_t)gridDim.x * blockDim.x) {
      const float4 x = src[k];
      for (int q = 0; q < world; ++q)
        if (q != root) reinterpret_cast<float4*>(P.param[q])[k] = x;
    }
    __threadfence_system();
  }
  grid.sync();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (rank == root) {
      for (int q = 0; q < world; ++q) st_release_sys(P.pad[q] + kFlagBcast + root, epoch);
    } else {
      long long it = 0;
      while (ld_acquire_sys(P.pad[rank] + kFlagBcast + root) != epoch) {
        if (++it > max_iters) {
          atomicCAS(status, 0, 16);
          break;
        }
        __nanosleep(128);
      }
    }
  }
  grid.sync();
}

struct Comm {
  int world = 1, rank = 0, device = 0;
  int64_t n = 0, n_padded = 0;
  void* base = nullptr;                 // local cudaMalloc region
  size_t bytes = 0;
  Ptrs P{};
  std::vector<void*> opened;
  uint32_t epoch = 0, stats_epoch = 0, bcast_epoch = 0;
  int grid = 0;
  bool oneshot = false;                 // small buffers: one-shot all-reduce, full local Adam
  float* scratch = nullptr;             // one-shot reduced gradient (local)
  torch::Tensor status;                 // int32 [1]

  ~Comm() {
    if (scratch) cudaFree(scratch);
    for (void* p : opened) cudaIpcCloseMemHandle(p);
    if (base) cudaFree(base);
  }
};

size_t region_bytes(int64_t n_padded) { return (size_t)n_padded * 8 + kPadWords * 4 * 2; }

struct CommHandle {
  std::shared_ptr<Comm> c;
};

// Allocate the local region [grad n_padded][param n_padded][signal pad]; its
// IPC handle is exchanged with the other ranks by `ipc_handle` / `open_peers`.
CommHandle create(int64_t n, int world, int rank, int64_t oneshot_bytes) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world) throw std::runtime_error("bad world/rank");
  auto c = std::make_shared<Comm>();
  c->world = world;
  c->rank = rank;
  cudaGetDevice(&c->device);
  c->n = n;
  const int64_t unit = 4 * (int64_t)world;
  c->n_padded = (n + unit - 1) / unit * unit;
  c->bytes = region_bytes(c->n_padded);
  if (cudaMalloc(&c->base, c->bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc of the comm region failed");
  cudaMemset(c->base, 0, c->bytes);
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, c->device);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fused_allreduce_adam_kernel, kThreads, 0);
  c->grid = std::max(1, std::min(kMaxCta, sms * std::max(1, per_sm)));
  c->oneshot = world > 1 && c->n_padded * 4 <= oneshot_bytes;
  if (c->oneshot) {
    if (cudaMalloc(&c->scratch, (size_t)c->n_padded * 4) != cudaSuccess)
      throw std::runtime_error("cudaMalloc of the one-shot scratch failed");
    int per_sm1 = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm1, oneshot_allreduce_adam_kernel, kThreads, 0);
    c->grid = std::max(1, std::min(c->grid, sms * std::max(1, per_sm1)));
  }
  c->status = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt32).device(torch::kCUDA, c->device));
  return CommHandle{c};
}

py::bytes ipc_handle(const CommHandle& h) {
  cudaIpcMemHandle_t handle;
  if (cudaIpcGetMemHandle(&handle, h.c->base) != cudaSuccess) throw std::runtime_error("cudaIpcGetMemHandle failed");
  return py::bytes(reinterpret_cast<const char*>(&handle), sizeof(handle));
}

void open_peers(CommHandle& h, std::vector<std::string> handles) {
  Comm& c = *h.c;
  if ((int)handles.size() != c.world) throw std::runtime_error("need one IPC handle per rank");
  for (int q = 0; q < c.world; ++q) {
    char* base;
    if (q == c.rank) {
      base = reinterpret_cast<char*>(c.base);
    } else {
      cudaIpcMemHandle_t handle;
      if (handles[q].size() != sizeof(handle)) throw std::runtime_error("bad IPC handle size");
      std::memcpy(&handle, handles[q].data(), sizeof(handle));
      void* p = nullptr;
      cudaError_t err = cudaIpcOpenMemHandle(&p, handle, cudaIpcMemLazyEnablePeerAccess);
      if (err != cudaSuccess) throw std::runtime_error(std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(err));
      c.opened.push_back(p);
      base = reinterpret_cast<char*>(p);
    }
    c.P.grad[q] = reinterpret_cast<float*>(base);
    c.P.param[q] = reinterpret_cast<float*>(base + (size_t)c.n_padded * 4);
    c.P.pad[q] = reinterpret_cast<uint32_t*>(base + (size_t)c.n_padded * 8);
  }
}

// Views of the local gradient and parameter buffers (first n elements).
std::vector<torch::Tensor> local_buffers(const CommHandle& h) {
  const Comm& c = *h.c;
  auto opts = torch::TensorOptions().dtype(torch::kFloat32).device(torch::kCUDA, c.device);
  char* base = reinterpret_cast<char*>(c.base);
  auto g = torch::from_blob(base, {c.n}, [](void*) {}, opts);
  auto p = torch::from_blob(base + (size_t)c.n_padded * 4, {c.n}, [](void*) {}, opts);
  return {g, p};
}

void step(CommHandle& h, torch::Tensor m, torch::Tensor v, torch::Tensor norm_out, int64_t step_index, double lr,
          double b1, double b2, double eps, double wd, double max_norm, int64_t max_iters) {
  Comm& c = *h.c;
  TORCH_CHECK(m.numel() >= c.n_padded && v.numel() >= c.n_padded, "moment buffers must cover the padded size");
  c.epoch += 1;
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  float bias1 = 1.f - (float)std::pow(b1, (double)step_index);
  float bias2 = 1.f - (float)std::pow(b2, (double)step_index);
  float lr_f = (float)lr, b1_f = (float)b1, b2_f = (float)b2, eps_f = (float)eps, wd_f = (float)wd;
  float mn = (float)max_norm;
  long long iters = (long long)max_iters;
  float* mp = m.data_ptr<float>();
  float* vp = v.data_ptr<float>();
  float* np = norm_out.data_ptr<float>();
  int* sp = c.status.data_ptr<int>();
  int world = c.world, rank = c.rank;
  int64_t npad = c.n_padded;
  uint32_t epoch = c.epoch;
  cudaError_t err;
  if (c.oneshot) {
    float* sc = c.scratch;
    void* args[] = {&c.P, &world, &rank, &npad, &sc, &mp, &vp, &epoch, &lr_f, &b1_f, &b2_f, &eps_f, &wd_f,
                    &bias1, &bias2, &mn, &np, &sp, &iters};
    // latency-bound: about two float4 per thread, so the grid-wide syncs span
    // only the CTAs that have work
    const int64_t want = (npad / 4 + 2 * kThreads - 1) / (2 * kThreads);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(c.grid, want));
    err = cudaLaunchCooperativeKernel((void*)oneshot_allreduce_adam_kernel, dim3(grid), dim3(kThreads), args, 0, st);
  } else {
    void* args[] = {&c.P, &world, &rank, &npad, &mp, &vp, &epoch, &lr_f, &b1_f, &b2_f, &eps_f, &wd_f,
                    &bias1, &bias2, &mn, &np, &sp, &iters};
    err = cudaLaunchCooperativeKernel((void*)fused_allreduce_adam_kernel, dim3(c.grid), dim3(kThreads), args, 0, st);
  }
  if (err != cudaSuccess) throw std::runtime_error(std::string("fused all-reduce launch: ") + cudaGetErrorString(err));
}

// In-place: sums[0..nsum) summed, maxes[0..nmax) max-reduced across ranks.
void stats_allreduce(CommHandle& h, torch::Tensor sums, c10::optional<torch::Tensor> maxes, int64_t max_iters) {
  Comm& c = *h.c;
  TORCH_CHECK(sums.is_cuda() && sums.scalar_type() == torch::kFloat64 && sums.is_contiguous(), "sums: CUDA float64");
  const int nsum = (int)sums.numel();
  int nmax = 0;
  if (maxes && maxes->defined()) {
    TORCH_CHECK(maxes->is_cuda() && maxes->scalar_type() == torch::kFloat64 && maxes->is_contiguous(),
                "maxes: CUDA float64");
    nmax = (int)maxes->numel();
  }
  TORCH_CHECK(nsum + nmax <= kMaxStats, "at most 16 values per stats all-reduce");
  auto in = nmax ? torch::cat({sums, *maxes}) : sums.clone();
  auto out = torch::empty_like(in);
  c.stats_epoch += 1;
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  peer_stats_kernel<<<1, 32, 0, st>>>(c.P, c.world, c.rank, in.data_ptr<double>(), out.data_ptr<double>(), nsum,
                                       nmax, c.stats_epoch, c.status.data_ptr<int>(), (long long)max_iters);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "peer_stats_kernel launch failed");
  sums.copy_(out.narrow(0, 0, nsum));
  if (nmax) maxes->copy_(out.narrow(0, nsum, nmax));
}

void broadcast_params(CommHandle& h, int64_t root, int64_t max_iters) {
  Comm& c = *h.c;
  TORCH_CHECK(root >= 0 && root < c.world, "root out of range");
  c.bcast_epoch += 1;
  int world = c.world, rank = c.rank, r = (int)root;
  int64_t npad = c.n_padded;
  uint32_t epoch = c.bcast_epoch;
  int* sp = c.status.data_ptr<int>();
  long long iters = (long long)max_iters;
  void* args[] = {&c.P, &world, &rank, &r, &npad, &epoch, &sp, &iters};
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  cudaError_t err = cudaLaunchCooperativeKernel((void*)peer_broadcast_kernel, dim3(std::min(c.grid, 148)),
                                                dim3(kThreads), args, 0, st);
  if (err != cudaSuccess) throw std::runtime_error(std::string("peer broadcast launch: ") + cudaGetErrorString(err));
}

}  // namespace

void register_comm_ops(py::module& m) {
  py::class_<CommHandle>(m, "PeerComm")
      .def_property_readonly("n_padded", [](const CommHandle& h) { return h.c->n_padded; })
      .def_property_readonly("grid", [](const CommHandle& h) { return h.c->grid; })
      .def_property_readonly("status", [](const CommHandle& h) { return h.c->status; })
      .def_property_readonly("epoch", [](const CommHandle& h) { return h.c->epoch; })
      .def_property_readonly("oneshot", [](const CommHandle& h) { return h.c->oneshot; });
  m.def("peer_comm_create", &create, "allocate the IPC-exported gradient/parameter/signal region",
        py::arg("n"), py::arg("world"), py::arg("rank"), py::arg("oneshot_bytes") = 0);
  m.def("peer_comm_ipc_handle", &ipc_handle);
  m.def("peer_comm_open", &open_peers, "open every peer's region from the exchanged IPC handles");
  m.def("peer_comm_buffers", &local_buffers, "local [grad, param] views");
  m.def("peer_stats_allreduce", &stats_allreduce, "sum / max all-reduce of up to 16 float64 values over peer memory",
        py::arg("comm"), py::arg("sums"), py::arg("maxes") = py::none(), py::arg("max_iters") = 1 << 24);
  m.def("peer_broadcast_params", &broadcast_params, "broadcast the root rank's flat parameters with peer stores",
        py::arg("comm"), py::arg("root") = 0, py::arg("max_iters") = 1 << 24);
  m.def("peer_comm_step", &step, "fused all-reduce + clip + Adam over peer memory (cooperative launch)");
}
