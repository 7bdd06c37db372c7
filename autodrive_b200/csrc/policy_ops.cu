// Training-side kernels (sm_100a):
//
//   gae_scan       reverse generalised-advantage scan, one thread per rollout
//                  column; also accumulates sum(adv), sum(adv^2), count for
//                  the global advantage normalisation so the statistics need
//                  no extra pass (reference: frc_defense/tensor_training_runtime.py:303-316)
//   adam_fused     global gradient norm, clip and Adam update over one flat
//                  fp32 parameter buffer in two launches with no host sync
//                  (reference: torch clip_grad_norm_ + Adam, tensor_training_ppo.py:433-434)
//
// CPU tensors run the same arithmetic in plain loops (host twins).
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>

#include <cmath>
#include <stdexcept>

namespace py = pybind11;

namespace {

constexpr int kNormBlocks = 296;   // 2 per SM on a 148-SM B200
constexpr int kNormThreads = 512;

__global__ void gae_kernel(const float* __restrict__ rew, const uint8_t* __restrict__ done,
                           const uint8_t* __restrict__ trunc, const float* __restrict__ val,
                           const float* __restrict__ next_val, float* __restrict__ adv, int T, int B,
                           float gamma, float lam, double* __restrict__ stats) {
  int b = blockIdx.x * blockDim.x + threadIdx.x;
  double s1 = 0., s2 = 0.;
  if (b < B) {
    float last = 0.f;
    for (int t = T - 1; t >= 0; --t) {
      size_t k = (size_t)t * B + b;
      float nonterminal = done[k] ? 0.f : 1.f;
      float delta = rew[k] + gamma * next_val[k] * nonterminal - val[k];
      float cont = (done[k] | trunc[k]) ? 0.f : 1.f;
      last = delta + gamma * lam * cont * last;
      adv[k] = last;
      s1 += last;
      s2 += (double)last * last;
    }
  }
  // block reduce then one atomic per block
  for (int o = 16; o > 0; o >>= 1) {
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    s2 += __shfl_xor_sync(0xffffffffu, s2, o);
  }
  __shared__ double r1[32], r2[32];
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    r1[warp] = s1;
    r2[warp] = s2;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0., c = 0.;
    for (int w = 0; w < (int)(blockDim.x + 31) / 32; ++w) {
      a += r1[w];
      c += r2[w];
    }
    atomicAdd(stats, a);
    atomicAdd(stats + 1, c);
    if (blockIdx.x == 0) stats[2] = (double)T * (double)B;
  }
}

void gae(torch::Tensor rew, torch::Tensor done, torch::Tensor trunc, torch::Tensor val,
         torch::Tensor next_val, torch::Tensor adv, double gamma, double lam, torch::Tensor stats) {
  TORCH_CHECK(rew.dim() == 2 && rew.scalar_type() == torch::kFloat32, "rewards must be float32 [T, B]");
  TORCH_CHECK(done.scalar_type() == torch::kUInt8 && trunc.scalar_type() == torch::kUInt8, "flags must be uint8");
  TORCH_CHECK(stats.scalar_type() == torch::kFloat64 && stats.numel() >= 3, "stats must be float64 [3]");
  for (auto* t : {&rew, &done, &trunc, &val, &next_val, &adv})
    TORCH_CHECK(t->is_contiguous() && t->sizes() == rew.sizes(), "GAE inputs must be contiguous [T, B]");
  const int T = rew.size(0), B = rew.size(1);
  if (rew.is_cuda()) {
    auto st = c10::cuda::getCurrentCUDAStream().stream();
    cudaMemsetAsync(stats.data_ptr<double>(), 0, 2 * sizeof(double), st);
    gae_kernel<<<(B + 255) / 256, 256, 0, st>>>(rew.data_ptr<float>(), done.data_ptr<uint8_t>(),
                                                trunc.data_ptr<uint8_t>(), val.data_ptr<float>(),
                                                next_val.data_ptr<float>(), adv.data_ptr<float>(), T, B,
                                                (float)gamma, (float)lam, stats.data_ptr<double>());
    TORCH_CHECK(cudaGetLastError() == cudaSuccess, "gae_kernel launch failed");
    return;
  }
  const float* r = rew.data_ptr<float>();
  const uint8_t* d = done.data_ptr<uint8_t>();
  const uint8_t* tr = trunc.data_ptr<uint8_t>();
  const float* v = val.data_ptr<float>();
  const float* nv = next_val.data_ptr<float>();
  float* a = adv.data_ptr<float>();
  double s1 = 0., s2 = 0.;
  for (int b = 0; b < B; ++b) {
    float last = 0.f;
    for (int t = T - 1; t >= 0; --t) {
      size_t k = (size_t)t * B + b;
      float delta = r[k] + (float)gamma * nv[k] * (d[k] ? 0.f : 1.f) - v[k];
      last = delta + (float)gamma * (float)lam * ((d[k] | tr[k]) ? 0.f : 1.f) * last;
      a[k] = last;
      s1 += last;
      s2 += (double)last * last;
    }
  }
  double* s = stats.data_ptr<double>();
  s[0] = s1;
  s[1] = s2;
  s[2] = (double)T * B;
}

// ---------------------------------------------------------------------------
// Fused clip + Adam over a flat buffer
// ---------------------------------------------------------------------------
__global__ void sumsq_partial_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ partial) {
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float x = g[i];
    acc += x * x;
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float red[32];
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) t += red[w];
    partial[blockIdx.x] = t;
  }
}

__global__ void adam_apply_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                  float* __restrict__ v, int64_t n, const float* __restrict__ partial, int nparts,
                                  float max_norm, float lr, float b1, float b2, float eps, float wd,
                                  float bias1, float bias2, float* __restrict__ norm_out) {
  __shared__ float scale_s;
  if (threadIdx.x < 32) {
    float t = 0.f;
    for (int k = threadIdx.x; k < nparts; k += 32) t += partial[k];
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) {
      float norm = sqrtf(t);
      scale_s = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
      if (blockIdx.x == 0 && norm_out) *norm_out = norm;
    }
  }
  __syncthreads();
  const float scale = scale_s;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float gi = g[i] * scale + wd * p[i];
    float mi = b1 * m[i] + (1.f - b1) * gi;
    float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    float denom = sqrtf(vi / bias2) + eps;
    p[i] -= lr * (mi / bias1) / denom;
  }
}

// Returns nothing; writes the pre-clip gradient norm into norm_out[0].
void adam_fused(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, torch::Tensor partial,
                torch::Tensor norm_out, int64_t step, double lr, double b1, double b2, double eps, double wd,
                double max_norm) {
  TORCH_CHECK(p.scalar_type() == torch::kFloat32 && p.is_contiguous(), "params must be contiguous float32");
  for (auto* t : {&g, &m, &v}) TORCH_CHECK(t->is_contiguous() && t->numel() == p.numel(), "Adam buffer mismatch");
  const int64_t n = p.numel();
  const float bias1 = 1.f - (float)std::pow(b1, (double)step);
  const float bias2 = 1.f - (float)std::pow(b2, (double)step);
  if (p.is_cuda()) {
    TORCH_CHECK(partial.numel() >= kNormBlocks, "partial buffer too small");
    auto st = c10::cuda::getCurrentCUDAStream().stream();
    sumsq_partial_kernel<<<kNormBlocks, kNormThreads, 0, st>>>(g.data_ptr<float>(), n, partial.data_ptr<float>());
    adam_apply_kernel<<<kNormBlocks, kNormThreads, 0, st>>>(
        p.data_ptr<float>(), g.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), n,
        partial.data_ptr<float>(), kNormBlocks, (float)max_norm, (float)lr, (float)b1, (float)b2, (float)eps,
        (float)wd, bias1, bias2, norm_out.data_ptr<float>());
    TORCH_CHECK(cudaGetLastError() == cudaSuccess, "adam kernels launch failed");
    return;
  }
  float* P = p.data_ptr<float>();
  const float* G = g.data_ptr<float>();
  float* M = m.data_ptr<float>();
  float* V = v.data_ptr<float>();
  double ss = 0.;
  for (int64_t i = 0; i < n; ++i) ss += (double)G[i] * G[i];
  float norm = (float)std::sqrt(ss);
  float scale = max_norm > 0. ? std::fmin(1.f, (float)max_norm / (norm + 1e-6f)) : 1.f;
  for (int64_t i = 0; i < n; ++i) {
    float gi = G[i] * scale + (float)wd * P[i];
    M[i] = (float)b1 * M[i] + (1.f - (float)b1) * gi;
    V[i] = (float)b2 * V[i] + (1.f - (float)b2) * gi * gi;
    P[i] -= (float)lr * (M[i] / bias1) / (std::sqrt(V[i] / bias2) + (float)eps);
  }
  norm_out.data_ptr<float>()[0] = norm;
}

}  // namespace

void register_policy_ops(py::module& m) {
  m.def("gae", &gae, "generalised advantage estimation with fused advantage statistics");
  m.def("adam_fused", &adam_fused, "global-norm clip + Adam over one flat parameter buffer");
  m.attr("ADAM_NORM_BLOCKS") = kNormBlocks;
}
