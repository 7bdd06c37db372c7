// Row LayerNorm for bf16 activations: y = (x - mean) * rstd * gamma + beta
// with fp32 statistics, fp32 affine parameters and a bf16 result, and its
// backward (dx in bf16, dgamma / dbeta in fp32).
//
// One warp per row, rows handed out grid-stride; a row of D = 32 * P columns
// is held in registers (P consecutive columns per lane, loaded and stored as
// 4- to 16-byte vectors), so each element is read once and written once:
// forward 4 bytes per element, backward 6, against 20 / 22 for the
// cast -> fp32 LayerNorm -> cast sequence that mixed-precision autocast runs.
// The mean and variance come from the row held in registers (two passes
// over registers, no E[x^2] - E[x]^2 cancellation). The backward keeps each
// lane's dgamma / dbeta columns in registers over its rows, reduces the
// block's warps in shared memory and writes one partial row per block; the
// host sums the partials.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <algorithm>

namespace py = pybind11;

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

template <int P>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&v)[P]) {
  static_assert(P % 2 == 0, "P must be even");
  uint32_t w[P / 2];
  if constexpr (P % 8 == 0) {
#pragma unroll
    for (int j = 0; j < P / 8; ++j) {
      const uint4 u = reinterpret_cast<const uint4*>(p)[j];
      w[4 * j] = u.x, w[4 * j + 1] = u.y, w[4 * j + 2] = u.z, w[4 * j + 3] = u.w;
    }
  } else if constexpr (P == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    w[0] = u.x, w[1] = u.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
#pragma unroll
  for (int i = 0; i < P / 2; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    v[2 * i] = f.x, v[2 * i + 1] = f.y;
  }
}

template <int P>
__device__ __forceinline__ void store_row(__nv_bfloat16* p, const float (&v)[P]) {
  uint32_t w[P / 2];
#pragma unroll
  for (int i = 0; i < P / 2; ++i) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    w[i] = *reinterpret_cast<const uint32_t*>(&b);
  }
  if constexpr (P % 8 == 0) {
#pragma unroll
    for (int j = 0; j < P / 8; ++j)
      reinterpret_cast<uint4*>(p)[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  } else if constexpr (P == 4) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  }
}

__device__ __forceinline__ float warp_sum(float s) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

template <int P>
__global__ void __launch_bounds__(kThreads, 2)
ln_fwd_kernel(const __nv_bfloat16* __restrict__ x, const float* __restrict__ gamma, const float* __restrict__ beta,
              __nv_bfloat16* __restrict__ y, float* __restrict__ mean_out, float* __restrict__ rstd_out,
              int64_t rows, float eps) {
  constexpr int D = 32 * P;
  const int lane = threadIdx.x & 31;
  const int64_t w0 = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * kWarps;
  float g[P], b[P];
#pragma unroll
  for (int i = 0; i < P; ++i) g[i] = gamma[lane * P + i], b[i] = beta[lane * P + i];
  for (int64_t r = w0; r < rows; r += nw) {
    float v[P];
    load_row<P>(x + r * D + lane * P, v);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < P; ++i) s += v[i];
    const float mean = warp_sum(s) * (1.f / D);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < P; ++i) q += (v[i] - mean) * (v[i] - mean);
    const float rstd = rsqrtf(warp_sum(q) * (1.f / D) + eps);
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] = (v[i] - mean) * rstd * g[i] + b[i];
    store_row<P>(y + r * D + lane * P, v);
    if (lane == 0) mean_out[r] = mean, rstd_out[r] = rstd;
  }
}

template <int P>
__global__ void __launch_bounds__(kThreads, 2)
ln_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
              const float* __restrict__ gamma, const float* __restrict__ mean_in, const float* __restrict__ rstd_in,
              __nv_bfloat16* __restrict__ dx, float* __restrict__ part, int64_t rows) {
  constexpr int D = 32 * P;
  __shared__ float red[kWarps][2][D];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t w0 = (int64_t)blockIdx.x * kWarps + warp;
  const int64_t nw = (int64_t)gridDim.x * kWarps;
  float g[P], dg[P], db[P];
#pragma unroll
  for (int i = 0; i < P; ++i) g[i] = gamma[lane * P + i], dg[i] = 0.f, db[i] = 0.f;
  for (int64_t r = w0; r < rows; r += nw) {
    float xv[P], gv[P];
    load_row<P>(x + r * D + lane * P, xv);
    load_row<P>(dy + r * D + lane * P, gv);
    const float mean = mean_in[r], rstd = rstd_in[r];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const float xh = (xv[i] - mean) * rstd;
      const float gd = gv[i] * g[i];
      dg[i] += gv[i] * xh;
      db[i] += gv[i];
      xv[i] = xh;
      s1 += gd;
      s2 += gd * xh;
    }
    s1 = warp_sum(s1) * (1.f / D);
    s2 = warp_sum(s2) * (1.f / D);
#pragma unroll
    for (int i = 0; i < P; ++i) xv[i] = rstd * (gv[i] * g[i] - s1 - xv[i] * s2);
    store_row<P>(dx + r * D + lane * P, xv);
  }
#pragma unroll
  for (int i = 0; i < P; ++i) red[warp][0][lane * P + i] = dg[i], red[warp][1][lane * P + i] = db[i];
  __syncthreads();
  for (int c = threadIdx.x; c < 2 * D; c += kThreads) {
    const int k = c / D, col = c % D;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w][k][col];
    part[((int64_t)blockIdx.x * 2 + k) * D + col] = s;
  }
}

int blocks_for(int64_t rows) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (rows + kWarps - 1) / kWarps;
  return (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)sms * 8));
}

void check_common(const torch::Tensor& x, const torch::Tensor& gamma, int64_t D) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.is_contiguous(),
              "layer_norm_bf16: x must be a contiguous CUDA bf16 [rows, D] tensor");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "layer_norm_bf16: x must be 16-byte aligned");
  TORCH_CHECK(D == 64 || D == 128 || D == 256 || D == 512, "layer_norm_bf16: D must be 64, 128, 256 or 512");
  TORCH_CHECK(gamma.is_cuda() && gamma.scalar_type() == torch::kFloat32 && gamma.numel() == D && gamma.is_contiguous(),
              "layer_norm_bf16: weight must be fp32 [D]");
}

#define AD_LN_DISPATCH(D, ...)                                  \
  switch (D) {                                                  \
    case 64: { constexpr int P = 2; __VA_ARGS__; } break;       \
    case 128: { constexpr int P = 4; __VA_ARGS__; } break;      \
    case 256: { constexpr int P = 8; __VA_ARGS__; } break;      \
    default: { constexpr int P = 16; __VA_ARGS__; } break;      \
  }

std::vector<torch::Tensor> layer_norm_bf16_fwd(torch::Tensor x, torch::Tensor gamma, torch::Tensor beta, double eps) {
  const int64_t rows = x.size(0), D = x.size(1);
  check_common(x, gamma, D);
  TORCH_CHECK(beta.is_cuda() && beta.scalar_type() == torch::kFloat32 && beta.numel() == D && beta.is_contiguous(),
              "layer_norm_bf16: bias must be fp32 [D]");
  auto y = torch::empty_like(x);
  auto mean = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  auto rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  if (rows == 0) return {y, mean, rstd};
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  const int grid = blocks_for(rows);
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr<at::BFloat16>());
  AD_LN_DISPATCH(D, ln_fwd_kernel<P><<<grid, kThreads, 0, st>>>(xp, gamma.data_ptr<float>(), beta.data_ptr<float>(), yp,
                                                               mean.data_ptr<float>(), rstd.data_ptr<float>(), rows,
                                                               (float)eps))
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "layer_norm_bf16 forward launch failed");
  return {y, mean, rstd};
}

// Returns dx (bf16), dgamma, dbeta (fp32).
std::vector<torch::Tensor> layer_norm_bf16_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor gamma,
                                               torch::Tensor mean, torch::Tensor rstd) {
  const int64_t rows = x.size(0), D = x.size(1);
  check_common(x, gamma, D);
  check_common(dy, gamma, D);
  TORCH_CHECK(dy.sizes() == x.sizes(), "layer_norm_bf16: dy and x differ in shape");
  TORCH_CHECK(mean.scalar_type() == torch::kFloat32 && rstd.scalar_type() == torch::kFloat32 &&
                  mean.numel() == rows && rstd.numel() == rows && mean.is_contiguous() && rstd.is_contiguous(),
              "layer_norm_bf16: mean / rstd must be fp32 [rows]");
  auto dx = torch::empty_like(x);
  if (rows == 0) return {dx, torch::zeros({D}, gamma.options()), torch::zeros({D}, gamma.options())};
  const int grid = blocks_for(rows);
  auto part = torch::empty({grid, 2, D}, gamma.options());
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  const auto* dyp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr<at::BFloat16>());
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>());
  auto* dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr<at::BFloat16>());
  AD_LN_DISPATCH(D, ln_bwd_kernel<P><<<grid, kThreads, 0, st>>>(dyp, xp, gamma.data_ptr<float>(), mean.data_ptr<float>(),
                                                               rstd.data_ptr<float>(), dxp, part.data_ptr<float>(), rows))
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "layer_norm_bf16 backward launch failed");
  auto sums = part.sum(0);
  return {dx, sums[0], sums[1]};
}

}  // namespace

void register_layernorm_ops(py::module& m) {
  m.def("layer_norm_bf16_fwd", &layer_norm_bf16_fwd, "bf16 LayerNorm forward (fp32 statistics): y, mean, rstd",
        py::arg("x"), py::arg("weight"), py::arg("bias"), py::arg("eps"));
  m.def("layer_norm_bf16_bwd", &layer_norm_bf16_bwd, "bf16 LayerNorm backward: dx, dweight, dbias",
        py::arg("dy"), py::arg("x"), py::arg("weight"), py::arg("mean"), py::arg("rstd"));
}
