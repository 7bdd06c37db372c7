// Allocation-free fused clip + Adam (see noalloc_adam.h for who needs it and
// the contract). Same arithmetic as `adam_fused` in policy_ops.cu, but the
// partial sums live in a static device array rather than a caller tensor.
#include "noalloc_adam.h"

#include <cmath>
#include <mutex>

namespace {

constexpr int kThreads = 512;
constexpr int kDefaultBlocks = 296;
constexpr int kMaxDevices = 64;

// Scratch: one partial sum of squared gradients per CTA.
static __device__ __align__(256) float g_partials[AD_NOALLOC_MAX_BLOCKS];

// Device address of g_partials per device ordinal, looked up once per device.
float* g_partials_addr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

__global__ void noalloc_sumsq_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ partial) {
  float acc = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float x = g[i];
    acc += x * x;
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float red[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) t += red[w];
    partial[blockIdx.x] = t;
  }
}

__global__ void noalloc_apply_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                     float* __restrict__ v, int64_t n, const float* __restrict__ partial,
                                     int nparts, float max_norm, float lr, float b1, float b2, float eps,
                                     float wd, float bias1, float bias2, float* __restrict__ norm_out) {
  __shared__ float scale_s;
  if (threadIdx.x < 32) {
    float t = 0.f;
    for (int k = threadIdx.x; k < nparts; k += 32) t += partial[k];
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) {
      const float norm = sqrtf(t);
      scale_s = max_norm > 0.f ? fminf(1.f, max_norm / (norm + 1e-6f)) : 1.f;
      if (blockIdx.x == 0 && norm_out) *norm_out = norm;
    }
  }
  __syncthreads();
  const float scale = scale_s;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = g[i] * scale + wd * p[i];
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    p[i] -= lr * (mi / bias1) / (sqrtf(vi / bias2) + eps);
  }
}

// Device address of the scratch array on the current device (set-up on first use).
int scratch_for_current_device(float** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AD_NOALLOC_CUDA_ERROR;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_partials_addr[dev] == nullptr) {
    float* ptr = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&ptr), g_partials) != cudaSuccess || ptr == nullptr)
      return AD_NOALLOC_CUDA_ERROR;
    g_partials_addr[dev] = ptr;
  }
  *out = g_partials_addr[dev];
  return AD_NOALLOC_OK;
}

// A failed launch may mean the device was reset (the cached address is then
// stale): drop the current device's cached address so the next call looks it
// up again.
int forget_scratch_after_failure() {
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    g_partials_addr[dev] = nullptr;
  }
  return AD_NOALLOC_CUDA_ERROR;
}

}  // namespace

extern "C" int ad_adam_fused_noalloc(float* params, const float* grads, float* exp_avg, float* exp_avg_sq,
                                     int64_t n, int64_t step, float lr, float beta1, float beta2, float eps,
                                     float weight_decay, float max_grad_norm, int blocks, float* grad_norm_out,
                                     cudaStream_t stream) {
  if (n < 0 || step < 1 || (n > 0 && (!params || !grads || !exp_avg || !exp_avg_sq)) || !grad_norm_out)
    return AD_NOALLOC_BAD_ARGUMENT;
  if (blocks < 0) return AD_NOALLOC_BAD_ARGUMENT;
  if (blocks == 0) blocks = kDefaultBlocks;
  if (blocks > AD_NOALLOC_MAX_BLOCKS) return AD_NOALLOC_TOO_MANY_BLOCKS;
  if (cudaPeekAtLastError() != cudaSuccess) return AD_NOALLOC_PENDING_ERROR;
  float* partial = nullptr;
  int status = scratch_for_current_device(&partial);
  if (status != AD_NOALLOC_OK) return status;
  const float bias1 = 1.f - (float)std::pow((double)beta1, (double)step);
  const float bias2 = 1.f - (float)std::pow((double)beta2, (double)step);
  noalloc_sumsq_kernel<<<blocks, kThreads, 0, stream>>>(grads, n, partial);
  if (cudaGetLastError() != cudaSuccess) return forget_scratch_after_failure();
  noalloc_apply_kernel<<<blocks, kThreads, 0, stream>>>(params, grads, exp_avg, exp_avg_sq, n, partial, blocks,
                                                        max_grad_norm, lr, beta1, beta2, eps, weight_decay,
                                                        bias1, bias2, grad_norm_out);
  if (cudaGetLastError() != cudaSuccess) return forget_scratch_after_failure();
  return AD_NOALLOC_OK;
}

extern "C" const char* ad_adam_fused_noalloc_message(int status) {
  switch (status) {
    case AD_NOALLOC_OK: return "ok";
    case AD_NOALLOC_BAD_ARGUMENT:
      return "bad argument: null pointer, negative size, negative block count or step < 1";
    case AD_NOALLOC_TOO_MANY_BLOCKS:
      return "blocks exceeds AD_NOALLOC_MAX_BLOCKS (1024): the static scratch array holds 1024 partial sums";
    case AD_NOALLOC_CUDA_ERROR: return "CUDA error while locating the scratch array or launching the kernels";
    case AD_NOALLOC_PENDING_ERROR:
      return "an earlier CUDA call on this thread left an error pending; nothing was launched";
    default: return "unknown status";
  }
}
