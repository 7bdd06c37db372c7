// Allocation-free C entry point for the fused clip + Adam update.
//
// This entry point has no counterpart in the reference code base. It exists
// for callers that cannot allocate GPU memory themselves: code running inside
// a host framework whose memory pool must not be bypassed, a plugin that gets
// only raw device pointers and a stream, or a process that must keep its
// device footprint fixed once it is running. Such callers cannot hand the
// existing `adam_fused` a scratch tensor, so this variant keeps its scratch
// (the per-block partial sums of squared gradients) in a file-scope device
// array of AD_NOALLOC_MAX_BLOCKS floats (4 KB) instead. Every GPU that loads
// the library reserves that array until the process exits.
//
// Contract:
//   * The caller passes every input and output (parameters, gradients, the
//     two Adam moment buffers, the norm output) as device pointers plus the
//     stream to run on. Nothing is allocated or freed: no cudaMalloc,
//     cudaFree or allocating library call happens on any path.
//   * `blocks` is the number of partial sums (and CTAs) to use; 0 selects the
//     default of 296. More than AD_NOALLOC_MAX_BLOCKS is rejected with
//     AD_NOALLOC_TOO_MANY_BLOCKS before any work is launched.
//   * `stream` must belong to the device that is current on the calling
//     thread: the scratch address used is the current device's.
//   * The first call on each device looks up the device address of the
//     scratch array (cudaGetSymbolAddress) with that device current; make
//     that first call outside any stream capture. The address is cached per
//     device ordinal; it is not valid after cudaDeviceReset, so a call whose
//     launch fails drops the cached address and the next call looks it up
//     again.
//   * A CUDA error left pending by an earlier call on this thread is not
//     attributed to this call: the call launches nothing and returns
//     AD_NOALLOC_PENDING_ERROR (the error stays pending for its owner).
//   * All calls share the one scratch array. Each call overwrites the
//     entries it reads before reading them, so nothing carries over from the
//     previous call, but calls that overlap on the GPU (different streams, or
//     different host threads without ordering) race on the array.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#define AD_NOALLOC_MAX_BLOCKS 1024

enum AdNoallocStatus {
  AD_NOALLOC_OK = 0,
  AD_NOALLOC_BAD_ARGUMENT = 1,
  AD_NOALLOC_TOO_MANY_BLOCKS = 2,
  AD_NOALLOC_CUDA_ERROR = 3,
  AD_NOALLOC_PENDING_ERROR = 4,
};

#ifdef __cplusplus
extern "C" {
#endif

// Global-norm clip (scale = min(1, max_grad_norm / (||g|| + 1e-6)); no clip
// when max_grad_norm <= 0) followed by one Adam step with bias correction
// for step number `step` (>= 1), updating params, exp_avg and exp_avg_sq in
// place and writing the pre-clip gradient norm to grad_norm_out[0].
// Returns an AdNoallocStatus code.
__attribute__((visibility("default"))) int ad_adam_fused_noalloc(
    float* params, const float* grads, float* exp_avg, float* exp_avg_sq, int64_t n, int64_t step,
    float lr, float beta1, float beta2, float eps, float weight_decay, float max_grad_norm, int blocks,
    float* grad_norm_out, cudaStream_t stream);

// Human-readable text for a status code returned by ad_adam_fused_noalloc.
__attribute__((visibility("default"))) const char* ad_adam_fused_noalloc_message(int status);

#ifdef __cplusplus
}
#endif
