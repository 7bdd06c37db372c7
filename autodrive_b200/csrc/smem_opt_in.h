// Opting a kernel into more than 48 KB of dynamic shared memory
// (cudaFuncSetAttribute) takes effect on the current device only; `opt_in`
// remembers, per device, the largest size already set for a kernel, so a
// process that drives several GPUs sets the attribute on each of them.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

namespace dynsmem {

constexpr int kMaxDevices = 64;

template <typename K>
inline cudaError_t opt_in(K* kernel, size_t bytes, size_t (&done)[kMaxDevices]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (bytes <= done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) done[dev] = bytes;
  return e;
}

}  // namespace dynsmem
