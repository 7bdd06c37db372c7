// Host-side TMA tensor maps for 2-D bf16 matrices (shared by the tcgen05
// GEMM and attention kernels).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

namespace tma {

// The driver's tensor-map encoder, looked up through the runtime so the
// extension carries no link-time dependency on libcuda (it imports on hosts
// without a GPU driver).
inline PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    TORCH_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
                    q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled is not available from the CUDA driver");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2-D bf16 tensor map over a row-major [rows][cols] matrix with row stride
// `ld` elements; box = 64 columns x box_rows rows with 128-byte swizzle, so
// one box lands as one 64-column block of a shared-memory SW128 image.
// Rows past the end read as zero.
inline CUtensorMap bf16_sw128(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (ld * 2) % 16 == 0,
              "TMA operands need 16-byte aligned bases and row strides");
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = encoder()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (", (int)r, ")");
  return m;
}

}  // namespace tma
