// General bf16 tensor-core GEMM for sm_100a: C[M,N] = A[M,K] * B[N,K]^T with
// fp32 accumulation in TMEM and a fused bias + activation epilogue.
//
// Either operand may be stored K-major (row-major [rows][K]) or MN-major
// (row-major [K][rows], i.e. the transpose), selected per call, so the three
// GEMMs of a linear layer need no transposed copies:
//   forward  Y  = X W^T      A = X  (K-major),  B = W  (K-major)
//   dX       dX = dY W       A = dY (K-major),  B = W  (MN-major)
//   dW       dW = dY^T X     A = dY (MN-major), B = X  (MN-major)
//
// Persistent kernel: one CTA per SM (at most one per work item) walks the
// 128 x BN output tiles (BN = 256 for wide outputs of long contractions with
// A read K-major, 128 otherwise; x split-K slices) in a static round-robin, N tiles fastest so
// the CTAs running at the same time share A row blocks in L2.
// 320 threads:
//   warp 0  TMA producer: 2-D tiled loads (128-byte swizzle) of the A and B
//           tiles of each 64-deep K step into a 4-stage shared-memory ring
//           that runs continuously across tiles;
//   warp 1  allocates 2 BN TMEM columns (two BN-column fp32 accumulators);
//           one lane issues 4 tcgen05.mma per K step into the accumulator of
//           the current tile, commits each stage back to the producer and
//           the finished accumulator to the epilogue;
//   warps 2-9 epilogue, two per TMEM lane quadrant, each owning half of the
//           column chunks: both of its tcgen05.ld loads in flight at once, the
//           accumulator handed back to the MMA warp as soon as it is read,
//           then + bias, activation, fp32 or bf16 stores with bounds checks.
// With two accumulators the epilogue of tile i overlaps the loads and MMAs
// of tile i+1. Out-of-range tile parts are zero-filled by the TMA unit.
// Every mbarrier wait is bounded in wall-clock time (`wait_ns`, 2 s by
// default); a wait that runs out sets a bit in a device status word
// (1 producer/stage free, 2 MMA/stage loaded, 4 epilogue/accumulator full,
// 8 MMA/accumulator free) and a shared failure flag that stops the other
// roles. Before the CTA frees its TMEM and exits it drains what it already
// issued: the producer waits for its last loads to land and the MMA warp
// commits its issued MMAs to a drain barrier and waits for it (each wait
// bounded by 200 ms; a drain that gives up sets bit 16 or 32).
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

#include "tc_sm100.h"
#include "tma_map.h"
#include "smem_opt_in.h"

namespace py = pybind11;

namespace {

// Output tiles are 128 rows x BN columns, BN = 128 or 256 (a template
// parameter; 256 halves the A re-reads and tile hand-offs on wide outputs).
constexpr int kBM = 128, kBK = 64, kStages = 4;
constexpr int kEpiWarps = 8;                    // two warps per TMEM lane quadrant
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kTileBytes = 128 * 128;        // the 128 x 64 bf16 A tile of one K step
constexpr uint64_t kDrainNs = 200000000ull;       // 200 ms for in-flight copies / MMAs after a failure
template <int BN> __host__ __device__ constexpr uint32_t stage_bytes() { return kTileBytes + (uint32_t)BN * 128u; }
template <int BN> __host__ __device__ constexpr uint32_t smem_bytes() { return kStages * stage_bytes<BN>() + 1024 + 256; }

struct GemmArgs {
  int M, N, K;
  float* c_f32;
  __nv_bfloat16* c_bf16;
  int64_t ldc;
  const float* bias;   // [N] or null
  int act;             // 0 none, 1 tanh, 2 relu, 3 gelu (tanh form), 4 gelu (erf form),
                       // 5 times GELU'(aux_in) (erf form; the backward of act 4)
  __nv_bfloat16* aux_out;        // act 4: the pre-activation, bf16, same layout as C (or null)
  const __nv_bfloat16* aux_in;   // act 5: the pre-activation the gradient is scaled by
  int accumulate;      // C += result (fp32 output only)
  int k_steps;         // K steps (of kBK) per split-K slice
  int splits;          // split-K slices (1: no split)
  int64_t split_stride;  // elements between the fp32 partial outputs of two slices
  int* status;
  uint64_t wait_ns;    // limit of every pipeline wait
};

__device__ __forceinline__ float apply_act(float x, int act) {
  switch (act) {
    case 1: return tanhf(x);
    case 2: return fmaxf(x, 0.f);
    case 3: {
      const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
      return 0.5f * x * (1.f + tanhf(u));
    }
    default: return x;
  }
}

// GELU (erf form) z Phi(z) and its derivative Phi(z) + z phi(z), with
// erf from Abramowitz & Stegun, Handbook of Mathematical Functions, formula
// 7.1.26: erf(x) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-x^2),
// t = 1 / (1 + p x), x >= 0, |error| <= 1.5e-7 (odd extension for x < 0).
// For x = |z| / sqrt(2) the factor exp(-x^2) = exp(-z^2 / 2) is also the
// normal density's, so the backward takes one exponential and one reciprocal.
struct PhiParts { float cdf, pdf; };   // Phi(z), phi(z)
__device__ __forceinline__ PhiParts normal_parts(float z) {
  const float x = fabsf(z) * 0.7071067811865476f;
  const float t = __fdividef(1.f, fmaf(0.3275911f, x, 1.f));
  const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f),
                                      -0.284496736f), 0.254829592f);
  const float e = exp2f(-0.7213475204444817f * z * z);   // exp(-z^2 / 2) = 2^(-z^2 / (2 ln 2))
  const float erf_x = 1.f - poly * e;
  return PhiParts{0.5f * (1.f + copysignf(erf_x, z)), 0.3989422804014327f * e};
}
__device__ __forceinline__ float gelu_erf(float x) { return x * normal_parts(x).cdf; }
__device__ __forceinline__ float gelu_erf_grad(float z) {
  const PhiParts q = normal_parts(z);
  return q.cdf + z * q.pdf;
}

// Work item w -> (m0, n0, split slice z); N tiles fastest.
struct TileCoord { int m0, n0, z; };
__device__ __forceinline__ TileCoord tile_of(int w, int tiles_n, int tiles_m, int bn) {
  TileCoord t;
  t.n0 = (w % tiles_n) * bn;
  const int r = w / tiles_n;
  t.m0 = (r % tiles_m) * kBM;
  t.z = r / tiles_m;
  return t;
}

// One accumulator's 32 x 32 chunk of this thread's row: bias, activation and
// the store (16-byte vectors for a full aligned chunk, scalars otherwise).
// The GELU (erf) epilogues, compiled into their own kernel instantiations so
// the plain GEMM keeps its register budget: act 4 adds the bias, keeps the
// pre-activation in aux_out and applies GELU; act 5 scales the product by
// GELU' of the pre-activation aux_in. Then the common store.
__device__ __forceinline__ void gelu_epilogue(const GemmArgs& g, float (&v)[32], int row, int c0) {
  const int64_t off0 = (int64_t)row * g.ldc + c0;
// GELU (erf) forward with the pre-activation kept, or its backward
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] += (g.bias && c0 + i < g.N ? g.bias[c0 + i] : 0.f);
  const bool vec_aux = c0 + 32 <= g.N && (g.ldc % 8) == 0;   // aux bases are 16-byte aligned (host check)
  if (g.act == 4) {
    if (g.aux_out) {
      if (vec_aux) {
        uint4* dst = reinterpret_cast<uint4*>(g.aux_out + off0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 u;
          uint32_t* w = &u.x;
#pragma unroll
          for (int hh = 0; hh < 4; ++hh) {
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[8 * j + 2 * hh], v[8 * j + 2 * hh + 1]);
            w[hh] = *reinterpret_cast<const uint32_t*>(&b2);
          }
          dst[j] = u;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (c0 + i < g.N) g.aux_out[off0 + i] = __float2bfloat16_rn(v[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
  } else {
    float zv[32];
    if (vec_aux) {
      const uint4* src = reinterpret_cast<const uint4*>(g.aux_in + off0);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 u = src[j];
        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int hh = 0; hh < 4; ++hh) {
          const float2 f = __bfloat1622float2(b2[hh]);
          zv[8 * j + 2 * hh] = f.x;
          zv[8 * j + 2 * hh + 1] = f.y;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) zv[i] = c0 + i < g.N ? __bfloat162float(g.aux_in[off0 + i]) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] *= gelu_erf_grad(zv[i]);
  }
}

template <bool GELU>
__device__ __forceinline__ void store_chunk(const GemmArgs& g, float (&v)[32], int row, int c0, int z) {
  const int64_t off0 = (int64_t)z * g.split_stride + (int64_t)row * g.ldc + c0;
  if constexpr (GELU) {
    gelu_epilogue(g, v, row, c0);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = apply_act(v[i] + (g.bias && c0 + i < g.N ? g.bias[c0 + i] : 0.f), g.act);
  }
  // each thread owns one output row: a full in-bounds 32-column chunk goes
  // out as 16-byte vector stores (64 B bf16 / 128 B fp32 per row)
  const bool vec = c0 + 32 <= g.N && (g.ldc % 8) == 0 &&
                   ((reinterpret_cast<uintptr_t>(g.c_f32 ? (void*)g.c_f32 : (void*)g.c_bf16)) & 15) == 0;
  if (vec && g.c_f32) {
    float4* dst = reinterpret_cast<float4*>(g.c_f32 + off0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 x = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      if (g.accumulate) {
        const float4 o = dst[j];
        x.x += o.x, x.y += o.y, x.z += o.z, x.w += o.w;
      }
      dst[j] = x;
    }
  } else if (vec) {
    uint4* dst = reinterpret_cast<uint4*>(g.c_bf16 + off0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 u;
      uint32_t* w = &u.x;
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const __nv_bfloat162 b2 = __floats2bfloat162_rn(v[8 * j + 2 * h], v[8 * j + 2 * h + 1]);
        w[h] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      dst[j] = u;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (c0 + i < g.N) {
        if (g.c_f32) g.c_f32[off0 + i] = g.accumulate ? g.c_f32[off0 + i] + v[i] : v[i];
        else g.c_bf16[off0 + i] = __float2bfloat16_rn(v[i]);
      }
    }
  }
}

template <bool A_MN, bool B_MN, bool GELU, int BN>
__global__ void __launch_bounds__(kThreads, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, const GemmArgs g) {
  constexpr uint32_t kStageBytes = stage_bytes<BN>();
  constexpr uint32_t kAccCols = BN;               // one fp32 accumulator: 128 lanes x BN columns
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* misc = smem + kStages * kStageBytes;
  const uint32_t full0 = tc::smem_u32(misc);             // kStages mbarriers: stage loaded
  const uint32_t empty0 = full0 + 8 * kStages;           // kStages mbarriers: stage consumed
  const uint32_t tfull0 = empty0 + 8 * kStages;          // 2 mbarriers: accumulator complete
  const uint32_t tempty0 = tfull0 + 16;                  // 2 mbarriers: accumulator read out
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(misc + 8 * (2 * kStages + 4));
  int* s_fail = reinterpret_cast<int*>(misc + 8 * (2 * kStages + 4) + 8);
  const uint32_t drain = tc::smem_u32(misc + 8 * (2 * kStages + 4) + 16);  // MMA drain after a failure
  volatile int* fail = s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = (g.N + BN - 1) / BN, tiles_m = (g.M + kBM - 1) / kBM;
  const int total = tiles_n * tiles_m * g.splits;
  const int KT_all = (g.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(full0 + 8 * s, 1);
      tc::mbar_init(empty0 + 8 * s, 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(tfull0 + 8 * a, 1);
      tc::mbar_init(tempty0 + 8 * a, 32 * kEpiWarps);   // every epilogue thread arrives
    }
    tc::mbar_init(drain, 1);
    tc::mbar_init_fence();
    *s_fail = 0;
  }
  if (warp == 1) {
    tc::tmem_alloc(tc::smem_u32(s_tmem), 2 * kAccCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (warp == 0 && lane == 0) {
    // ---- TMA producer: one ring position per K step, across all tiles ----
    uint32_t it = 0;
    for (int w = blockIdx.x; w < total && !*fail; w += gridDim.x) {
      const TileCoord t = tile_of(w, tiles_n, tiles_m, BN);
      const int kb = t.z * g.k_steps, ke = min(KT_all, kb + g.k_steps);
      for (int kt = kb; kt < ke; ++kt, ++it) {
        const uint32_t s = it % kStages;
        if (it >= kStages && !tc::mbar_wait(empty0 + 8 * s, ((it / kStages) - 1) & 1, g.wait_ns)) {
          atomicOr(g.status, 1);
          atomicExch(s_fail, 1);
          break;
        }
        if (*fail) break;
        const uint32_t sa = tc::smem_u32(smem + s * kStageBytes);
        const uint32_t sb = sa + kTileBytes;
        const uint32_t full = full0 + 8 * s;
        tc::mbar_arrive_expect_tx(full, kStageBytes);
        const int k0 = kt * kBK;
        if (A_MN) {
          tc::tma_load_2d(sa, &ta, t.m0, k0, full);
          tc::tma_load_2d(sa + kTileBytes / 2, &ta, t.m0 + 64, k0, full);
        } else {
          tc::tma_load_2d(sa, &ta, k0, t.m0, full);
        }
        if (B_MN) {   // BN / 64 boxes of 64 N columns x 64 K rows
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tc::tma_load_2d(sb + j * (kTileBytes / 2), &tb, t.n0 + 64 * j, k0, full);
        } else {
          tc::tma_load_2d(sb, &tb, k0, t.n0, full);
        }
      }
    }
    if (*fail) {
      // `it` loads were issued; every stage's latest one may still be in
      // flight (earlier ones were consumed). Wait for them to land.
      for (uint32_t i = it > (uint32_t)kStages ? it - kStages : 0u; i < it; ++i)
        if (!tc::mbar_wait(full0 + 8 * (i % kStages), (i / kStages) & 1, kDrainNs)) atomicOr(g.status, 16);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer: tile lt accumulates into TMEM columns (lt & 1) * 128 ----
    const uint32_t id = tc::idesc_bf16(kBM, BN, A_MN, B_MN);
    uint32_t it = 0;
    int lt = 0;
    for (int w = blockIdx.x; w < total && !*fail; w += gridDim.x, ++lt) {
      const TileCoord t = tile_of(w, tiles_n, tiles_m, BN);
      const int kb = t.z * g.k_steps, ke = min(KT_all, kb + g.k_steps);
      const int acc = lt & 1;
      if (lt >= 2 && !tc::mbar_wait(tempty0 + 8 * acc, ((lt >> 1) - 1) & 1, g.wait_ns)) {
        atomicOr(g.status, 8);
        atomicExch(s_fail, 1);
        break;
      }
      tc::tc_fence_after();
      const uint32_t d = tmem + acc * kAccCols;
      bool ok = true;
      for (int kt = kb; kt < ke; ++kt, ++it) {
        const uint32_t s = it % kStages;
        if (!tc::mbar_wait(full0 + 8 * s, (it / kStages) & 1, g.wait_ns)) {
          atomicOr(g.status, 2);
          atomicExch(s_fail, 1);
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t sa = tc::smem_u32(smem + s * kStageBytes);
        const uint32_t sb = sa + kTileBytes;
#pragma unroll
        for (int ks = 0; ks < kBK / 16; ++ks) {
          const uint64_t da = A_MN ? tc::desc_mnmajor(sa, kBK, ks) : tc::desc_kmajor(sa, kBM, ks);
          const uint64_t db = B_MN ? tc::desc_mnmajor(sb, kBK, ks) : tc::desc_kmajor(sb, BN, ks);
          tc::mma_bf16(d, da, db, id, kt > kb || ks > 0);
        }
        tc::mma_commit(empty0 + 8 * s);   // stage free once these MMAs have read it
      }
      tc::mma_commit(tfull0 + 8 * acc);   // accumulator complete (or nothing issued)
      if (!ok) break;
    }
    if (*fail) {
      // MMAs issued so far may still read shared memory / write TMEM
      tc::mma_commit(drain);
      if (!tc::mbar_wait(drain, 0, kDrainNs)) atomicOr(g.status, 32);
    }
  }

  if (warp >= 2) {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its quadrant) and
    // the column chunks of its half (two warps per quadrant); both chunks'
    // loads are in flight together, and the accumulator is handed back to the
    // MMA warp before the stores
    const int q = warp & 3;
    const int half = (warp - 2) >> 2;
    constexpr int kChunks = BN / 32 / 2;  // chunks per warp (2 or 4)
    static_assert(kChunks % 2 == 0, "epilogue reads chunks in pairs");
    int lt = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++lt) {
      const TileCoord t = tile_of(w, tiles_n, tiles_m, BN);
      const int acc = lt & 1;
      const bool got = tc::mbar_wait(tfull0 + 8 * acc, (lt >> 1) & 1, g.wait_ns);
      if (!got) {
        atomicOr(g.status, 4);
        atomicExch(s_fail, 1);
      }
      if (!got || *fail) break;
      tc::tc_fence_after();
      const int row = t.m0 + 32 * q + lane;
      const uint32_t base = tmem + acc * kAccCols + ((uint32_t)(32 * q) << 16);
      // two chunks in flight at a time (a 256-wide tile's four would spill);
      // the accumulator is handed back once its last chunks are read
#pragma unroll
      for (int k0 = 0; k0 < kChunks; k0 += 2) {
        float v[2][32];
#pragma unroll
        for (int k = 0; k < 2; ++k) tc::tmem_ld32_issue(base + 32 * (2 * (k0 + k) + half), v[k]);
        tc::tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 2; ++k) tc::tmem_regs_ready(v[k]);
        if (k0 + 2 >= kChunks) {
          tc::tc_fence_before();
          tc::mbar_arrive(tempty0 + 8 * acc);   // accumulator read out: the MMA warp may reuse it
        }
        if (row < g.M) {
#pragma unroll
          for (int k = 0; k < 2; ++k)
            store_chunk<GELU>(g, v[k], row, t.n0 + 32 * (2 * (k0 + k) + half), t.z);
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 2 * kAccCols);
  }
}

CUtensorMap make_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  return tma::bf16_sw128(ptr, rows, cols, ld, box_rows);
}

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  TORCH_CHECK(cudaGetDevice(&dev) == cudaSuccess, "cudaGetDevice failed");
  TORCH_CHECK(dev >= 0 && dev < 64, "tc_gemm: device index out of range");
  if (!counts[dev])
    TORCH_CHECK(cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev) == cudaSuccess,
                "cudaDeviceGetAttribute(multiProcessorCount) failed");
  return counts[dev];
}

template <bool A_MN, bool B_MN, bool GELU, int BN>
void launch(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& g, cudaStream_t st) {
  constexpr uint32_t kSmemBytes = smem_bytes<BN>();
  static size_t configured[dynsmem::kMaxDevices] = {};
  TORCH_CHECK(dynsmem::opt_in(tc_gemm_kernel<A_MN, B_MN, GELU, BN>, kSmemBytes, configured) == cudaSuccess,
              "tc_gemm shared-memory attribute");
  // persistent: one CTA per SM, never more CTAs than work items
  const int64_t total = (int64_t)((g.N + BN - 1) / BN) * ((g.M + kBM - 1) / kBM) * g.splits;
  TORCH_CHECK(total < (1ll << 31), "tc_gemm: too many output tiles");
  const int grid = (int)std::min<int64_t>(total, sm_count());
  tc_gemm_kernel<A_MN, B_MN, GELU, BN><<<grid, kThreads, kSmemBytes, st>>>(ta, tb, g);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "tc_gemm launch failed");
}

// C = op(A) op(B)^T. `a_mn`: A is stored [K][M] (else [M][K]); `b_mn`: B is
// stored [K][N] (else [N][K]). Storage row strides must be multiples of 8
// elements and the base pointers 16-byte aligned (TMA rules).
void tc_gemm(torch::Tensor a, bool a_mn, torch::Tensor b, bool b_mn, torch::Tensor c,
             c10::optional<torch::Tensor> bias, int64_t act, bool accumulate, torch::Tensor status,
             int64_t wait_ns, c10::optional<torch::Tensor> aux) {
  for (auto* t : {&a, &b, &c, &status})
    TORCH_CHECK(t->is_cuda() && t->dim() >= 1, "tc_gemm operands must be CUDA tensors");
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16,
              "tc_gemm operands must both be bf16");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && c.dim() == 2, "tc_gemm takes 2-D operands");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && c.stride(1) == 1, "innermost dims must be contiguous");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "row strides must be multiples of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 &&
              reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0, "operands must be 16-byte aligned");
  const int64_t M = a_mn ? a.size(1) : a.size(0);
  const int64_t K = a_mn ? a.size(0) : a.size(1);
  const int64_t N = b_mn ? b.size(1) : b.size(0);
  const int64_t Kb = b_mn ? b.size(0) : b.size(1);
  TORCH_CHECK(K == Kb, "tc_gemm: inner dimensions differ");
  TORCH_CHECK(c.size(0) == M && c.size(1) == N, "tc_gemm: output must be [M, N]");
  TORCH_CHECK(c.scalar_type() == torch::kFloat32 || c.scalar_type() == torch::kBFloat16, "output fp32 or bf16");
  TORCH_CHECK(!accumulate || c.scalar_type() == torch::kFloat32, "accumulate needs an fp32 output");
  TORCH_CHECK(status.scalar_type() == torch::kInt32, "status must be int32");
  TORCH_CHECK(wait_ns >= 0, "wait_ns must be non-negative");
  TORCH_CHECK(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "tc_gemm dimensions too large");
  if (M == 0 || N == 0) return;
  GemmArgs g{};
  g.M = (int)M;
  g.N = (int)N;
  g.K = (int)K;
  g.c_f32 = c.scalar_type() == torch::kFloat32 ? c.data_ptr<float>() : nullptr;
  g.c_bf16 = c.scalar_type() == torch::kBFloat16 ? reinterpret_cast<__nv_bfloat16*>(c.data_ptr<at::BFloat16>()) : nullptr;
  g.ldc = c.stride(0);
  g.bias = nullptr;
  if (bias && bias->defined()) {
    TORCH_CHECK(bias->is_cuda() && bias->scalar_type() == torch::kFloat32 && bias->numel() == N && bias->is_contiguous(),
                "bias must be fp32 [N]");
    g.bias = bias->data_ptr<float>();
  }
  g.act = (int)act;
  TORCH_CHECK(act >= 0 && act <= 5, "tc_gemm: unknown activation");
  g.accumulate = accumulate ? 1 : 0;
  if (act >= 4) {
    TORCH_CHECK(!accumulate, "tc_gemm: GELU epilogues do not accumulate");
    TORCH_CHECK(act == 4 || (aux && aux->defined()), "tc_gemm: the GELU backward epilogue needs the pre-activation");
  }
  if (aux && aux->defined()) {
    TORCH_CHECK(act >= 4, "tc_gemm: an auxiliary tensor goes with the GELU epilogues only");
    TORCH_CHECK(aux->is_cuda() && aux->scalar_type() == torch::kBFloat16 && aux->dim() == 2 && aux->size(0) == M &&
                    aux->size(1) == N && aux->stride(1) == 1 && aux->stride(0) == c.stride(0) &&
                    reinterpret_cast<uintptr_t>(aux->data_ptr()) % 16 == 0,
                "tc_gemm: aux must be bf16 [M, N] with C's row stride, 16-byte aligned");
    if (act == 4) g.aux_out = reinterpret_cast<__nv_bfloat16*>(aux->data_ptr<at::BFloat16>());
    else g.aux_in = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr<at::BFloat16>());
  }
  g.status = status.data_ptr<int>();
  g.wait_ns = (uint64_t)wait_ns;
  // Epilogue of a result computed outside the kernel (empty contraction, split-K sums).
  auto finish = [&](torch::Tensor z) {
    if (act == 4) {
      if (aux && aux->defined()) aux->copy_(z);
      z = torch::gelu(z);
    } else if (act == 5) {
      const auto p = aux->to(torch::kFloat32);
      z = z * (0.5 * (1 + torch::erf(p * M_SQRT1_2)) + p * (0.5 * M_2_SQRTPI * M_SQRT1_2) * torch::exp(-0.5 * p * p));
    } else if (act == 1) {
      z = z.tanh();
    } else if (act == 2) {
      z = z.relu();
    } else if (act == 3) {
      z = torch::gelu(z, "tanh");
    }
    if (accumulate) c.add_(z);
    else c.copy_(z);
  };
  if (K == 0) {  // empty contraction: C = act(bias) (or unchanged when accumulating zero)
    auto z = torch::zeros({M, N}, c.options().dtype(torch::kFloat32));
    if (g.bias) z += *bias;
    finish(z);
    return;
  }
  // A: K-major [M][K] -> box 64 K x 128 rows; MN-major [K][M] -> box 64 M x 64 K rows
  const CUtensorMap ta = a_mn ? make_map(a.data_ptr(), K, M, a.stride(0), kBK) : make_map(a.data_ptr(), M, K, a.stride(0), kBM);
  // 256-wide output tiles where the main loop dominates: wide outputs, A read
  // K-major, long contractions (K >= 512), plain epilogue. On the K = 256
  // layers the output stores bound the kernel and 128-wide tiles are as fast;
  // the GELU epilogue is slower with 256-wide tiles.
  const int bn = (!a_mn && N >= 256 && K >= 512 && act < 4) ? 256 : 128;
  const CUtensorMap tb = b_mn ? make_map(b.data_ptr(), K, N, b.stride(0), kBK) : make_map(b.data_ptr(), N, K, b.stride(0), bn);
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  // Few output tiles over a long contraction (weight gradients: K = tokens)
  // leave most SMs idle; split K into about two work items per SM, each over
  // at least 8 K steps, into fp32 partials that are summed afterwards.
  const int64_t KT = (K + kBK - 1) / kBK;
  const int64_t tiles = ((N + bn - 1) / bn) * ((M + kBM - 1) / kBM);
  int64_t splits = 1;
  if (tiles < 148 && KT >= 16) splits = std::min<int64_t>(KT / 8, (296 + tiles - 1) / tiles);
  g.k_steps = (int)((KT + splits - 1) / splits);
  splits = (KT + g.k_steps - 1) / g.k_steps;
  g.splits = (int)splits;
  torch::Tensor partial;
  if (splits > 1) {
    partial = torch::empty({splits, M, N}, c.options().dtype(torch::kFloat32));
    g.c_f32 = partial.data_ptr<float>();
    g.c_bf16 = nullptr;
    g.ldc = N;
    g.split_stride = M * N;
    g.bias = nullptr;
    g.act = 0;
    g.accumulate = 0;
    g.aux_out = nullptr;
    g.aux_in = nullptr;
  }
  // GELU epilogues exist for the two layouts a feed-forward layer uses them
  // in (forward: both K-major; backward dX: B MN-major); other layouts run
  // the plain GEMM and the activation afterwards.
  const bool gelu = g.act >= 4;
  const bool gelu_fused = gelu && !a_mn && ((g.act == 4 && !b_mn) || (g.act == 5 && b_mn));
  if (gelu && !gelu_fused) {
    partial = torch::empty({M, N}, c.options().dtype(torch::kFloat32));
    g.c_f32 = partial.data_ptr<float>();
    g.c_bf16 = nullptr;
    g.ldc = N;
    g.split_stride = 0;
    g.bias = nullptr;
    g.act = 0;
    g.aux_out = nullptr;
    g.aux_in = nullptr;
  }
  if (bn == 256) {
    if (!b_mn) launch<false, false, false, 256>(ta, tb, g, st);
    else launch<false, true, false, 256>(ta, tb, g, st);
  } else if (gelu_fused && !a_mn && !b_mn) launch<false, false, true, 128>(ta, tb, g, st);
  else if (gelu_fused) launch<false, true, true, 128>(ta, tb, g, st);
  else if (!a_mn && !b_mn) launch<false, false, false, 128>(ta, tb, g, st);
  else if (!a_mn && b_mn) launch<false, true, false, 128>(ta, tb, g, st);
  else if (a_mn && !b_mn) launch<true, false, false, 128>(ta, tb, g, st);
  else launch<true, true, false, 128>(ta, tb, g, st);
  if (gelu && !gelu_fused) {
    torch::Tensor z = partial;
    if (bias && bias->defined()) z += *bias;
    finish(z);
    return;
  }
  if (splits > 1) {
    auto z = partial.sum(0);
    if (bias && bias->defined()) z += *bias;
    finish(z);
  }
}

}  // namespace

void register_tc_gemm_ops(py::module& m) {
  m.def("tc_gemm", &tc_gemm, "bf16 tcgen05 GEMM C = op(A) op(B)^T (+bias, activation), TMA-fed, fp32 accumulate",
        py::arg("a"), py::arg("a_mn"), py::arg("b"), py::arg("b_mn"), py::arg("c"), py::arg("bias"),
        py::arg("act"), py::arg("accumulate"), py::arg("status"), py::arg("wait_ns") = 2000000000ll,
        py::arg("aux") = py::none());
}
