// Variable-length multi-head self-attention on sm_100a tensor cores
// (tcgen05 MMAs, fp32 accumulators in TMEM), forward and backward.
//
// Layout: the valid tokens of all samples are packed back to back; sample i
// holds rows cu[i]..cu[i+1] of the projection qkv [total, 3 * heads * 64]
// whose last dimension is [3][heads][64] (queries, keys, values), as the
// entity encoder's in-projection writes it (frc_defense/architecture_entities.py:
// 51-69 is the reference model; there attention runs on padded batches).
// Each token attends to the tokens of its own sample only; head dim 64,
// softmax scale 1/8.
//
// Forward, one CTA per (sample, head, 128-query block), 160 threads:
//   warp 4 (one lane) is the control warp: TMA loads of the query block and
//   of each 128-key block's keys (two-deep ring) and values as SW128 images,
//   and the tensor-core MMAs. S = Q K^T lands in TMEM; warps 0-3 (thread t =
//   TMEM lane t = query row t) take the row maximum in a first pass over S,
//   write P = exp2(S * scale * log2 e - max) as a bf16 image in a second
//   pass and signal; the control warp then issues the next block's S = Q K^T
//   (it overlaps this block's output update) and P V into a second TMEM
//   region, which the softmax warps add into their register-resident output
//   row after the online-softmax rescale. Output rows are normalised at the
//   end; the base-2 log-sum-exp of each row is kept for the backward.
//
// Backward, one CTA per (sample, head), 160 threads, key blocks outer and
// query blocks inner. Warp 4 loads the key / value blocks and the query /
// output-gradient blocks by TMA (both two-deep) and issues two MMA groups per
// (key block, query block) pair: S = Q K^T and dP = dO V^T, then, once warps
// 0-3 have written P (recomputed from the saved log-sum-exp) and
// dS = P (dP - D) / 8 (D = rowsum(dO * O), computed once per row up front)
// as bf16 images, dV += P^T dO and dK += dS^T Q (TMEM accumulators over the
// query blocks; the transposes are the same images read MN-major) and
// dQ = dS K. Warps 0-3 add dQ into an fp32 row buffer owned by this CTA (no
// atomics: the result is deterministic) and write it as bf16 after the last
// key block; dK and dV leave after each key block.
//
// Rows of a tile past the end of its sample are loaded from the next sample
// (or read as zero past the end of the tensor): their probabilities and
// gradients are forced to zero and their outputs are not written.
//
// Every mbarrier wait is bounded (`wait_ns`); a wait that runs out sets a
// bit of the status word (64 forward, 128 backward; 256 if the MMAs still
// in flight did not finish within 200 ms after that), the CTA stops its
// loop, frees its TMEM and returns without writing results.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

#include "tc_sm100.h"
#include "tma_map.h"
#include "smem_opt_in.h"

namespace py = pybind11;

namespace {

constexpr int kDh = 64;                         // head dimension: one 64-column image block
constexpr int kBlk = 128;                       // queries / keys per tile (UMMA M and N)
constexpr int kCompute = 128;                   // warps 0-3: thread t <-> TMEM lane t <-> tile row t
constexpr int kThreads = kCompute + 32;         // + warp 4: TMA loads and MMA issue
constexpr uint32_t kImg64 = kBlk * 128;         // 128 rows x 64 bf16 = 16 KB
constexpr uint32_t kImg128 = 2 * kImg64;        // 128 rows x 128 bf16 = 32 KB
constexpr uint64_t kDrainNs = 200000000ull;
constexpr int kBitFwd = 64, kBitBwd = 128, kBitDrain = 256;

// forward: Q | K ring (2) | V | P | barriers
constexpr uint32_t kFwdQ = 0, kFwdK = kImg64, kFwdV = 3 * kImg64, kFwdP = 4 * kImg64, kFwdMisc = kFwdP + kImg128;
constexpr uint32_t kFwdSmem = kFwdMisc + 128 + 1024;
// backward: Q ring (2) | dO ring (2) | K ring (2) | V ring (2) | P | dS | barriers
constexpr uint32_t kBwdQ = 0, kBwdDO = 2 * kImg64, kBwdK = 4 * kImg64, kBwdV = 6 * kImg64, kBwdP = 8 * kImg64,
                   kBwdDS = kBwdP + kImg128, kBwdStats = kBwdDS + kImg128;
constexpr int kStatRows = 1024;                 // rows whose log-sum-exp and D stay in shared memory
constexpr uint32_t kBwdMisc = kBwdStats + 2 * kStatRows * 4;
constexpr uint32_t kBwdSmem = kBwdMisc + 128 + 1024;

struct AttnArgs {
  const int* cu_q;            // [samples + 1]: query rows of each sample
  const int* cu_k;            // [samples + 1]: key / value rows of each sample
  int q_col, k_col, v_col;    // column of head 0's queries / keys / values in their sources
  int heads;
  int64_t total_q;            // query rows (rows of out, dout, lse)
  float scale_log2;           // softmax scale * log2(e)
  float scale;                // softmax scale
  __nv_bfloat16* out;         // [total_q, heads * 64]
  float* lse;                 // [heads, total_q]: base-2 log-sum-exp of the scaled scores
  const __nv_bfloat16* dout;  // [total_q, heads * 64]
  __nv_bfloat16* dq;          // query gradient rows (stride ldq), head 0 at column dq_col
  int64_t ldq;
  int dq_col;
  __nv_bfloat16* dkv;         // key / value gradient rows (stride ldkv)
  int64_t ldkv;
  int dk_col, dv_col;
  float* dq_acc;              // [total_q, heads * 64] fp32 (samples with several key blocks)
  float* dvec;                // [heads, total_q] fp32: rowsum(dO * O)
  int* status;
  uint64_t wait_ns;
};

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// 32 consecutive values of this thread's row as bf16 into image columns c0..c0+31.
__device__ __forceinline__ void store_row32(uint8_t* img, int row, int c0, const float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * j], v[8 * j + 1]);
    u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    *reinterpret_cast<uint4*>(img + tc::sw128_offset(row, c0 + 8 * j, kBlk)) = u;
  }
}

// Bounded wait shared by all roles: gives up when the limit runs out (status
// bit set, the CTA's failure flag raised) or when another role of the CTA
// has already failed.
__device__ __forceinline__ bool wait_or_fail(uint32_t bar, uint32_t parity, const AttnArgs& a, int* s_fail, int bit) {
  if (tc::mbar_try_wait(bar, parity)) return true;
  volatile int* fail = s_fail;
  const uint64_t t0 = tc::globaltimer_ns();
  while (true) {
    if (tc::mbar_try_wait(bar, parity)) return true;
    if (*fail) return false;
    if (tc::globaltimer_ns() - t0 > a.wait_ns) {
      atomicOr(a.status, bit);
      *fail = 1;
      return false;
    }
  }
}

// After a failure: let the MMAs and TMA loads of this thread finish
// (bounded) before the CTA frees TMEM and exits. The load barriers are
// consecutive mbarriers from `bar0`; bit i of `pending` marks a load on
// barrier i not yet waited for, bit i of `parity` that barrier's phase parity.
__device__ __forceinline__ void drain_after_failure(uint32_t drain_bar, uint32_t bar0, uint32_t pending,
                                                    uint32_t parity, int nbars, const AttnArgs& a) {
  tc::mma_commit(drain_bar);
  if (!tc::mbar_wait(drain_bar, 0, kDrainNs)) atomicOr(a.status, kBitDrain);
  for (int i = 0; i < nbars; ++i)
    if ((pending >> i) & 1u)
      if (!tc::mbar_wait(bar0 + 8u * i, (parity >> i) & 1u, kDrainNs)) atomicOr(a.status, kBitDrain);
}

__global__ void __launch_bounds__(kThreads, 2)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv, const AttnArgs a,
                int nqb) {
  const int qb = blockIdx.x % nqb;
  const int h = (blockIdx.x / nqb) % a.heads;
  const int seq = blockIdx.x / (nqb * a.heads);
  const int sq0 = a.cu_q[seq], Lq = a.cu_q[seq + 1] - sq0;
  const int sk0 = a.cu_k[seq], Lk = a.cu_k[seq + 1] - sk0;
  const int q0 = qb * kBlk;
  if (q0 >= Lq) return;   // whole CTA, before any barrier or TMEM allocation
  if (Lk <= 0) {          // no keys: zero output rows
    for (int i = threadIdx.x; i < min(kBlk, Lq - q0) * 8; i += blockDim.x)
      reinterpret_cast<uint4*>(a.out + (int64_t)(sq0 + q0 + (i >> 3)) * (a.heads * kDh) + h * kDh)[i & 7] =
          make_uint4(0u, 0u, 0u, 0u);
    for (int i = threadIdx.x; i < min(kBlk, Lq - q0); i += blockDim.x)
      a.lse[(int64_t)h * a.total_q + sq0 + q0 + i] = -INFINITY;
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* misc = smem + kFwdMisc;
  const uint32_t sb = tc::smem_u32(smem);
  const uint32_t bar_k0 = tc::smem_u32(misc);      // K ring slot 0 (+ the query block)
  const uint32_t bar_k1 = bar_k0 + 8;              // K ring slot 1
  const uint32_t bar_v = bar_k0 + 16;              // value block
  const uint32_t s_full = bar_k0 + 24;             // S = Q K^T complete
  const uint32_t p_full = bar_k0 + 32;             // P written, S and the previous P V read (128 arrivals)
  const uint32_t o_full = bar_k0 + 40;             // P V complete
  const uint32_t drain = bar_k0 + 48;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(misc + 64);
  int* s_fail = reinterpret_cast<int*>(misc + 72);
  const int t = threadIdx.x, warp = t >> 5;
  const int nkb = (Lk + kBlk - 1) / kBlk;

  if (t == kCompute) {
    tc::mbar_init(bar_k0, 1);
    tc::mbar_init(bar_k1, 1);
    tc::mbar_init(bar_v, 1);
    tc::mbar_init(s_full, 1);
    tc::mbar_init(p_full, kCompute);
    tc::mbar_init(o_full, 1);
    tc::mbar_init(drain, 1);
    tc::mbar_init_fence();
    *s_fail = 0;
  }
  if (warp == 4) {
    tc::tmem_alloc(tc::smem_u32(s_tmem), 256);   // S: columns 0-127, P V: 128-191
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (t == kCompute) {
    // ---- control: TMA loads and MMA issue ----
    const int xq = a.q_col + h * kDh, xk = a.k_col + h * kDh, xv = a.v_col + h * kDh;
    uint32_t pending = 0, parity = 0;   // loads in flight per barrier (k0, k1, v), phase parities
    tc::mbar_arrive_expect_tx(bar_k0, 2 * kImg64);
    tc::tma_load_2d(sb + kFwdQ, &tm_q, xq, sq0 + q0, bar_k0);
    tc::tma_load_2d(sb + kFwdK, &tm_kv, xk, sk0, bar_k0);
    pending |= 1u;
    tc::mbar_arrive_expect_tx(bar_v, kImg64);
    tc::tma_load_2d(sb + kFwdV, &tm_kv, xv, sk0, bar_v);
    pending |= 4u;
    if (nkb > 1) {
      tc::mbar_arrive_expect_tx(bar_k1, kImg64);
      tc::tma_load_2d(sb + kFwdK + kImg64, &tm_kv, xk, sk0 + kBlk, bar_k1);
      pending |= 2u;
    }
    const uint32_t id_s = tc::idesc_bf16(kBlk, kBlk, false, false);
    const uint32_t id_o = tc::idesc_bf16(kBlk, kDh, false, true);
    bool ok = wait_or_fail(bar_k0, 0, a, s_fail, kBitFwd);
    if (ok) {
      pending &= ~1u;
      parity ^= 1u;
      tc::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kDh / 16; ++ks)
        tc::mma_bf16(tmem, tc::desc_kmajor(sb + kFwdQ, kBlk, ks), tc::desc_kmajor(sb + kFwdK, kBlk, ks), id_s, ks > 0);
      tc::mma_commit(s_full);
    }
    for (int kb = 0; kb < nkb && ok; ++kb) {
      if (!(ok = wait_or_fail(p_full, kb & 1, a, s_fail, kBitFwd))) break;
      tc::tc_fence_after();
      if (kb + 1 < nkb) {   // next block's scores overlap this block's output update
        const int r = (kb + 1) & 1;
        if (!(ok = wait_or_fail(bar_k0 + 8u * r, ((kb + 1) >> 1) & 1, a, s_fail, kBitFwd))) break;
        pending &= ~(1u << r);
        parity ^= 1u << r;
        tc::tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kDh / 16; ++ks)
          tc::mma_bf16(tmem, tc::desc_kmajor(sb + kFwdQ, kBlk, ks), tc::desc_kmajor(sb + kFwdK + r * kImg64, kBlk, ks),
                       id_s, ks > 0);
        tc::mma_commit(s_full);
      }
      if (!(ok = wait_or_fail(bar_v, kb & 1, a, s_fail, kBitFwd))) break;
      pending &= ~4u;
      parity ^= 4u;
      tc::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kBlk / 16; ++ks)
        tc::mma_bf16(tmem + 128, tc::desc_kmajor(sb + kFwdP, kBlk, ks), tc::desc_mnmajor(sb + kFwdV, kBlk, ks), id_o,
                     ks > 0);
      tc::mma_commit(o_full);
      if (kb + 2 < nkb) {   // K slot kb & 1 was read by S_kb, which completed before P_kb was written
        const uint32_t bk = bar_k0 + 8u * (kb & 1);
        tc::mbar_arrive_expect_tx(bk, kImg64);
        tc::tma_load_2d(sb + kFwdK + (kb & 1) * kImg64, &tm_kv, xk, sk0 + (kb + 2) * kBlk, bk);
        pending |= 1u << (kb & 1);
      }
      if (kb + 1 < nkb) {   // the value block is reloaded once P V has read it
        if (!(ok = wait_or_fail(o_full, kb & 1, a, s_fail, kBitFwd))) break;
        tc::mbar_arrive_expect_tx(bar_v, kImg64);
        tc::tma_load_2d(sb + kFwdV, &tm_kv, xv, sk0 + (kb + 1) * kBlk, bar_v);
        pending |= 4u;
      }
    }
    if (!ok) drain_after_failure(drain, bar_k0, pending, parity, 3, a);
  } else if (t < kCompute) {
    // ---- softmax warps: thread t owns query row q0 + t ----
    const uint32_t lane = (uint32_t)(32 * warp) << 16;
    float o[kDh];
#pragma unroll
    for (int i = 0; i < kDh; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
      if (!(ok = wait_or_fail(s_full, kb & 1, a, s_fail, kBitFwd))) break;
      tc::tc_fence_after();
      const int kvalid = Lk - kb * kBlk;
      float mb = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < 4; c0 += 2) {   // two 32-column loads in flight
        float v[2][32];
        tc::tmem_ld32_issue(tmem + lane + 32 * c0, v[0]);
        tc::tmem_ld32_issue(tmem + lane + 32 * c0 + 32, v[1]);
        tc::tmem_ld_wait();
        tc::tmem_regs_ready(v[0]);
        tc::tmem_regs_ready(v[1]);
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (32 * c0 + i < kvalid) mb = fmaxf(mb, v[i >> 5][i & 31] * a.scale_log2);
      }
      const float mn = fmaxf(m, mb);
      const float alpha = exp2f(m - mn);   // 0 on the first block (m = -inf)
      if (kb > 0) {   // previous block's P V: into the output row, then P may be overwritten
        if (!(ok = wait_or_fail(o_full, (kb - 1) & 1, a, s_fail, kBitFwd))) break;
        tc::tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; ++half) {   // 32 columns at a time keeps the register peak low
          float pv[32];
          tc::tmem_ld32_issue(tmem + lane + 128 + 32 * half, pv);
          tc::tmem_ld_wait();
          tc::tmem_regs_ready(pv);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[32 * half + i] = o[32 * half + i] * alpha_prev + pv[i];
        }
      }
      float sum = 0.f;
#pragma unroll
      for (int c0 = 0; c0 < 4; c0 += 2) {
        float v[2][32];
        tc::tmem_ld32_issue(tmem + lane + 32 * c0, v[0]);
        tc::tmem_ld32_issue(tmem + lane + 32 * c0 + 32, v[1]);
        tc::tmem_ld_wait();
        tc::tmem_regs_ready(v[0]);
        tc::tmem_regs_ready(v[1]);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float p = (32 * (c0 + h2) + i < kvalid) ? exp2f(v[h2][i] * a.scale_log2 - mn) : 0.f;
            v[h2][i] = p;
            sum += p;
          }
          store_row32(smem + kFwdP, t, 32 * (c0 + h2), v[h2]);
        }
      }
      l = l * alpha + sum;
      m = mn;
      alpha_prev = alpha;
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(p_full);
    }
    if (ok && wait_or_fail(o_full, (nkb - 1) & 1, a, s_fail, kBitFwd)) {
      tc::tc_fence_after();
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float pv[32];
        tc::tmem_ld32_issue(tmem + lane + 128 + 32 * half, pv);
        tc::tmem_ld_wait();
        tc::tmem_regs_ready(pv);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[32 * half + i] = o[32 * half + i] * alpha_prev + pv[i];
      }
      const int row = q0 + t;
      if (row < Lq) {
        const float inv = 1.f / l;
        uint4* dst = reinterpret_cast<uint4*>(a.out + (int64_t)(sq0 + row) * (a.heads * kDh) + h * kDh);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float y[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int i = 8 * j + e;
            y[e] = o[i] * inv;
          }
          dst[j] = make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                              pack_bf16x2(y[6], y[7]));
        }
        a.lse[(int64_t)h * a.total_q + sq0 + row] = m + log2f(l);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 256);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_kv,
                const __grid_constant__ CUtensorMap tm_dout, const AttnArgs a) {
  const int h = blockIdx.x % a.heads, seq = blockIdx.x / a.heads;
  const int sq0 = a.cu_q[seq], Lq = a.cu_q[seq + 1] - sq0;
  const int sk0 = a.cu_k[seq], Lk = a.cu_k[seq + 1] - sk0;
  if (Lq <= 0 || Lk <= 0) {   // no attention pairs: zero gradients
    for (int i = threadIdx.x; i < Lq * 8; i += blockDim.x)
      reinterpret_cast<uint4*>(a.dq + (int64_t)(sq0 + (i >> 3)) * a.ldq + a.dq_col + h * kDh)[i & 7] =
          make_uint4(0u, 0u, 0u, 0u);
    for (int i = threadIdx.x; i < Lk * 8; i += blockDim.x) {
      const int64_t r = (int64_t)(sk0 + (i >> 3)) * a.ldkv;
      reinterpret_cast<uint4*>(a.dkv + r + a.dk_col + h * kDh)[i & 7] = make_uint4(0u, 0u, 0u, 0u);
      reinterpret_cast<uint4*>(a.dkv + r + a.dv_col + h * kDh)[i & 7] = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  uint8_t* misc = smem + kBwdMisc;
  const uint32_t sb = tc::smem_u32(smem);
  const uint32_t bar_q0 = tc::smem_u32(misc);      // Q / dO ring slot 0
  const uint32_t bar_q1 = bar_q0 + 8;              // Q / dO ring slot 1
  const uint32_t bar_kv0 = bar_q0 + 16;            // K / V ring slot 0
  const uint32_t bar_kv1 = bar_q0 + 24;            // K / V ring slot 1
  const uint32_t g1 = bar_q0 + 32;                 // S and dP complete
  const uint32_t ds_full = bar_q0 + 40;            // P and dS written, S and dP read (128 arrivals)
  const uint32_t g2 = bar_q0 + 48;                 // dV, dK, dQ MMAs complete
  const uint32_t drain = bar_q0 + 56;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(misc + 64);
  int* s_fail = reinterpret_cast<int*>(misc + 72);
  const int t = threadIdx.x, warp = t >> 5;
  const int nbq = (Lq + kBlk - 1) / kBlk, nbk = (Lk + kBlk - 1) / kBlk;
  const int npairs = nbk * nbq;
  const int dm = a.heads * kDh;

  if (t == kCompute) {
    tc::mbar_init(bar_q0, 1);
    tc::mbar_init(bar_q1, 1);
    tc::mbar_init(bar_kv0, 1);
    tc::mbar_init(bar_kv1, 1);
    tc::mbar_init(g1, 1);
    tc::mbar_init(ds_full, kCompute);
    tc::mbar_init(g2, 1);
    tc::mbar_init(drain, 1);
    tc::mbar_init_fence();
    *s_fail = 0;
  }
  if (warp == 4) {
    // S 0-127, dP 128-255, dV 256-319, dK 320-383, dQ 384-447
    tc::tmem_alloc(tc::smem_u32(s_tmem), 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *s_tmem;

  if (t == kCompute) {
    // ---- control: TMA loads, two MMA groups per (key block, query block) pair ----
    const int xq = a.q_col + h * kDh, xk = a.k_col + h * kDh, xv = a.v_col + h * kDh;
    uint32_t pending = 0, parity = 0;   // loads in flight per barrier (q0, q1, kv0, kv1), phase parities
    auto load_q = [&](int p) {
      const int r = p & 1, q0 = (p % nbq) * kBlk;
      const uint32_t bq = bar_q0 + 8u * r;
      tc::mbar_arrive_expect_tx(bq, 2 * kImg64);
      tc::tma_load_2d(sb + kBwdQ + r * kImg64, &tm_q, xq, sq0 + q0, bq);
      tc::tma_load_2d(sb + kBwdDO + r * kImg64, &tm_dout, h * kDh, sq0 + q0, bq);
      pending |= 1u << r;
    };
    auto load_kv = [&](int kb) {
      const int r = kb & 1;
      const uint32_t bkv = bar_kv0 + 8u * r;
      tc::mbar_arrive_expect_tx(bkv, 2 * kImg64);
      tc::tma_load_2d(sb + kBwdK + r * kImg64, &tm_kv, xk, sk0 + kb * kBlk, bkv);
      tc::tma_load_2d(sb + kBwdV + r * kImg64, &tm_kv, xv, sk0 + kb * kBlk, bkv);
      pending |= 4u << r;
    };
    load_kv(0);
    load_q(0);
    const uint32_t id_sq = tc::idesc_bf16(kBlk, kBlk, false, false);   // queries x keys over dh
    const uint32_t id_t = tc::idesc_bf16(kBlk, kDh, true, true);       // keys x dh over queries
    const uint32_t id_q = tc::idesc_bf16(kBlk, kDh, false, true);      // queries x dh over keys
    bool ok = true;
    for (int p = 0; p < npairs && ok; ++p) {
      const int kb = p / nbq, qb = p % nbq, r = p & 1, rk = kb & 1;
      if (p == 0) {
        if (npairs > 1) load_q(1);
        if (nbk > 1) load_kv(1);
      }
      if (!(ok = wait_or_fail(bar_q0 + 8u * r, (p >> 1) & 1, a, s_fail, kBitBwd))) break;
      pending &= ~(1u << r);
      parity ^= 1u << r;
      if (qb == 0) {
        if (!(ok = wait_or_fail(bar_kv0 + 8u * rk, (kb >> 1) & 1, a, s_fail, kBitBwd))) break;
        pending &= ~(4u << rk);
        parity ^= 4u << rk;
      }
      tc::tc_fence_after();
      const uint32_t q_img = sb + kBwdQ + r * kImg64, do_img = sb + kBwdDO + r * kImg64;
      const uint32_t k_img = sb + kBwdK + rk * kImg64, v_img = sb + kBwdV + rk * kImg64;
#pragma unroll
      for (int ks = 0; ks < kDh / 16; ++ks) {
        tc::mma_bf16(tmem, tc::desc_kmajor(q_img, kBlk, ks), tc::desc_kmajor(k_img, kBlk, ks), id_sq, ks > 0);
        tc::mma_bf16(tmem + 128, tc::desc_kmajor(do_img, kBlk, ks), tc::desc_kmajor(v_img, kBlk, ks), id_sq, ks > 0);
      }
      tc::mma_commit(g1);
      // S / dP of this pair are queued behind the previous pair's gradient MMAs;
      // once those finish, slot (p + 1) & 1 (and at a key block's start the K / V
      // slot of the key block after next) is free for the next loads
      if (p > 0) {
        if (!(ok = wait_or_fail(g2, (p - 1) & 1, a, s_fail, kBitBwd))) break;
        tc::tc_fence_after();
        if (p + 1 < npairs) load_q(p + 1);
        if (qb == 0 && kb + 1 < nbk) load_kv(kb + 1);
      }
      if (!(ok = wait_or_fail(ds_full, p & 1, a, s_fail, kBitBwd))) break;
      tc::tc_fence_after();
#pragma unroll
      for (int ks = 0; ks < kBlk / 16; ++ks) {
        const bool acc = qb > 0 || ks > 0;
        tc::mma_bf16(tmem + 256, tc::desc_mnmajor(sb + kBwdP, kBlk, ks), tc::desc_mnmajor(do_img, kBlk, ks), id_t, acc);
        tc::mma_bf16(tmem + 320, tc::desc_mnmajor(sb + kBwdDS, kBlk, ks), tc::desc_mnmajor(q_img, kBlk, ks), id_t, acc);
        tc::mma_bf16(tmem + 384, tc::desc_kmajor(sb + kBwdDS, kBlk, ks), tc::desc_mnmajor(k_img, kBlk, ks), id_q, ks > 0);
      }
      tc::mma_commit(g2);
    }
    if (!ok) drain_after_failure(drain, bar_q0, pending, parity, 4, a);
  } else if (t < kCompute) {
    // ---- elementwise warps: thread t owns row t of each query block (S, dP, dQ)
    // and row t of each key block (dK, dV) ----
    // D = rowsum(dO * O) and the log-sum-exp of rows t, t + 128, ... (the
    // rows this thread owns in every query block), while the first MMAs run;
    // kept in shared memory (only this thread reads them back)
    float* s_lse = reinterpret_cast<float*>(smem + kBwdStats);
    float* s_D = s_lse + kStatRows;
    for (int row = t; row < Lq; row += kCompute) {
      const uint4* po = reinterpret_cast<const uint4*>(a.out + (int64_t)(sq0 + row) * dm + h * kDh);
      const uint4* pd = reinterpret_cast<const uint4*>(a.dout + (int64_t)(sq0 + row) * dm + h * kDh);
      float D = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 x = __ldg(po + j), y = __ldg(pd + j);
        const __nv_bfloat162* xo = reinterpret_cast<const __nv_bfloat162*>(&x);
        const __nv_bfloat162* yd = reinterpret_cast<const __nv_bfloat162*>(&y);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 u = __bfloat1622float2(xo[k]), w = __bfloat1622float2(yd[k]);
          D += u.x * w.x + u.y * w.y;
        }
      }
      const float lse2 = a.lse[(int64_t)h * a.total_q + sq0 + row];
      if (row < kStatRows) {
        s_D[row] = D;
        s_lse[row] = lse2;
      } else {
        a.dvec[(int64_t)h * a.total_q + sq0 + row] = D;
      }
    }
    float acc[kDh];   // running dQ row of the next pair, fetched a pair ahead
    const uint32_t lane = (uint32_t)(32 * warp) << 16;
    for (int p = 0; p < npairs; ++p) {
      const int kb = p / nbq, qb = p % nbq;
      const int k0 = kb * kBlk, row = qb * kBlk + t;
      const bool live = row < Lq;
      float D = 0.f, lse2 = 0.f;
      if (live) {
        if (row < kStatRows) {
          D = s_D[row];
          lse2 = s_lse[row];
        } else {
          D = a.dvec[(int64_t)h * a.total_q + sq0 + row];
          lse2 = a.lse[(int64_t)h * a.total_q + sq0 + row];
        }
      }
      if (!wait_or_fail(g1, p & 1, a, s_fail, kBitBwd)) break;
      tc::tc_fence_after();
      const int kvalid = Lk - k0;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float s[32], dp[32];
        tc::tmem_ld32_issue(tmem + lane + 32 * c, s);
        tc::tmem_ld32_issue(tmem + lane + 128 + 32 * c, dp);
        tc::tmem_ld_wait();
        tc::tmem_regs_ready(s);
        tc::tmem_regs_ready(dp);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float pr = (live && 32 * c + i < kvalid) ? exp2f(s[i] * a.scale_log2 - lse2) : 0.f;
          s[i] = pr;
          dp[i] = pr * (dp[i] - D) * a.scale;
        }
        store_row32(smem + kBwdP, t, 32 * c, s);
        store_row32(smem + kBwdDS, t, 32 * c, dp);
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
      tc::mbar_arrive(ds_full);
      if (!wait_or_fail(g2, p & 1, a, s_fail, kBitBwd)) break;
      tc::tc_fence_after();
      float g[2][32];
      tc::tmem_ld32_issue(tmem + lane + 384, g[0]);
      tc::tmem_ld32_issue(tmem + lane + 416, g[1]);
      tc::tmem_ld_wait();
      tc::tmem_regs_ready(g[0]);
      tc::tmem_regs_ready(g[1]);
      if (live) {
        if (kb > 0) {
#pragma unroll
          for (int i = 0; i < kDh; ++i) g[i >> 5][i & 31] += acc[i];
        }
        if (kb + 1 < nbk) {
          float4* dst = reinterpret_cast<float4*>(a.dq_acc + (int64_t)(sq0 + row) * dm + h * kDh);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float* gj = &g[j >> 3][(j & 7) * 4];
            dst[j] = make_float4(gj[0], gj[1], gj[2], gj[3]);
          }
        } else {   // last key block: the finished dQ row
          uint4* dst = reinterpret_cast<uint4*>(a.dq + (int64_t)(sq0 + row) * a.ldq + a.dq_col + h * kDh);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float* gj = &g[j >> 2][(j & 3) * 8];
            dst[j] = make_uint4(pack_bf16x2(gj[0], gj[1]), pack_bf16x2(gj[2], gj[3]), pack_bf16x2(gj[4], gj[5]),
                                pack_bf16x2(gj[6], gj[7]));
          }
        }
      }
      if (p + 1 < npairs) {   // the next pair's running dQ row (written nbq pairs earlier)
        const int kb2 = (p + 1) / nbq, row2 = ((p + 1) % nbq) * kBlk + t;
        if (kb2 > 0 && row2 < Lq) {
          const float4* src = reinterpret_cast<const float4*>(a.dq_acc + (int64_t)(sq0 + row2) * dm + h * kDh);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float4 x = src[j];
            acc[4 * j] = x.x, acc[4 * j + 1] = x.y, acc[4 * j + 2] = x.z, acc[4 * j + 3] = x.w;
          }
        }
      }
      if (qb + 1 == nbq) {   // the key block's dK and dV (TMEM lane t = key row k0 + t)
        const int krow = k0 + t;
        float dv[2][32], dk[2][32];
        tc::tmem_ld32_issue(tmem + lane + 256, dv[0]);
        tc::tmem_ld32_issue(tmem + lane + 288, dv[1]);
        tc::tmem_ld32_issue(tmem + lane + 320, dk[0]);
        tc::tmem_ld32_issue(tmem + lane + 352, dk[1]);
        tc::tmem_ld_wait();
        tc::tmem_regs_ready(dv[0]);
        tc::tmem_regs_ready(dv[1]);
        tc::tmem_regs_ready(dk[0]);
        tc::tmem_regs_ready(dk[1]);
        if (krow < Lk) {
          uint4* pk = reinterpret_cast<uint4*>(a.dkv + (int64_t)(sk0 + krow) * a.ldkv + a.dk_col + h * kDh);
          uint4* pv = reinterpret_cast<uint4*>(a.dkv + (int64_t)(sk0 + krow) * a.ldkv + a.dv_col + h * kDh);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float* k8 = &dk[j >> 2][(j & 3) * 8];
            const float* v8 = &dv[j >> 2][(j & 3) * 8];
            pk[j] = make_uint4(pack_bf16x2(k8[0], k8[1]), pack_bf16x2(k8[2], k8[3]), pack_bf16x2(k8[4], k8[5]),
                               pack_bf16x2(k8[6], k8[7]));
            pv[j] = make_uint4(pack_bf16x2(v8[0], v8[1]), pack_bf16x2(v8[2], v8[3]), pack_bf16x2(v8[4], v8[5]),
                               pack_bf16x2(v8[6], v8[7]));
          }
        }
      }
      tc::tc_fence_before();
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

void check_operand(const torch::Tensor& x, const char* what) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 &&
                  x.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0 &&
                  x.size(0) < (1ll << 31),
              "attention: ", what, " must be a CUDA bf16 matrix with contiguous, 16-byte aligned rows");
}

void check_cols(const torch::Tensor& x, int64_t col, int64_t heads, const char* what) {
  TORCH_CHECK(col >= 0 && col % 8 == 0 && col + heads * kDh <= x.size(1), "attention: ", what,
              " columns out of range or not a multiple of 8");
}

AttnArgs base_args(const torch::Tensor& q, int64_t q_col, const torch::Tensor& kv, int64_t k_col, int64_t v_col,
                   const torch::Tensor& cu_q, const torch::Tensor& cu_k, int64_t heads, torch::Tensor& status,
                   int64_t wait_ns) {
  check_operand(q, "the query source");
  check_operand(kv, "the key / value source");
  TORCH_CHECK(heads > 0 && heads < 65536, "attention: bad head count");
  check_cols(q, q_col, heads, "query");
  check_cols(kv, k_col, heads, "key");
  check_cols(kv, v_col, heads, "value");
  for (auto* c : {&cu_q, &cu_k})
    TORCH_CHECK(c->is_cuda() && c->scalar_type() == torch::kInt32 && c->dim() == 1 && c->is_contiguous() &&
                    c->numel() >= 2 && c->numel() - 1 < (1ll << 31), "attention: cu must be CUDA int32 [samples + 1]");
  TORCH_CHECK(cu_q.numel() == cu_k.numel(), "attention: query and key offsets differ in sample count");
  TORCH_CHECK(status.is_cuda() && status.scalar_type() == torch::kInt32, "attention: status must be CUDA int32");
  TORCH_CHECK(wait_ns >= 0, "attention: negative wait");
  AttnArgs a{};
  a.cu_q = cu_q.data_ptr<int>();
  a.cu_k = cu_k.data_ptr<int>();
  a.q_col = (int)q_col;
  a.k_col = (int)k_col;
  a.v_col = (int)v_col;
  a.heads = (int)heads;
  a.total_q = q.size(0);
  a.scale = 0.125f;
  a.scale_log2 = 0.125f * 1.4426950408889634f;
  a.status = status.data_ptr<int>();
  a.wait_ns = (uint64_t)wait_ns;
  return a;
}

void check_rows(const torch::Tensor& x, int64_t rows, int64_t cols, torch::ScalarType type, const char* what) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == type && x.is_contiguous() && x.numel() == rows * cols &&
                  reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0,
              "attention: ", what, " has the wrong shape, type or layout");
}

// Sample i's queries are rows cu_q[i]..cu_q[i+1] of `q` (head h at column
// q_col + 64 h), its keys and values rows cu_k[i]..cu_k[i+1] of `kv` (columns
// k_col + 64 h and v_col + 64 h). out [total_q, heads * 64] bf16, lse
// [heads, total_q] fp32. `max_q` must be at least the most queries of a
// sample (it sizes the grid of query blocks).
void attn_fwd(torch::Tensor q, int64_t q_col, torch::Tensor kv, int64_t k_col, int64_t v_col, torch::Tensor cu_q,
              torch::Tensor cu_k, int64_t max_q, int64_t heads, torch::Tensor out, torch::Tensor lse,
              torch::Tensor status, int64_t wait_ns) {
  AttnArgs a = base_args(q, q_col, kv, k_col, v_col, cu_q, cu_k, heads, status, wait_ns);
  check_rows(out, q.size(0), heads * kDh, torch::kBFloat16, "out");
  check_rows(lse, heads, q.size(0), torch::kFloat32, "lse");
  TORCH_CHECK(max_q >= 0, "attention: negative max_q");
  const int64_t samples = cu_q.numel() - 1;
  if (q.size(0) == 0 || max_q == 0) return;
  if (kv.size(0) == 0) {   // no keys anywhere: zero output
    out.zero_();
    lse.fill_(-INFINITY);
    return;
  }
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>());
  a.lse = lse.data_ptr<float>();
  static size_t configured[dynsmem::kMaxDevices] = {};
  TORCH_CHECK(dynsmem::opt_in(attn_fwd_kernel, kFwdSmem, configured) == cudaSuccess,
              "attention: shared-memory attribute");
  const int64_t nqb = (max_q + kBlk - 1) / kBlk;
  const int64_t blocks = samples * heads * nqb;
  TORCH_CHECK(blocks < (1ll << 31), "attention: too many query blocks");
  const CUtensorMap tq = tma::bf16_sw128(q.data_ptr(), q.size(0), q.size(1), q.stride(0), kBlk);
  const CUtensorMap tkv = tma::bf16_sw128(kv.data_ptr(), kv.size(0), kv.size(1), kv.stride(0), kBlk);
  attn_fwd_kernel<<<(unsigned)blocks, kThreads, kFwdSmem, c10::cuda::getCurrentCUDAStream().stream()>>>(tq, tkv, a,
                                                                                                     (int)nqb);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "attention forward launch failed");
}

// Gradients of attn_fwd: dq has q's shape and strides (head h's gradient at
// column dq_col + 64 h), dkv kv's (dk_col, dv_col). Every query and key row of
// every head is written. `max_k` must be at least the most keys of a sample.
void attn_bwd(torch::Tensor q, int64_t q_col, torch::Tensor kv, int64_t k_col, int64_t v_col, torch::Tensor cu_q,
              torch::Tensor cu_k, int64_t max_k, int64_t heads, torch::Tensor out, torch::Tensor dout,
              torch::Tensor lse, torch::Tensor dq, int64_t dq_col, torch::Tensor dkv, int64_t dk_col, int64_t dv_col,
              torch::Tensor status, int64_t wait_ns) {
  AttnArgs a = base_args(q, q_col, kv, k_col, v_col, cu_q, cu_k, heads, status, wait_ns);
  check_rows(out, q.size(0), heads * kDh, torch::kBFloat16, "out");
  check_rows(dout, q.size(0), heads * kDh, torch::kBFloat16, "dout");
  check_rows(lse, heads, q.size(0), torch::kFloat32, "lse");
  check_operand(dq, "dq");
  check_operand(dkv, "dkv");
  TORCH_CHECK(dq.sizes() == q.sizes() && dkv.sizes() == kv.sizes(), "attention: gradient shapes differ from inputs");
  check_cols(dq, dq_col, heads, "dq");
  check_cols(dkv, dk_col, heads, "dk");
  check_cols(dkv, dv_col, heads, "dv");
  TORCH_CHECK(max_k >= 0, "attention: negative max_k");
  const int64_t samples = cu_q.numel() - 1;
  if (q.size(0) == 0 || kv.size(0) == 0) {   // no attention pairs at all
    if (q.size(0)) dq.narrow(1, dq_col, heads * kDh).zero_();
    if (kv.size(0)) {
      dkv.narrow(1, dk_col, heads * kDh).zero_();
      dkv.narrow(1, dv_col, heads * kDh).zero_();
    }
    return;
  }
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>());
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr<at::BFloat16>());
  a.lse = lse.data_ptr<float>();
  a.dq = reinterpret_cast<__nv_bfloat16*>(dq.data_ptr<at::BFloat16>());
  a.ldq = dq.stride(0);
  a.dq_col = (int)dq_col;
  a.dkv = reinterpret_cast<__nv_bfloat16*>(dkv.data_ptr<at::BFloat16>());
  a.ldkv = dkv.stride(0);
  a.dk_col = (int)dk_col;
  a.dv_col = (int)dv_col;
  torch::Tensor acc;
  if (max_k > kBlk) {   // dQ rows summed over several key blocks
    acc = torch::empty({q.size(0), heads * kDh}, q.options().dtype(torch::kFloat32));
    a.dq_acc = acc.data_ptr<float>();
  }
  torch::Tensor dvec = torch::empty({heads, q.size(0)}, q.options().dtype(torch::kFloat32));
  a.dvec = dvec.data_ptr<float>();
  static size_t configured[dynsmem::kMaxDevices] = {};
  TORCH_CHECK(dynsmem::opt_in(attn_bwd_kernel, kBwdSmem, configured) == cudaSuccess,
              "attention: shared-memory attribute");
  TORCH_CHECK(samples * heads < (1ll << 31), "attention: too many samples");
  const CUtensorMap tq = tma::bf16_sw128(q.data_ptr(), q.size(0), q.size(1), q.stride(0), kBlk);
  const CUtensorMap tkv = tma::bf16_sw128(kv.data_ptr(), kv.size(0), kv.size(1), kv.stride(0), kBlk);
  const CUtensorMap td = tma::bf16_sw128(dout.data_ptr(), dout.size(0), dout.size(1), heads * kDh, kBlk);
  attn_bwd_kernel<<<(unsigned)(samples * heads), kThreads, kBwdSmem, c10::cuda::getCurrentCUDAStream().stream()>>>(
      tq, tkv, td, a);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "attention backward launch failed");
}

}  // namespace

void register_attention_ops(py::module& m) {
  m.def("attn_fwd", &attn_fwd, "variable-length multi-head attention forward (tcgen05, head dim 64)",
        py::arg("q"), py::arg("q_col"), py::arg("kv"), py::arg("k_col"), py::arg("v_col"), py::arg("cu_q"),
        py::arg("cu_k"), py::arg("max_q"), py::arg("heads"), py::arg("out"), py::arg("lse"), py::arg("status"),
        py::arg("wait_ns") = 2000000000ll);
  m.def("attn_bwd", &attn_bwd, "variable-length multi-head attention backward (tcgen05, head dim 64)",
        py::arg("q"), py::arg("q_col"), py::arg("kv"), py::arg("k_col"), py::arg("v_col"), py::arg("cu_q"),
        py::arg("cu_k"), py::arg("max_k"), py::arg("heads"), py::arg("out"), py::arg("dout"), py::arg("lse"),
        py::arg("dq"), py::arg("dq_col"), py::arg("dkv"), py::arg("dk_col"), py::arg("dv_col"), py::arg("status"),
        py::arg("wait_ns") = 2000000000ll);
}
