// Tensor-core (tcgen05 / TMEM) kernels for the actor-critic policy
// obs(D) -> Linear(D,128) -> tanh -> Linear(128,128) -> tanh -> {actor(A), critic(1)}
// (frc_defense/tensor_training_runtime.py:40-94), categorical actions.
//
//   policy_pack      fp32 master weights -> bf16 SW128 shared-memory images in
//                    global memory, so one bulk async copy per matrix lands
//                    them in shared memory already in UMMA layout.
//   policy_act       one CTA per 128 observations: obs rows -> bf16 image,
//                    L1 and L2 on tcgen05 with fp32 accumulators in TMEM, bias +
//                    tanh epilogues from TMEM, heads on CUDA cores, then the
//                    masked categorical sample (Gumbel-max over Philox draws),
//                    its log-probability and the value
//                    (ActorCritic.sample, tensor_training_runtime.py:63-71).
//   policy_train     the same forward for a PPO minibatch gathered by index,
//                    the clipped-PPO + value + entropy loss gradient per row
//                    (tensor_training_ppo.py:403-430) and the whole backward:
//                    dH1 = dZ2 W2, dW2 = dZ2^T [H1 | 1], dW1 = dZ1^T [X | 1] on
//                    tcgen05 (bias gradients ride along as a column of ones),
//                    head gradients on CUDA cores. Each CTA writes its own
//                    partial gradient row (deterministic, no float atomics).
//   grad_reduce      sums the partial rows, adds the L2 term of the weight
//                    matrices, writes the flat gradient buffer.
//   adv_stats        sum / sum of squares / count of the minibatch advantages.
//
// The forward code is shared by act and train, so a policy's log-probability
// at sampling time and at the first PPO epoch are bitwise equal.
//
// Every wait on an mbarrier is bounded in wall-clock time; a wait that runs
// out sets a bit in a device status word and the kernel frees its TMEM and
// returns.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

#include "common.h"
#include "tc_sm100.h"
#include "smem_opt_in.h"

namespace py = pybind11;

namespace {

constexpr int kHidden = 128;
constexpr int kRows = 128;            // observations per CTA (UMMA M)
constexpr int kThreads = 256;
constexpr int kMaxObs = 191;          // obs features (+1 ones column) fit three 64-wide blocks
constexpr int kMaxHeads = 10;         // actor logits + value
constexpr int kImgCols1 = 192;        // W1 / X image width
constexpr uint32_t kBlockBytes = kRows * 128;                 // one 64-column block of a 128-row image
constexpr uint32_t kW1Bytes = 3 * kBlockBytes;                // 49152
constexpr uint32_t kW2Bytes = 2 * kBlockBytes;                // 32768
constexpr uint64_t kWaitNs = 1000000000ull;                   // 1 s

// shared-memory map (offsets from a 1024-aligned base)
constexpr uint32_t kXR = 0;
constexpr uint32_t kW1R = kXR + kW1Bytes;
constexpr uint32_t kH1R = kW1R + kW1Bytes;
constexpr uint32_t kW2R = kH1R + 3 * kBlockBytes;
constexpr uint32_t kDZ2R = kW2R + kW2Bytes;
constexpr uint32_t kMiscAct = kDZ2R;
constexpr uint32_t kMiscTrain = kDZ2R + kW2Bytes;
// misc block
constexpr uint32_t kMB1 = 0;                                   // b1[128] f32
constexpr uint32_t kMB2 = kMB1 + 512;                          // b2[128] f32
constexpr uint32_t kMWH = kMB2 + 512;                          // heads W [kMaxHeads][128] f32
constexpr uint32_t kMBH = kMWH + kMaxHeads * kHidden * 4;      // heads b [16] f32
constexpr uint32_t kMROW = kMBH + 64;                          // [128][kMaxHeads] f32 (partials, then dheads)
constexpr uint32_t kMBAR = kMROW + kRows * kMaxHeads * 4;      // 2 mbarriers
constexpr uint32_t kMTMEM = kMBAR + 16;                        // TMEM base address
constexpr uint32_t kMiscBytes = kMTMEM + 16;

constexpr uint32_t smem_bytes(bool train) { return (train ? kMiscTrain : kMiscAct) + kMiscBytes + 1024; }

struct Offsets {
  int w1, b1, w2, b2, wa, ba, wc, bc;
};

struct TcArgs {
  const float* obs;            // [N, D]
  const int64_t* idx;          // [B] rows of obs (nullptr: rows 0..B-1)
  int B, D, A;
  const __nv_bfloat16* images; // W1 image (kW1Bytes) then W2 image (kW2Bytes)
  const float* params;         // flat fp32 master parameters
  Offsets off;
  int* status;
  // act
  int mode;                    // 0 value only, 1 sample, 2 greedy
  uint32_t seed_lo, seed_hi, counter;
  int64_t* action;
  float* logp;
  float* value;
  uint8_t* mask_out;
  // train
  const int64_t* actions;      // [N]
  const uint8_t* mask;         // [N, A] or nullptr (all valid)
  const float* old_logp;       // [N]
  const float* adv;            // [N]
  const float* ret;            // [N]
  const double* adv_stats;     // sum, sum of squares, count
  const float* ent_coef;       // device scalar
  float clip, vcoef;
  float* partials;             // [gridDim.x, pstride]
  int pstride;
  float* loss_stats;           // kl_sum, clipped, entropy mean, pg mean, value-loss mean
};

__device__ __forceinline__ uint32_t bf2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Store 8 consecutive fp32 values (columns col..col+7, col % 8 == 0) of `row`
// into an SW128 image as one 16-byte chunk.
__device__ __forceinline__ void store_chunk8(uint8_t* img, int row, int col, const float* v) {
  uint4 q;
  q.x = bf2(v[0], v[1]);
  q.y = bf2(v[2], v[3]);
  q.z = bf2(v[4], v[5]);
  q.w = bf2(v[6], v[7]);
  *reinterpret_cast<uint4*>(img + tc::sw128_offset(row, col, kRows)) = q;
}

__device__ __forceinline__ float img_load(const uint8_t* img, int row, int col) {
  return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(img + tc::sw128_offset(row, col, kRows)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <bool TRAIN>
__global__ void __launch_bounds__(kThreads, 1) policy_tc_kernel(const TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xr = smem + kXR;
  uint8_t* w1r = smem + kW1R;
  uint8_t* h1r = smem + kH1R;
  uint8_t* w2r = smem + kW2R;
  uint8_t* dz2r = smem + kDZ2R;
  uint8_t* misc = smem + (TRAIN ? kMiscTrain : kMiscAct);
  float* sb1 = reinterpret_cast<float*>(misc + kMB1);
  float* sb2 = reinterpret_cast<float*>(misc + kMB2);
  float* swh = reinterpret_cast<float*>(misc + kMWH);
  float* sbh = reinterpret_cast<float*>(misc + kMBH);
  float* srow = reinterpret_cast<float*>(misc + kMROW);
  const uint32_t bar_w = tc::smem_u32(misc + kMBAR);
  const uint32_t bar_mma = bar_w + 8;
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(misc + kMTMEM);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q = warp & 3, hf = warp >> 2;
  const int r = 32 * q + lane;                     // this thread's tile row == TMEM lane
  const int row0 = blockIdx.x * kRows;
  const int nvalid = min(kRows, args.B - row0);
  const int D = args.D, A = args.A, NH = A + 1;
  const Offsets off = args.off;
  constexpr uint32_t kCols = TRAIN ? 512 : 256;
  const int ks1 = (D + 1 + 15) / 16;               // L1 k-slices (ones column included)
  uint32_t mma_phase = 0;
  bool failed = false;

  // ---- prologue: barriers, TMEM, weight copies, biases, observation tile ----
  if (tid == 0) {
    tc::mbar_init(bar_w, 1);
    tc::mbar_init(bar_mma, 1);
    tc::mbar_init_fence();
  }
  if (warp == 0) {
    tc::tmem_alloc(tc::smem_u32(s_tmem), kCols);
    tc::tmem_relinquish();
  }
  __syncthreads();
  if (tid == 0) {
    tc::mbar_arrive_expect_tx(bar_w, kW1Bytes + kW2Bytes);
    tc::bulk_g2s(tc::smem_u32(w1r), args.images, kW1Bytes, bar_w);
    tc::bulk_g2s(tc::smem_u32(w2r), reinterpret_cast<const uint8_t*>(args.images) + kW1Bytes, kW2Bytes, bar_w);
  }
  for (int i = tid; i < kHidden; i += kThreads) {
    sb1[i] = args.params[off.b1 + i];
    sb2[i] = args.params[off.b2 + i];
  }
  for (int i = tid; i < kMaxHeads * kHidden; i += kThreads) {
    const int j = i / kHidden, c = i % kHidden;
    float w = 0.f;
    if (j < A) w = args.params[off.wa + j * kHidden + c];
    else if (j == A) w = args.params[off.wc + c];
    swh[i] = w;
  }
  if (tid < 16) sbh[tid] = tid < A ? args.params[off.ba + tid] : (tid == A ? args.params[off.bc] : 0.f);
  // observation tile -> bf16 image; column D is the ones column in training
  {
    const float ones = TRAIN ? 1.f : 0.f;
    for (int e = tid; e < kRows * (kImgCols1 / 8); e += kThreads) {
      const int rr = e / (kImgCols1 / 8), c0 = (e % (kImgCols1 / 8)) * 8;
      float v[8];
      if (rr < nvalid) {
        const int64_t src = args.idx ? args.idx[row0 + rr] : (int64_t)(row0 + rr);
        const float* o = args.obs + src * (int64_t)D;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int c = c0 + k;
          v[k] = c < D ? __ldg(o + c) : (c == D ? ones : 0.f);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = 0.f;
      }
      store_chunk8(xr, rr, c0, v);
    }
    if (TRAIN) {  // H1 image block 2: ones column at 128 for valid rows, zeros elsewhere
      for (int e = tid; e < kRows * 8; e += kThreads) {
        const int rr = e / 8, c0 = 128 + (e % 8) * 8;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (c0 == 128 && rr < nvalid) v[0] = 1.f;
        store_chunk8(h1r, rr, c0, v);
      }
    }
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *s_tmem;
  const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);

  // ---- L1: Z1 = X W1^T (TMEM cols 0..127) ----
  if (tid == 0) {
    bool ok = tc::mbar_wait(bar_w, 0, kWaitNs);
    if (ok) {
      tc::tc_fence_after();
      const uint32_t id = tc::idesc_bf16(kRows, kHidden, false, false);
      for (int ks = 0; ks < ks1; ++ks)
        tc::mma_bf16(tmem + 0, tc::desc_kmajor(tc::smem_u32(xr), kRows, ks),
                     tc::desc_kmajor(tc::smem_u32(w1r), kRows, ks), id, ks > 0);
      tc::mma_commit(bar_mma);
    } else {
      atomicOr(args.status, 1);
      failed = true;
    }
  }
  if (__syncthreads_or(failed)) goto cleanup;
  failed = !tc::mbar_wait(bar_mma, mma_phase, kWaitNs);
  mma_phase ^= 1;
  if (__syncthreads_or(failed)) { if (tid == 0) atomicOr(args.status, 2); goto cleanup; }
  tc::tc_fence_after();

  // ---- epilogue 1: H1 = tanh(Z1 + b1) -> bf16 image ----
#pragma unroll
  for (int cc = 0; cc < 2; ++cc) {
    const int col0 = 64 * hf + 32 * cc;
    float v[32];
    tc::tmem_ld32(lane_base + col0, v);
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = tanhf(v[i] + sb1[col0 + i]);
#pragma unroll
    for (int m = 0; m < 4; ++m) store_chunk8(h1r, r, col0 + 8 * m, v + 8 * m);
  }
  tc::fence_proxy_async_smem();
  tc::tc_fence_before();
  __syncthreads();

  // ---- L2: Z2 = H1 W2^T (TMEM cols 128..255) ----
  if (tid == 0) {
    tc::tc_fence_after();
    const uint32_t id = tc::idesc_bf16(kRows, kHidden, false, false);
    for (int ks = 0; ks < kHidden / 16; ++ks)
      tc::mma_bf16(tmem + 128, tc::desc_kmajor(tc::smem_u32(h1r), kRows, ks),
                   tc::desc_kmajor(tc::smem_u32(w2r), kRows, ks), id, ks > 0);
    tc::mma_commit(bar_mma);
  }
  failed = !tc::mbar_wait(bar_mma, mma_phase, kWaitNs);
  mma_phase ^= 1;
  if (__syncthreads_or(failed)) { if (tid == 0) atomicOr(args.status, 2); goto cleanup; }
  tc::tc_fence_after();

  {
    // ---- epilogue 2: H2 = tanh(Z2 + b2), head partial sums ----
    float h2[64];
    float acc[kMaxHeads];
#pragma unroll
    for (int j = 0; j < kMaxHeads; ++j) acc[j] = 0.f;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int col0 = 64 * hf + 32 * cc;
      float v[32];
      tc::tmem_ld32(lane_base + 128 + col0, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float h = tanhf(v[i] + sb2[col0 + i]);
        h2[32 * cc + i] = h;
#pragma unroll
        for (int j = 0; j < kMaxHeads; ++j) acc[j] = fmaf(h, swh[j * kHidden + col0 + i], acc[j]);
      }
    }
    if (hf == 1) {
#pragma unroll
      for (int j = 0; j < kMaxHeads; ++j) srow[r * kMaxHeads + j] = acc[j];
    }
    __syncthreads();
    const bool valid = r < nvalid;
    if (hf == 0) {
      float l[kMaxHeads];
#pragma unroll
      for (int j = 0; j < kMaxHeads; ++j) l[j] = acc[j] + srow[r * kMaxHeads + j] + sbh[j];
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxHeads; ++j) if (j == A) v = l[j];
      const int grow = row0 + r;
      const int64_t src = valid ? (args.idx ? args.idx[grow] : (int64_t)grow) : 0;
      // action mask
      bool m[kMaxHeads];
      int nok = 0;
#pragma unroll
      for (int j = 0; j < kMaxHeads; ++j) {
        bool ok = false;
        if (j < A && valid) {
          if (TRAIN) ok = args.mask ? args.mask[src * A + j] != 0 : true;
          else ok = args.obs[src * (int64_t)D + (D - A) + j] > .5f;
        }
        m[j] = ok;
        nok += ok;
      }
      if (nok == 0) {  // fully masked row: uniform over all actions
#pragma unroll
        for (int j = 0; j < kMaxHeads; ++j) {
          m[j] = j < A;
          if (j < A) l[j] = 0.f;
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kMaxHeads; ++j) if (m[j]) mx = fmaxf(mx, l[j]);
      float se = 0.f;
#pragma unroll
      for (int j = 0; j < kMaxHeads; ++j) if (m[j]) se += __expf(l[j] - mx);
      const float lse = mx + __logf(se);

      if (!TRAIN) {
        if (valid) {
          if (args.mode != 0) {
            int best = 0;
            float bv = -INFINITY;
            ad::U4 u0 = ad::philox4x32(ad::U4{(uint32_t)grow, args.counter, 0u, 0u}, args.seed_lo, args.seed_hi);
            ad::U4 u1 = ad::philox4x32(ad::U4{(uint32_t)grow, args.counter, 1u, 0u}, args.seed_lo, args.seed_hi);
            ad::U4 u2 = ad::philox4x32(ad::U4{(uint32_t)grow, args.counter, 2u, 0u}, args.seed_lo, args.seed_hi);
            const uint32_t bits[12] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w, u2.x, u2.y, u2.z, u2.w};
#pragma unroll
            for (int j = 0; j < kMaxHeads; ++j) {
              if (!m[j]) continue;
              float s = l[j];
              if (args.mode == 1) {  // Gumbel-max: argmax(l + G), G = -log(-log U)
                const float uu = fminf(fmaxf(ad::u01(bits[j]), 1e-7f), 1.f - 6e-8f);
                s -= __logf(-__logf(uu));
              }
              if (s > bv) { bv = s; best = j; }
            }
            args.action[grow] = best;
            float lb = 0.f;
#pragma unroll
            for (int j = 0; j < kMaxHeads; ++j) if (j == best) lb = l[j];
            args.logp[grow] = lb - lse;
          }
          args.value[grow] = v;
          if (args.mask_out) {
#pragma unroll
            for (int j = 0; j < kMaxHeads; ++j) if (j < A) args.mask_out[(int64_t)grow * A + j] = (nok == 0) ? 0 : m[j];
          }
        }
      } else {
        float dl[kMaxHeads];
#pragma unroll
        for (int j = 0; j < kMaxHeads; ++j) dl[j] = 0.f;
        float kl = 0.f, clipped = 0.f, ent = 0.f, pg = 0.f, vl = 0.f;
        if (valid) {
          const float invB = 1.f / (float)args.B;
          const int a = (int)args.actions[src];
          const double s = args.adv_stats[0], ss = args.adv_stats[1], cnt = fmax(args.adv_stats[2], 1.0);
          const double mean = s / cnt;
          const double var = fmax(ss / cnt - mean * mean, 0.0);
          const float advn = (float)(((double)args.adv[src] - mean) / (sqrt(var) + 1e-8));
          float la = 0.f, H = 0.f;
          float p[kMaxHeads];
#pragma unroll
          for (int j = 0; j < kMaxHeads; ++j) {
            p[j] = m[j] ? __expf(l[j] - lse) : 0.f;
            if (j == a) la = l[j];
            if (m[j]) H -= p[j] * (l[j] - lse);
          }
          const float logp_a = la - lse;
          const float lr = logp_a - args.old_logp[src];
          const float ratio = __expf(lr);
          const float c = args.clip;
          const float rc = fminf(fmaxf(ratio, 1.f - c), 1.f + c);
          const float u = -advn * ratio, w = -advn * rc;
          const bool through = (ratio >= 1.f - c && ratio <= 1.f + c) || u > w;
          const float g = through ? -advn * ratio * invB : 0.f;
          const float ec = *args.ent_coef;
#pragma unroll
          for (int j = 0; j < kMaxHeads; ++j) {
            if (!m[j]) continue;
            const float lp = l[j] - lse;
            dl[j] = g * ((j == a ? 1.f : 0.f) - p[j]) + ec * invB * p[j] * (lp + H);
          }
          const float dv = args.vcoef * (v - args.ret[src]) * invB;
#pragma unroll
          for (int j = 0; j < kMaxHeads; ++j) if (j == A) dl[j] = dv;
          kl = (ratio - 1.f) - lr;
          clipped = fabsf(ratio - 1.f) > c ? 1.f : 0.f;
          ent = H * invB;
          pg = fmaxf(u, w) * invB;
          vl = .5f * (v - args.ret[src]) * (v - args.ret[src]) * invB;
        }
#pragma unroll
        for (int j = 0; j < kMaxHeads; ++j) srow[r * kMaxHeads + j] = dl[j];
        kl = warp_sum(kl);
        clipped = warp_sum(clipped);
        ent = warp_sum(ent);
        pg = warp_sum(pg);
        vl = warp_sum(vl);
        if (lane == 0) {
          atomicAdd(args.loss_stats + 0, kl);
          atomicAdd(args.loss_stats + 1, clipped);
          atomicAdd(args.loss_stats + 2, ent);
          atomicAdd(args.loss_stats + 3, pg);
          atomicAdd(args.loss_stats + 4, vl);
        }
      }
    }
    if (TRAIN) {
      __syncthreads();  // dheads rows visible to both column halves
      // dZ2 = (dheads Wh) * (1 - H2^2) -> image; H2 -> image (W1 region is free)
      float dh[kMaxHeads];
#pragma unroll
      for (int j = 0; j < kMaxHeads; ++j) dh[j] = srow[r * kMaxHeads + j];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const int col0 = 64 * hf + 8 * cc;
        float dz[8], hv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int c = col0 + i;
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < kMaxHeads; ++j) s = fmaf(dh[j], swh[j * kHidden + c], s);
          const float h = h2[8 * cc + i];
          dz[i] = s * (1.f - h * h);
          hv[i] = h;
        }
        store_chunk8(dz2r, r, col0, dz);
        store_chunk8(w1r, r, col0, hv);
      }
      tc::fence_proxy_async_smem();
      tc::tc_fence_before();
    }
  }

  if (TRAIN) {
    __syncthreads();
    // ---- dH1 = dZ2 W2 (cols 128..255), dW2 = dZ2^T [H1 | 1] (cols 256..447) ----
    if (tid == 0) {
      tc::tc_fence_after();
      const uint32_t id_h = tc::idesc_bf16(kRows, kHidden, false, true);
      const uint32_t id_w = tc::idesc_bf16(kHidden, 192, true, true);
      for (int ks = 0; ks < kHidden / 16; ++ks)
        tc::mma_bf16(tmem + 128, tc::desc_kmajor(tc::smem_u32(dz2r), kRows, ks),
                     tc::desc_mnmajor(tc::smem_u32(w2r), kRows, ks), id_h, ks > 0);
      for (int ks = 0; ks < kRows / 16; ++ks)
        tc::mma_bf16(tmem + 256, tc::desc_mnmajor(tc::smem_u32(dz2r), kRows, ks),
                     tc::desc_mnmajor(tc::smem_u32(h1r), kRows, ks), id_w, ks > 0);
      tc::mma_commit(bar_mma);
    }
    // head weight / bias gradients on CUDA cores while the tensor cores run
    {
      float* part = args.partials + (int64_t)blockIdx.x * args.pstride;
      const int c = tid & 127, jset = tid >> 7;
      const int j0 = jset ? 5 : 0, j1 = jset ? NH : min(5, NH);
      float s[5] = {0.f, 0.f, 0.f, 0.f, 0.f};
      for (int rr = 0; rr < kRows; ++rr) {
        const float h = img_load(w1r, rr, c);
#pragma unroll
        for (int jj = 0; jj < 5; ++jj)
          if (j0 + jj < j1) s[jj] = fmaf(srow[rr * kMaxHeads + j0 + jj], h, s[jj]);
      }
#pragma unroll
      for (int jj = 0; jj < 5; ++jj) {
        const int j = j0 + jj;
        if (j >= j1) continue;
        if (j < A) part[off.wa + j * kHidden + c] = s[jj];
        else part[off.wc + c] = s[jj];
      }
      if (tid < NH) {
        float sb = 0.f;
        for (int rr = 0; rr < kRows; ++rr) sb += srow[rr * kMaxHeads + tid];
        if (tid < A) part[off.ba + tid] = sb;
        else part[off.bc] = sb;
      }
    }
    failed = !tc::mbar_wait(bar_mma, mma_phase, kWaitNs);
    mma_phase ^= 1;
    if (__syncthreads_or(failed)) { if (tid == 0) atomicOr(args.status, 2); goto cleanup; }
    tc::tc_fence_after();

    // ---- epilogue 3: dZ1 = dH1 * (1 - tanh(Z1 + b1)^2) -> image; dW2 partial ----
    {
      float* part = args.partials + (int64_t)blockIdx.x * args.pstride;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int col0 = 64 * hf + 32 * cc;
        float dh[32], z[32];
        tc::tmem_ld32(lane_base + 128 + col0, dh);
        tc::tmem_ld32(lane_base + 0 + col0, z);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float h = tanhf(z[i] + sb1[col0 + i]);
          dh[i] *= 1.f - h * h;
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) store_chunk8(w1r, r, col0 + 8 * m, dh + 8 * m);
      }
      // dW2 row o = r: columns 0..127 weights, column 128 bias
      const int o = r;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int col0 = 64 * hf + 32 * cc;
        float g[32];
        tc::tmem_ld32(lane_base + 256 + col0, g);
        float4* dst = reinterpret_cast<float4*>(part + off.w2 + o * kHidden + col0);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = make_float4(g[4 * i], g[4 * i + 1], g[4 * i + 2], g[4 * i + 3]);
      }
      if (hf == 0) {  // warp-uniform branch
        float g[32];
        tc::tmem_ld32(lane_base + 256 + 128, g);
        part[off.b2 + o] = g[0];
      }
    }
    tc::fence_proxy_async_smem();
    tc::tc_fence_before();
    __syncthreads();

    // ---- dW1 = dZ1^T [X | 1] (cols 0..191) ----
    if (tid == 0) {
      tc::tc_fence_after();
      const uint32_t id_w = tc::idesc_bf16(kHidden, 192, true, true);
      for (int ks = 0; ks < kRows / 16; ++ks)
        tc::mma_bf16(tmem + 0, tc::desc_mnmajor(tc::smem_u32(w1r), kRows, ks),
                     tc::desc_mnmajor(tc::smem_u32(xr), kRows, ks), id_w, ks > 0);
      tc::mma_commit(bar_mma);
    }
    failed = !tc::mbar_wait(bar_mma, mma_phase, kWaitNs);
    mma_phase ^= 1;
    if (__syncthreads_or(failed)) { if (tid == 0) atomicOr(args.status, 2); goto cleanup; }
    tc::tc_fence_after();

    // ---- epilogue 4: dW1 partial (row o, columns 0..D-1), db1 (column D) ----
    {
      float* part = args.partials + (int64_t)blockIdx.x * args.pstride;
      const int o = r;
#pragma unroll
      for (int cc = 0; cc < 3; ++cc) {
        const int col0 = 96 * hf + 32 * cc;
        float g[32];
        tc::tmem_ld32(lane_base + col0, g);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int k = col0 + i;
          if (k < D) part[off.w1 + o * D + k] = g[i];
          else if (k == D) part[off.b1 + o] = g[i];
        }
      }
    }
  }

cleanup:
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(*s_tmem, kCols);
  }
}

// fp32 master weights -> bf16 SW128 images (W1: 3 blocks x 128 rows, W2: 2 blocks)
__global__ void policy_pack_kernel(const float* __restrict__ params, int off_w1, int off_w2, int D,
                                   __nv_bfloat16* __restrict__ images) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  uint8_t* img = reinterpret_cast<uint8_t*>(images);
  if (e < kHidden * kImgCols1) {
    const int o = e / kImgCols1, k = e % kImgCols1;
    const float w = k < D ? params[off_w1 + o * D + k] : 0.f;
    *reinterpret_cast<__nv_bfloat16*>(img + tc::sw128_offset(o, k, kRows)) = __float2bfloat16_rn(w);
  } else if (e < kHidden * kImgCols1 + kHidden * kHidden) {
    const int f = e - kHidden * kImgCols1;
    const int o = f / kHidden, i = f % kHidden;
    *reinterpret_cast<__nv_bfloat16*>(img + kW1Bytes + tc::sw128_offset(o, i, kRows)) =
        __float2bfloat16_rn(params[off_w2 + o * kHidden + i]);
  }
}

__global__ void adv_stats_kernel(const float* __restrict__ adv, const int64_t* __restrict__ idx, int B,
                                 double* __restrict__ out) {
  double s = 0., ss = 0.;
  for (int i = threadIdx.x; i < B; i += blockDim.x) {
    const double a = adv[idx ? idx[i] : i];
    s += a;
    ss += a * a;
  }
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  __shared__ double r1[32], r2[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { r1[warp] = s; r2[warp] = ss; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0., b = 0.;
    for (int w = 0; w < (int)blockDim.x / 32; ++w) { a += r1[w]; b += r2[w]; }
    out[0] = a;
    out[1] = b;
    out[2] = (double)B;
  }
}

struct L2Ranges {
  int start[4];
  int len[4];
};

__global__ void grad_reduce_kernel(const float* __restrict__ partials, int nblk, int pstride,
                                   const float* __restrict__ params, float* __restrict__ grad, int P,
                                   float l2x2, L2Ranges ranges) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  float s = 0.f;
  for (int b = 0; b < nblk; ++b) s += partials[(int64_t)b * pstride + i];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (i >= ranges.start[k] && i < ranges.start[k] + ranges.len[k]) s += l2x2 * params[i];
  grad[i] = s;
}

Offsets parse_offsets(const std::vector<int64_t>& o) {
  TORCH_CHECK(o.size() == 8, "offsets: w1, b1, w2, b2, wa, ba, wc, bc");
  return Offsets{(int)o[0], (int)o[1], (int)o[2], (int)o[3], (int)o[4], (int)o[5], (int)o[6], (int)o[7]};
}

void check_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), name, " must be a contiguous CUDA tensor");
}

template <bool TRAIN>
void launch(const TcArgs& a, cudaStream_t st) {
  const uint32_t smem = smem_bytes(TRAIN);
  static size_t configured[dynsmem::kMaxDevices] = {};   // one table per instantiation
  TORCH_CHECK(dynsmem::opt_in(policy_tc_kernel<TRAIN>, smem, configured) == cudaSuccess,
              "policy kernel shared-memory attribute");
  const int grid = (a.B + kRows - 1) / kRows;
  policy_tc_kernel<TRAIN><<<grid, kThreads, smem, st>>>(a);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "policy_tc_kernel launch failed");
}

void common_args(TcArgs& a, const torch::Tensor& obs, int A, const torch::Tensor& images,
                 const torch::Tensor& params, const std::vector<int64_t>& offsets, const torch::Tensor& status) {
  check_cuda(obs, "obs");
  check_cuda(images, "images");
  check_cuda(params, "params");
  check_cuda(status, "status");
  TORCH_CHECK(obs.scalar_type() == torch::kFloat32 && obs.dim() == 2, "obs must be float32 [N, D]");
  TORCH_CHECK(images.scalar_type() == torch::kBFloat16 && images.numel() * 2 >= kW1Bytes + kW2Bytes,
              "images must be the packed bf16 weight images");
  TORCH_CHECK(status.scalar_type() == torch::kInt32, "status must be int32");
  a.obs = obs.data_ptr<float>();
  a.D = (int)obs.size(1);
  a.A = A;
  TORCH_CHECK(a.D >= A && a.D <= kMaxObs, "obs dim must be in [action_dim, 191]");
  TORCH_CHECK(A >= 1 && A + 1 <= kMaxHeads, "action dim must be in [1, 9]");
  a.images = reinterpret_cast<const __nv_bfloat16*>(images.data_ptr<at::BFloat16>());
  a.params = params.data_ptr<float>();
  a.off = parse_offsets(offsets);
  a.status = status.data_ptr<int>();
}

void policy_pack(torch::Tensor params, std::vector<int64_t> offsets, int64_t D, torch::Tensor images) {
  check_cuda(params, "params");
  check_cuda(images, "images");
  TORCH_CHECK(images.scalar_type() == torch::kBFloat16 && images.numel() * 2 >= kW1Bytes + kW2Bytes,
              "images must hold the W1 and W2 images");
  TORCH_CHECK(D >= 1 && D <= kMaxObs, "obs dim must be in [1, 191]");
  const Offsets off = parse_offsets(offsets);
  const int n = kHidden * kImgCols1 + kHidden * kHidden;
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  policy_pack_kernel<<<(n + 255) / 256, 256, 0, st>>>(params.data_ptr<float>(), off.w1, off.w2, (int)D,
                                                      reinterpret_cast<__nv_bfloat16*>(images.data_ptr<at::BFloat16>()));
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "policy_pack_kernel launch failed");
}

void policy_act(torch::Tensor obs, int64_t A, torch::Tensor images, torch::Tensor params,
                std::vector<int64_t> offsets, int64_t mode, int64_t seed, int64_t counter, torch::Tensor action,
                torch::Tensor logp, torch::Tensor value, c10::optional<torch::Tensor> mask_out,
                torch::Tensor status) {
  TcArgs a{};
  common_args(a, obs, (int)A, images, params, offsets, status);
  a.idx = nullptr;
  a.B = (int)obs.size(0);
  check_cuda(action, "action");
  check_cuda(logp, "logp");
  check_cuda(value, "value");
  TORCH_CHECK(action.scalar_type() == torch::kInt64 && action.numel() >= a.B, "action must be int64 [N]");
  TORCH_CHECK(logp.numel() >= a.B && value.numel() >= a.B, "logp / value must have N entries");
  a.mode = (int)mode;
  a.seed_lo = (uint32_t)(seed & 0xffffffff);
  a.seed_hi = (uint32_t)((uint64_t)seed >> 32);
  a.counter = (uint32_t)counter;
  a.action = action.data_ptr<int64_t>();
  a.logp = logp.data_ptr<float>();
  a.value = value.data_ptr<float>();
  a.mask_out = nullptr;
  if (mask_out && mask_out->defined()) {
    check_cuda(*mask_out, "mask_out");
    TORCH_CHECK(mask_out->element_size() == 1 && mask_out->numel() >= (int64_t)a.B * A, "mask_out must be [N, A] bytes");
    a.mask_out = reinterpret_cast<uint8_t*>(mask_out->data_ptr());
  }
  if (a.B == 0) return;
  launch<false>(a, c10::cuda::getCurrentCUDAStream().stream());
}

void policy_train(torch::Tensor obs, torch::Tensor idx, int64_t A, torch::Tensor images, torch::Tensor params,
                  std::vector<int64_t> offsets, torch::Tensor actions, c10::optional<torch::Tensor> mask,
                  torch::Tensor old_logp, torch::Tensor adv, torch::Tensor ret, torch::Tensor adv_stats,
                  torch::Tensor ent_coef, double clip, double vcoef, torch::Tensor partials,
                  torch::Tensor loss_stats, torch::Tensor status) {
  TcArgs a{};
  common_args(a, obs, (int)A, images, params, offsets, status);
  for (auto* t : {&idx, &actions, &old_logp, &adv, &ret, &adv_stats, &ent_coef, &partials, &loss_stats})
    check_cuda(*t, "train input");
  TORCH_CHECK(idx.scalar_type() == torch::kInt64, "idx must be int64");
  TORCH_CHECK(actions.scalar_type() == torch::kInt64, "actions must be int64");
  TORCH_CHECK(adv_stats.scalar_type() == torch::kFloat64 && adv_stats.numel() >= 3, "adv_stats must be float64 [3]");
  TORCH_CHECK(ent_coef.scalar_type() == torch::kFloat32, "ent_coef must be a float32 device scalar");
  a.idx = idx.data_ptr<int64_t>();
  a.B = (int)idx.numel();
  const int grid = (a.B + kRows - 1) / kRows;
  TORCH_CHECK(partials.dim() == 2 && partials.size(0) >= grid && partials.size(1) % 4 == 0,
              "partials must be [ceil(B/128), pstride], pstride % 4 == 0");
  TORCH_CHECK(a.off.w2 % 4 == 0, "W2 offset must be 16-byte aligned in the flat buffer");
  a.actions = actions.data_ptr<int64_t>();
  a.mask = nullptr;
  if (mask && mask->defined()) {
    check_cuda(*mask, "mask");
    TORCH_CHECK(mask->element_size() == 1, "mask must be bool / uint8");
    a.mask = reinterpret_cast<const uint8_t*>(mask->data_ptr());
  }
  a.old_logp = old_logp.data_ptr<float>();
  a.adv = adv.data_ptr<float>();
  a.ret = ret.data_ptr<float>();
  a.adv_stats = adv_stats.data_ptr<double>();
  a.ent_coef = ent_coef.data_ptr<float>();
  a.clip = (float)clip;
  a.vcoef = (float)vcoef;
  a.partials = partials.data_ptr<float>();
  a.pstride = (int)partials.size(1);
  a.loss_stats = loss_stats.data_ptr<float>();
  if (a.B == 0) return;
  launch<true>(a, c10::cuda::getCurrentCUDAStream().stream());
}

void adv_stats(torch::Tensor adv, c10::optional<torch::Tensor> idx, int64_t B, torch::Tensor out) {
  check_cuda(adv, "adv");
  check_cuda(out, "out");
  TORCH_CHECK(out.scalar_type() == torch::kFloat64 && out.numel() >= 3, "out must be float64 [3]");
  const int64_t* ip = nullptr;
  if (idx && idx->defined()) {
    check_cuda(*idx, "idx");
    ip = idx->data_ptr<int64_t>();
  }
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  adv_stats_kernel<<<1, 1024, 0, st>>>(adv.data_ptr<float>(), ip, (int)B, out.data_ptr<double>());
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "adv_stats_kernel launch failed");
}

void grad_reduce(torch::Tensor partials, int64_t nblk, torch::Tensor params, torch::Tensor grad, double l2_coef,
                 std::vector<int64_t> l2_ranges) {
  check_cuda(partials, "partials");
  check_cuda(params, "params");
  check_cuda(grad, "grad");
  TORCH_CHECK(l2_ranges.size() <= 8 && l2_ranges.size() % 2 == 0, "l2 ranges: up to 4 (start, length) pairs");
  L2Ranges rg{};
  for (int k = 0; k < 4; ++k) {
    rg.start[k] = (2 * k + 1 < (int)l2_ranges.size()) ? (int)l2_ranges[2 * k] : 0;
    rg.len[k] = (2 * k + 1 < (int)l2_ranges.size()) ? (int)l2_ranges[2 * k + 1] : 0;
  }
  const int P = (int)grad.numel();
  TORCH_CHECK(partials.size(1) >= P && partials.size(0) >= nblk, "partials too small");
  auto st = c10::cuda::getCurrentCUDAStream().stream();
  grad_reduce_kernel<<<(P + 255) / 256, 256, 0, st>>>(partials.data_ptr<float>(), (int)nblk, (int)partials.size(1),
                                                      params.data_ptr<float>(), grad.data_ptr<float>(), P,
                                                      (float)(2.0 * l2_coef), rg);
  TORCH_CHECK(cudaGetLastError() == cudaSuccess, "grad_reduce_kernel launch failed");
}

}  // namespace

void register_policy_tc_ops(py::module& m) {
  m.attr("POLICY_TC_ROWS") = kRows;
  m.attr("POLICY_TC_IMAGE_ELEMS") = (int)((kW1Bytes + kW2Bytes) / 2);
  m.def("policy_pack", &policy_pack, "fp32 policy weights -> bf16 UMMA shared-memory images");
  m.def("policy_act", &policy_act, "fused tcgen05 policy forward + masked categorical sample");
  m.def("policy_train", &policy_train, "fused tcgen05 PPO minibatch forward + backward (partial gradients)");
  m.def("policy_adv_stats", &adv_stats, "minibatch advantage sum / sum of squares / count");
  m.def("policy_grad_reduce", &grad_reduce, "sum per-CTA partial gradients + L2 term into the flat gradient");
}
