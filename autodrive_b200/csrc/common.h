// Shared helpers for the single-source simulator core.
//
// Every simulation routine is written once as a __host__ __device__ function.
// On the GPU one thread block (CTA) owns one environment and the PAR_FOR /
// BARRIER macros spread an element loop across the block's threads with a
// __syncthreads() between dependent phases. On the host the same source runs
// serially for one environment per OpenMP thread. Routines therefore keep
// per-element state in the environment's scratch arrays (shared memory on the
// GPU), never in registers that must survive a barrier.
#pragma once

#include <cstdint>
#include <cmath>
#include <cstring>

#if defined(__CUDACC__)
#define AD_HD __host__ __device__ __forceinline__
#define AD_DEV __device__ __forceinline__
#else
#define AD_HD inline
#define AD_DEV inline
#endif

#if defined(__CUDA_ARCH__)
#define AD_TID ((int)threadIdx.x)
#define AD_NT ((int)blockDim.x)
#define PAR_FOR(i, n) for (int i = (int)threadIdx.x; i < (int)(n); i += (int)blockDim.x)
#define BARRIER() __syncthreads()
#define SERIAL_BEGIN if (threadIdx.x == 0) {
#define SERIAL_END }
// Opt-in per-phase cycle accounting of the tick kernel: thread 0 adds the
// clock64() time since the previous mark to bucket k (marks sit right after
// CTA barriers, so a bucket is that phase's share of the CTA's critical path).
// `leader` is the thread that keeps the timeline (0: robot warp / whole CTA,
// 32: FUEL warps while the two groups run concurrently).
#define PHASE_MARK_BY(s, k, leader)                                 \
  do {                                                              \
    if ((s).prof_on && (int)threadIdx.x == (leader)) {              \
      const unsigned long long t_ = clock64();                      \
      (s).prof[(k)] += t_ - (s).prof_last[(leader) ? 1 : 0];        \
      (s).prof_last[(leader) ? 1 : 0] = t_;                         \
    }                                                               \
  } while (0)
#define PHASE_MARK(s, k) PHASE_MARK_BY(s, k, 0)
#else
#define AD_TID 0
#define AD_NT 1
#define PAR_FOR(i, n) for (int i = 0; i < (int)(n); ++i)
#define BARRIER() ((void)0)
#define SERIAL_BEGIN {
#define SERIAL_END }
#define PHASE_MARK_BY(s, k, leader) ((void)0)
#define PHASE_MARK(s, k) ((void)0)
#endif

// A set of threads of the CTA that runs one phase sequence on its own:
// `rank` is this thread's index in the group, `size` the group's thread count,
// `first` its first thread; `bar` selects the group barrier (0: the whole CTA,
// -1: a single warp, >0: named barrier id). On the host every group is the one
// serial caller (rank 0, size 1) and group barriers are no-ops.
struct Group {
  int rank, size, first, bar;
};

AD_HD Group group_all() {
#if defined(__CUDA_ARCH__)
  return Group{(int)threadIdx.x, (int)blockDim.x, 0, 0};
#else
  return Group{0, 1, 0, 0};
#endif
}

AD_HD void group_sync(const Group& g) {
#if defined(__CUDA_ARCH__)
  if (g.bar == 0) __syncthreads();
  else if (g.bar < 0) __syncwarp();
  else asm volatile("bar.sync %0, %1;" :: "r"(g.bar), "r"(g.size) : "memory");
#else
  (void)g;
#endif
}

#define GFOR(i, n, g) for (int i = (g).rank; i < (int)(n); i += (g).size)

// Group-wide OR of a flag (also a group barrier). Only whole-CTA and
// single-warp groups reduce; the host caller already holds the total.
AD_HD bool group_any(const Group& g, bool v) {
#if defined(__CUDA_ARCH__)
  if (g.bar == 0) return __syncthreads_or(v) != 0;
  __syncwarp();
  return __any_sync(0xffffffffu, v) != 0;
#else
  (void)g;
  return v;
#endif
}

namespace ad {

constexpr float kPi = 3.14159265358979323846f;
constexpr float kTwoPi = 6.28318530717958647692f;
constexpr float kG = 9.81f;
constexpr float kInf = 1e30f;

AD_HD float clampf(float v, float lo, float hi) { return fminf(fmaxf(v, lo), hi); }
AD_HD float sgnf(float v) { return v > 0.f ? 1.f : (v < 0.f ? -1.f : 0.f); }
AD_HD float sqr(float v) { return v * v; }
AD_HD int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
// Product rounded on its own (never fused into a following add), so device and
// host round a*b+c the same way.
AD_HD float mul_rn(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}
AD_HD float float_from_bits(uint32_t u) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(u);
#else
  float v;
  std::memcpy(&v, &u, sizeof(v));
  return v;
#endif
}
AD_HD uint32_t float_bits(float v) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(v);
#else
  uint32_t u;
  std::memcpy(&u, &v, sizeof(u));
  return u;
#endif
}

// Wrap an angle to [-pi, pi) with the floor-remainder convention used by the
// simulator everywhere a heading is wrapped: remainder(a + pi, 2 pi) - pi.
AD_HD float wrap_angle(float a) {
  float r = fmodf(a + kPi, kTwoPi);
  if (r < 0.f) r += kTwoPi;
  return r - kPi;
}

// Signed shortest angular difference atan2(sin d, cos d).
AD_HD float angle_diff(float a, float b) {
  float d = a - b;
  return atan2f(sinf(d), cosf(d));
}

struct V2 { float x, y; };
struct V3 { float x, y, z; };

AD_HD V3 cross3(V3 a, V3 b) {
  return V3{a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x};
}
AD_HD float dot3(V3 a, V3 b) { return a.x * b.x + a.y * b.y + a.z * b.z; }
AD_HD float norm3(V3 a) { return sqrtf(dot3(a, a)); }
AD_HD float cross2(float ax, float ay, float bx, float by) { return ax * by - ay * bx; }

// ---------------------------------------------------------------------------
// Counter-based random numbers: Philox4x32-10 (Salmon, Moraes, Dror, Shaw,
// "Parallel random numbers: as easy as 1, 2, 3", SC 2011). Each draw is a pure
// function of (key, counter), so a kernel and its host twin produce identical
// streams and inactive environments never perturb the draws of active ones.
// ---------------------------------------------------------------------------
AD_HD void mulhilo32(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  uint64_t p = (uint64_t)a * (uint64_t)b;
  hi = (uint32_t)(p >> 32);
  lo = (uint32_t)p;
}

struct U4 { uint32_t x, y, z, w; };

AD_HD U4 philox4x32(U4 ctr, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo32(M0, ctr.x, hi0, lo0);
    mulhilo32(M1, ctr.z, hi1, lo1);
    ctr = U4{hi1 ^ ctr.y ^ k0, lo1, hi0 ^ ctr.w ^ k1, lo0};
    k0 += W0;
    k1 += W1;
  }
  return ctr;
}

// Uniform in [0, 1) with 24 bits of mantissa.
AD_HD float u01(uint32_t v) { return (float)(v >> 8) * (1.0f / 16777216.0f); }

// Box-Muller transform (Box & Muller 1958) of two uniforms into one normal.
AD_HD float normal_from(uint32_t a, uint32_t b) {
  float u1 = fmaxf(u01(a), 1e-7f);
  float u2 = u01(b);
  return sqrtf(-2.f * logf(u1)) * cosf(kTwoPi * u2);
}

// Stream identifiers keep the draw families of one tick disjoint.
enum RngStream : uint32_t {
  RNG_RESET = 1,
  RNG_PERCEPTION = 2,
  RNG_OPPONENT = 3,
  RNG_LAUNCH = 4,
  RNG_POLICY = 5,
  RNG_DEFENSE = 6,
};

struct Rng {
  uint32_t k0, k1;
  // counter = (env, tick, stream, element)
  AD_HD U4 draw(uint32_t env, uint32_t tick, uint32_t stream, uint32_t elem) const {
    return philox4x32(U4{env, tick, stream, elem}, k0, k1);
  }
  AD_HD float uniform(uint32_t env, uint32_t tick, uint32_t stream, uint32_t elem) const {
    return u01(draw(env, tick, stream, elem).x);
  }
};

}  // namespace ad
