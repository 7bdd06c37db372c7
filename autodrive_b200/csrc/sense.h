// Anonymous stereo FUEL perception for the 3v3 environment.
//
// Each robot carries two stereo pairs: an intake pair at the front bumper and
// an opposite pair at the rear bumper, lenses offset by +/- half the stereo
// baseline along the chassis lateral axis, every lens with the configured
// field of view. One sensor update of robot r:
//
//   1. visibility per lens and free piece: range, half field of view, solid
//      field boxes (+3 cm margin, segment window 0.02..0.98) and other robots
//      (circle of their chassis half-diagonal);
//   2. angular clustering per lens: visible pieces sorted by bearing; each
//      piece covers an angular interval [b - h, b + h], h = atan(d/2 / range);
//      a 256-bin depth buffer over the field of view gives every piece the
//      fraction of its interval in which it is the nearest thing seen;
//      neighbours in bearing order join one apparent object when their
//      intervals overlap, their ranges differ by <= 0.20 m and both are more
//      than 5 % visible; an object reports the visibility-weighted mean
//      position / velocity, its spatial and angular extent, the mean visible
//      fraction (its confidence) and whether it merged several pieces;
//   3. stereo fusion per pair: both lenses' objects, in bearing order seen
//      from the chassis centre, join while their angular intervals touch and
//      their ranges differ by <= 0.20 m (confidence-weighted means, union of
//      extents, max confidence);
//   4. packing: rear objects at bearing >= 0, front objects, rear objects at
//      bearing < 0 (one bearing-ordered stream), at most P detections;
//   5. anonymous association: tracks sorted by bearing; detection i may
//      update the nearest of the tracks at bearing ranks i-1..i+1 within the
//      gate (0.35 m + 4 x position noise), the lowest detection index wins a
//      contested track, unmatched detections open free slots in slot order;
//      detection quality state (per detection slot) drives dropout, range- and
//      size-dependent measurement noise perturbs the written track.
//
// The tracker never sees simulator piece indices or exact group counts.
// Reference behaviour: frc_defense/_tensor_3v3_observation.py:117-420,
// frc_defense/tensor_perception.py:193-560 and its device kernels
// (frc_defense/csrc/tensor_perception_hip_kernel.cu: visibility_3v3 :161,
// angular_cluster_cameras :1194, stereo_fusion_pack :452,
// anonymous_track_update :830). Occluding robots are modelled at their chassis
// centres.
//
// Layout: one CTA (256 threads) per (environment, robot) row on the GPU; the
// host twin runs the same source serially per row. All per-element state lives
// in the row's scratch (dynamic shared memory), carved by sense_carve().
#pragma once

#include "rules.h"

namespace ad {

constexpr int kDepthBins = 256;
constexpr int kSortBuckets = 512;  // equal-width bearing buckets over [-pi, pi]
constexpr int kDirectRankMax = 256;  // lists up to this length are ranked all-pairs
constexpr uint32_t RNG_SENSE = 7;

struct SenseScratch {
  // free-piece state of the environment [P]
  float *px, *py;
  uint8_t* pfree;
  // per-lens / per-side / association work (aliased) -----------------------
  int16_t* cidx;     // [2P] compacted element -> source index
  float* key;        // [2P] bearing of compacted element
  int16_t* order;    // [2P] sorted position -> compacted element
  float *lo, *hi, *rng;  // [2P] per compacted element
  float* frac;       // [P]  visible fraction per compacted element (lens)
  uint8_t* flag;     // [2P] per-element flag (visibility / start of a group)
  int16_t* gstart;   // [2P + 1] group start positions in sorted order
  uint32_t* bins;    // [kDepthBins] depth buffer (float bits)
  // side object list (both lenses of one pair) [2P]
  float *cx, *cy, *cvx, *cvy, *cconf, *csx, *csy, *cang;
  uint8_t *cvalid, *cmerged;
  // fused detections: rear side [0, P), front side [P, 2P)
  float *fx, *fy, *fvx, *fvy, *fconf, *fsx, *fsy, *fang, *fbear;
  uint8_t* fmerged;
  int16_t* det;      // [P] packed detection slot -> fused entry
  // association [P]
  int16_t *cand, *target;
  int32_t* winner;
  float* qual;
  uint8_t *observed, *accepted;
  int32_t* misc;     // [64] warp scratch, profile counters, occluder counts
  float* occ;        // [4 (kMaxBoxes + kMaxRobots)] occluder table of the current lens
  uint8_t* occ_on;   // [kMaxBoxes + kMaxRobots] occluders that can touch its view
  uint8_t* occ_list; // [kMaxBoxes + kMaxRobots] those occluders' indices, boxes first
                     // (misc[kOccBoxes] boxes, misc[kOccAll] in all)
  // bucketed rank sort
  int32_t* sbucket;  // [kSortBuckets + 1] bucket counts, then bucket starts
  int16_t *stmp, *sslot;  // [2P] bucket-ordered elements, slot within the bucket
};

AD_HD size_t sense_align(size_t v) { return (v + 15) & ~(size_t)15; }

// Carve the scratch for P pieces out of `base` (nullptr: size only).
AD_HD size_t sense_carve(uint8_t* base, int P, SenseScratch* s) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> uint8_t* {
    uint8_t* p = base ? base + off : nullptr;
    off = sense_align(off + bytes);
    return p;
  };
  const size_t P1 = (size_t)P, P2 = 2 * (size_t)P;
  SenseScratch t{};
  t.px = (float*)take(P1 * 4);
  t.py = (float*)take(P1 * 4);
  t.pfree = take(P1);
  t.cidx = (int16_t*)take(P2 * 2);
  t.key = (float*)take(P2 * 4);
  t.order = (int16_t*)take(P2 * 2);
  t.lo = (float*)take(P2 * 4);
  t.hi = (float*)take(P2 * 4);
  t.rng = (float*)take(P2 * 4);
  t.frac = (float*)take(P1 * 4);
  t.flag = take(P2);
  t.gstart = (int16_t*)take((P2 + 1) * 2);
  t.bins = (uint32_t*)take(kDepthBins * 4);
  t.cx = (float*)take(P2 * 4);
  t.cy = (float*)take(P2 * 4);
  t.cvx = (float*)take(P2 * 4);
  t.cvy = (float*)take(P2 * 4);
  t.cconf = (float*)take(P2 * 4);
  t.csx = (float*)take(P2 * 4);
  t.csy = (float*)take(P2 * 4);
  t.cang = (float*)take(P2 * 4);
  t.cvalid = take(P2);
  t.cmerged = take(P2);
  t.fx = (float*)take(P2 * 4);
  t.fy = (float*)take(P2 * 4);
  t.fvx = (float*)take(P2 * 4);
  t.fvy = (float*)take(P2 * 4);
  t.fconf = (float*)take(P2 * 4);
  t.fsx = (float*)take(P2 * 4);
  t.fsy = (float*)take(P2 * 4);
  t.fang = (float*)take(P2 * 4);
  t.fbear = (float*)take(P2 * 4);
  t.fmerged = take(P2);
  t.det = (int16_t*)take(P1 * 2);
  // association arrays alias the lens work (used after the last fusion)
  t.cand = t.cidx;
  t.target = t.order;
  t.winner = (int32_t*)t.lo;
  t.qual = t.hi;
  t.observed = t.flag;
  t.accepted = t.flag + P1;
  t.misc = (int32_t*)take(64 * 4);
  t.sbucket = (int32_t*)take((kSortBuckets + 1) * 4);
  t.occ = (float*)take(4 * (kMaxBoxes + kMaxRobots) * 4);
  t.occ_on = take(kMaxBoxes + kMaxRobots);
  t.occ_list = take(kMaxBoxes + kMaxRobots);
  t.stmp = (int16_t*)take(P2 * 2);
  t.sslot = (int16_t*)take(P2 * 2);
  if (s) *s = t;
  return off;
}

constexpr int SM_WARP = 0;  // misc[0, 32): per-warp counts of a compaction
// Opt-in per-phase cycle accounting (GPU only): misc[32] switches it on,
// misc[34..52) holds kSensePhases 64-bit totals plus the last mark. Thread 0
// marks right after a CTA barrier, so a bucket is that phase's share of the
// row's critical path: 0 load, 1 lens visibility, 2 lens geometry + sort,
// 3 lens depth buffer, 4 lens objects, 5 stereo fusion, 6 packing,
// 7 association.
constexpr int kSenseProfOn = 32, kSenseProfAcc = 34, kSensePhases = 8;
constexpr int kOccBoxes = 56, kOccAll = 57;   // misc slots: lengths of the near-occluder list
#if defined(__CUDA_ARCH__)
#define SENSE_MARK(s, k)                                                                       \
  do {                                                                                         \
    if ((s).misc[kSenseProfOn] && threadIdx.x == 0) {                                          \
      unsigned long long* acc_ = reinterpret_cast<unsigned long long*>((s).misc + kSenseProfAcc); \
      const unsigned long long t_ = clock64();                                                 \
      acc_[(k)] += t_ - acc_[kSensePhases];                                                    \
      acc_[kSensePhases] = t_;                                                                 \
    }                                                                                          \
  } while (0)
#else
#define SENSE_MARK(s, k) ((void)0)
#endif

// Order-preserving compaction of the indices i < n whose flag is set:
// out[0..count) = those indices ascending. Every thread returns the count.
AD_HD int sense_compact(const uint8_t* flags, int n, int16_t* out, int32_t* warp_counts) {
#if defined(__CUDA_ARCH__)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int total = 0;
  for (int b0 = 0; b0 < n; b0 += blockDim.x) {
    const int i = b0 + threadIdx.x;
    const bool f = i < n && flags[i];
    const unsigned m = __ballot_sync(0xffffffffu, f);
    if (lane == 0) warp_counts[warp] = __popc(m);
    __syncthreads();
    int before = 0, all = 0;
    for (int w2 = 0; w2 < nw; ++w2) {
      const int c = warp_counts[w2];
      before += w2 < warp ? c : 0;
      all += c;
    }
    if (f) out[total + before + __popc(m & ((1u << lane) - 1u))] = (int16_t)i;
    total += all;
    __syncthreads();
  }
  return total;
#else
  (void)warp_counts;
  int c = 0;
  for (int i = 0; i < n; ++i)
    if (flags[i]) out[c++] = (int16_t)i;
  return c;
#endif
}

AD_HD int sense_bucket(float key) {
  return clampi((int)floorf((key + kPi) * ((float)kSortBuckets / kTwoPi)), 0, kSortBuckets - 1);
}

// In-place exclusive scan of counts[0..kSortBuckets); counts[kSortBuckets] = total.
AD_HD void sense_scan_buckets(int32_t* counts, int32_t* warp_sums) {
#if defined(__CUDA_ARCH__)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int per = (kSortBuckets + blockDim.x - 1) / blockDim.x;
  const int b0 = threadIdx.x * per;
  int local = 0;
  for (int k = 0; k < per; ++k) local += b0 + k < kSortBuckets ? counts[b0 + k] : 0;
  int incl = local;
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  int carry = 0, total = 0;
  for (int w2 = 0; w2 < nw; ++w2) {
    carry += w2 < warp ? warp_sums[w2] : 0;
    total += warp_sums[w2];
  }
  int run = carry + incl - local;
  for (int k = 0; k < per; ++k) {
    if (b0 + k < kSortBuckets) {
      const int c = counts[b0 + k];
      counts[b0 + k] = run;
      run += c;
    }
  }
  if (threadIdx.x == 0) counts[kSortBuckets] = total;
  __syncthreads();
#else
  (void)warp_sums;
  int run = 0;
  for (int b = 0; b < kSortBuckets; ++b) {
    const int c = counts[b];
    counts[b] = run;
    run += c;
  }
  counts[kSortBuckets] = run;
#endif
}

// Stable rank sort of keys in [-pi, pi]: order[rank] = j ascending by key,
// ties by j. The loop that writes keys[j] also calls sense_sort_add(s, j,
// key), which drops element j into an equal-width key bucket (a bucket's
// internal order is arbitrary); after a barrier sense_rank_sort() scans the
// bucket counts, lists every bucket's elements, and each element counts the
// smaller (key, index) pairs of its own bucket. Buckets hold few elements, so
// the cost is near linear. The bucket counts are zero between sorts (cleared
// at set-up and again at the end of every sort).
AD_HD void sense_sort_add(SenseScratch& s, int j, float key) {
  const int b = sense_bucket(key);
#if defined(__CUDA_ARCH__)
  s.sslot[j] = (int16_t)atomicAdd(&s.sbucket[b], 1);
#else
  s.sslot[j] = (int16_t)s.sbucket[b]++;
#endif
}

AD_HD void sense_rank_sort(const float* keys, int n, int16_t* order, SenseScratch& s) {
  int32_t* cnt = s.sbucket;
  if (n <= kDirectRankMax) {
    // short lists: all-pairs ranks in one pass beat the bucket passes' barriers
    PAR_FOR(j, n) {
      const float kj = keys[j];
      int r = 0;
      for (int k = 0; k < n; ++k) {
        const float kk = keys[k];
        r += (kk < kj) || (kk == kj && k < j);
      }
      order[r] = (int16_t)j;
    }
    BARRIER();
    PAR_FOR(b, kSortBuckets + 1) { cnt[b] = 0; }
    return;
  }
  sense_scan_buckets(cnt, s.misc + SM_WARP);
  PAR_FOR(j, n) { s.stmp[cnt[sense_bucket(keys[j])] + s.sslot[j]] = (int16_t)j; }
  BARRIER();
  PAR_FOR(j, n) {
    const float kj = keys[j];
    const int b = sense_bucket(kj);
    const int t0 = cnt[b], t1 = cnt[b + 1];
    int r = t0;
    for (int t = t0; t < t1; ++t) {
      const int k = s.stmp[t];
      const float kk = keys[k];
      r += (kk < kj) || (kk == kj && k < j);
    }
    order[r] = (int16_t)j;
  }
  BARRIER();
  // the next sort's first bucket access follows at least one more barrier
  PAR_FOR(b, kSortBuckets + 1) { cnt[b] = 0; }
}

// Bearing of (dx, dy) relative to the unit heading (hx, hy), in [-pi, pi].
AD_HD float sense_bearing(float dx, float dy, float hx, float hy) {
  return atan2f(hx * dy - hy * dx, hx * dx + hy * dy);
}

// Lens pose c (0/1 intake left/right, 2/3 opposite left/right) of robot r:
// optical centre (lx, ly) and unit viewing direction (hx, hy).
AD_HD void sense_lens_pose(const World& w, const SimParams& sp, int e, int r, int c, float& lx, float& ly,
                           float& hx, float& hy) {
  const size_t er = (size_t)e * sp.R + r;
  const float* p = w.r_pose + er * 3;
  const float L = w.r_param[er * kNumRobotParams + RP_LENGTH];
  const float cth = cosf(p[2]), sth = sinf(p[2]);
  const float fwd = c < 2 ? .5f * L : -.5f * L;
  const float lat = (c & 1) ? -.5f * sp.stereo_baseline : .5f * sp.stereo_baseline;
  lx = p[0] + cth * fwd - sth * lat;
  ly = p[1] + sth * fwd + cth * lat;
  hx = c < 2 ? cth : -cth;
  hy = c < 2 ? sth : -sth;
}

// Occluders that can touch lens c's field of view (a circle of radius `rad`
// around (cx, cy) reaching the range disc and the view cone). Slot k of the
// row's occluder table holds solid box k (+3 cm margin) as [x0, x1, y0, y1]
// or, after the boxes, robot q as [x, y, radius^2, 0]; slot flags mark the
// occluders that matter for this lens. One slot per thread; a barrier follows.
AD_HD bool sense_occluder_near(float cx, float cy, float rad, float lx, float ly, float hx, float hy, float range,
                               float hf, bool full_fov) {
  const float dx = cx - lx, dy = cy - ly;
  const float dist = sqrtf(dx * dx + dy * dy);
  if (dist > range + rad) return false;
  if (full_fov || dist <= rad) return true;
  const float ang = fabsf(sense_bearing(dx, dy, hx, hy));
  return ang <= hf + asinf(fminf(rad / dist, 1.f));
}

AD_HD void sense_build_occluders(const World& w, const SimParams& sp, SenseScratch& s, int e, int r, float lx,
                                 float ly, float hx, float hy, float hf, bool full_fov) {
  PAR_FOR(k, sp.num_boxes + sp.R) {
    float* o = s.occ + 4 * k;
    bool near = false;
    if (k < sp.num_boxes) {
      const Box& bx = sp.boxes[k];
      const float ex = bx.hx + .03f, ey = bx.hy + .03f;
      near = sense_occluder_near(bx.cx, bx.cy, sqrtf(ex * ex + ey * ey), lx, ly, hx, hy, sp.perception_range, hf,
                                 full_fov);
      o[0] = bx.cx - ex;
      o[1] = bx.cx + ex;
      o[2] = bx.cy - ey;
      o[3] = bx.cy + ey;
    } else {
      const int q = k - sp.num_boxes;
      const size_t eq = (size_t)e * sp.R + q;
      const float* qp = w.r_pose + eq * 3;
      const float rad = robot_radius_of(w.r_param[eq * kNumRobotParams + RP_LENGTH],
                                        w.r_param[eq * kNumRobotParams + RP_WIDTH]);
      near = q != r && sense_occluder_near(qp[0], qp[1], rad, lx, ly, hx, hy, sp.perception_range, hf, full_fov);
      o[0] = qp[0];
      o[1] = qp[1];
      o[2] = rad * rad;
      o[3] = 0.f;
    }
    s.occ_on[k] = near ? 1 : 0;
  }
  BARRIER();
  // compact the near occluders (at most kMaxBoxes + kMaxRobots <= 32: one warp)
  const int nall = sp.num_boxes + sp.R;
#if defined(__CUDA_ARCH__)
  if (threadIdx.x < 32) {
    const int k = threadIdx.x;
    const bool on = k < nall && s.occ_on[k];
    const unsigned bal = __ballot_sync(0xffffffffu, on);
    if (on) s.occ_list[__popc(bal & ((1u << k) - 1u))] = (uint8_t)k;
    if (k == 0) {
      s.misc[kOccBoxes] = __popc(bal & ((1u << sp.num_boxes) - 1u));
      s.misc[kOccAll] = __popc(bal);
    }
  }
#else
  int m = 0, mb = 0;
  for (int k = 0; k < nall; ++k) {
    if (!s.occ_on[k]) continue;
    s.occ_list[m++] = (uint8_t)k;
    if (k < sp.num_boxes) mb = m;
  }
  s.misc[kOccBoxes] = mb;
  s.misc[kOccAll] = m;
#endif
}

// Segment lens -> lens + (dx, dy) blocked by a near box (ignoring the
// first and last 2 % of the segment) or passing within a near robot's
// radius (closest point strictly inside the 2..98 % window); the near
// occluders are the compacted list of sense_build_occluders.
AD_HD bool sense_occluded(const SenseScratch& s, float lx, float ly, float dx, float dy) {
  const bool par_x = fabsf(dx) < 1e-8f, par_y = fabsf(dy) < 1e-8f;
  const float ix = par_x ? 0.f : 1.f / dx, iy = par_y ? 0.f : 1.f / dy;
  const int nbox = s.misc[kOccBoxes], nall = s.misc[kOccAll];
  for (int u = 0; u < nbox; ++u) {
    const float* o = s.occ + 4 * s.occ_list[u];
    if ((par_x && (lx < o[0] || lx > o[1])) || (par_y && (ly < o[2] || ly > o[3]))) continue;
    const float tx0 = (o[0] - lx) * ix, tx1 = (o[1] - lx) * ix;
    const float ty0 = (o[2] - ly) * iy, ty1 = (o[3] - ly) * iy;
    const float nx = par_x ? -kInf : fminf(tx0, tx1), fx = par_x ? kInf : fmaxf(tx0, tx1);
    const float ny = par_y ? -kInf : fminf(ty0, ty1), fy = par_y ? kInf : fmaxf(ty0, ty1);
    if (fminf(fminf(fx, fy), .98f) >= fmaxf(fmaxf(nx, ny), .02f)) return true;
  }
  const float inv_den = 1.f / fmaxf(dx * dx + dy * dy, 1e-8f);
  for (int u = nbox; u < nall; ++u) {
    const float* o = s.occ + 4 * s.occ_list[u];
    const float t = ((o[0] - lx) * dx + (o[1] - ly) * dy) * inv_den;
    if (!(t > .02f && t < .98f)) continue;
    const float cx = lx + t * dx - o[0], cy = ly + t * dy - o[1];
    if (cx * cx + cy * cy <= o[2]) return true;
  }
  return false;
}

// Cluster what lens c sees into the side object list at offset `base`;
// returns the number of object slots written (groups, valid or not).
AD_HD int sense_lens(const World& w, const SimParams& sp, SenseScratch& s, int e, int r, int c, int base) {
  const int P = sp.P;
  float lx, ly, hx, hy;
  sense_lens_pose(w, sp, e, r, c, lx, ly, hx, hy);
  const float hf = fminf(sp.perception_fov, kPi);
  const bool full_fov = sp.perception_fov >= kPi;
  const float D = sp.ball_diameter;
  // 1. visibility: range, view cone (angle to the viewing direction <= hf,
  // tested as dot >= |d| cos hf), then the occluders near this lens
  sense_build_occluders(w, sp, s, e, r, lx, ly, hx, hy, hf, full_fov);
  PAR_FOR(b, kDepthBins) { s.bins[b] = float_bits(kInf); }
  BARRIER();
  const float range2 = sp.perception_range * sp.perception_range, cos_hf = cosf(hf);
  PAR_FOR(i, P) {
    bool vis = s.pfree[i] != 0;
    if (vis) {
      const float dx = s.px[i] - lx, dy = s.py[i] - ly;
      const float d2 = dx * dx + dy * dy;
      vis = d2 <= range2;
      if (vis && !full_fov) vis = hx * dx + hy * dy >= cos_hf * sqrtf(d2);
      if (vis) vis = !sense_occluded(s, lx, ly, dx, dy);
    }
    s.flag[i] = vis ? 1 : 0;
  }
  BARRIER();
  const int n = sense_compact(s.flag, P, s.cidx, s.misc + SM_WARP);
  SENSE_MARK(s, 1);
  // 2. geometry of the visible pieces, bearing order
  PAR_FOR(j, n) {
    const int i = s.cidx[j];
    const float dx = s.px[i] - lx, dy = s.py[i] - ly;
    const float d = sqrtf(dx * dx + dy * dy);
    const float b = sense_bearing(dx, dy, hx, hy);
    const float h = atan2f(D * .5f, fmaxf(d, 1e-4f));
    s.key[j] = b;
    sense_sort_add(s, j, b);
    s.rng[j] = d;
    s.lo[j] = fmaxf(-hf, b - h);
    s.hi[j] = fminf(hf, b + h);
  }
  BARRIER();
  sense_rank_sort(s.key, n, s.order, s);
  SENSE_MARK(s, 2);
  // 3. depth buffer and visible fractions
  const float bw = 2.f * hf / (float)kDepthBins;
  PAR_FOR(j, n) {
    const int b0 = clampi((int)floorf((fmaxf(-hf, s.lo[j]) + hf) / bw), 0, kDepthBins - 1);
    const int b1 = clampi((int)floorf((fminf(hf, s.hi[j]) + hf) / bw), 0, kDepthBins - 1);
    const uint32_t db = float_bits(s.rng[j]);
    for (int b = b0; b <= b1; ++b) {
#if defined(__CUDA_ARCH__)
      atomicMin(&s.bins[b], db);
#else
      if (db < s.bins[b]) s.bins[b] = db;
#endif
    }
  }
  BARRIER();
  PAR_FOR(j, n) {
    const int b0 = clampi((int)floorf((fmaxf(-hf, s.lo[j]) + hf) / bw), 0, kDepthBins - 1);
    const int b1 = clampi((int)floorf((fminf(hf, s.hi[j]) + hf) / bw), 0, kDepthBins - 1);
    int seen = 0;
    for (int b = b0; b <= b1; ++b) {
      seen += float_from_bits(s.bins[b]) >= s.rng[j] - 1e-4f;
    }
    s.frac[j] = (float)seen / (float)(b1 - b0 + 1);
  }
  BARRIER();
  SENSE_MARK(s, 3);
  // 4. apparent objects: runs of joined neighbours in bearing order
  PAR_FOR(t, n) {
    bool join = false;
    if (t > 0) {
      const int j = s.order[t], q = s.order[t - 1];
      join = fminf(s.hi[j], s.hi[q]) - fmaxf(s.lo[j], s.lo[q]) > 0.f && fabsf(s.rng[j] - s.rng[q]) <= .20f &&
             s.frac[j] > .05f && s.frac[q] > .05f;
    }
    s.flag[t] = join ? 0 : 1;
  }
  BARRIER();
  int groups = sense_compact(s.flag, n, s.gstart, s.misc + SM_WARP);
  const int cap = 2 * P - base;
  if (groups > cap) groups = cap;
  SERIAL_BEGIN
  s.gstart[groups] = (int16_t)n;
  SERIAL_END
  BARRIER();
  PAR_FOR(gi, groups) {
    const int t1 = gi + 1 < groups ? s.gstart[gi + 1] : n;
    float den = 0.f, mem = 0.f, sx = 0.f, sy = 0.f, vx = 0.f, vy = 0.f;
    float mnx = kInf, mny = kInf, mxx = -kInf, mxy = -kInf, mna = kInf, mxa = -kInf;
    for (int t = s.gstart[gi]; t < t1; ++t) {
      const int j = s.order[t];
      const float f = s.frac[j];
      if (f <= .05f) continue;
      const int i = s.cidx[j];
      const float x = s.px[i], y = s.py[i];
      den += f;
      mem += 1.f;
      sx += x * f;
      sy += y * f;
      vx += w.f_vel[(size_t)e * 3 * P + i] * f;
      vy += w.f_vel[(size_t)e * 3 * P + P + i] * f;
      mnx = fminf(mnx, x);
      mny = fminf(mny, y);
      mxx = fmaxf(mxx, x);
      mxy = fmaxf(mxy, y);
      mna = fminf(mna, s.lo[j]);
      mxa = fmaxf(mxa, s.hi[j]);
    }
    const int o = base + gi;
    const bool valid = den > 0.f;
    s.cvalid[o] = valid ? 1 : 0;
    s.cx[o] = valid ? sx / den : 0.f;
    s.cy[o] = valid ? sy / den : 0.f;
    s.cvx[o] = valid ? vx / den : 0.f;
    s.cvy[o] = valid ? vy / den : 0.f;
    s.csx[o] = valid ? mxx - mnx + D : 0.f;
    s.csy[o] = valid ? mxy - mny + D : 0.f;
    s.cang[o] = valid ? fmaxf(0.f, mxa - mna) : 0.f;
    s.cmerged[o] = mem > 1.f ? 1 : 0;
    s.cconf[o] = valid ? fminf(1.f, den / fmaxf(mem, 1.f)) : 0.f;
  }
  BARRIER();
  SENSE_MARK(s, 4);
  return groups;
}

// Fuse the side object list [0, m) (both lenses of one pair) into fused
// detections at [out, out + P); returns how many.
AD_HD int sense_fuse(const World& w, const SimParams& sp, SenseScratch& s, int e, int r, int side, int m,
                     int out) {
  const int P = sp.P;
  const float* p = w.r_pose + ((size_t)e * sp.R + r) * 3;
  const float sgn = side ? -1.f : 1.f;
  const float hx = sgn * cosf(p[2]), hy = sgn * sinf(p[2]);
  PAR_FOR(k, m) { s.flag[k] = s.cvalid[k]; }
  BARRIER();
  const int n = sense_compact(s.flag, m, s.cidx, s.misc + SM_WARP);
  PAR_FOR(j, n) {
    const int k = s.cidx[j];
    const float dx = s.cx[k] - p[0], dy = s.cy[k] - p[1];
    const float b = sense_bearing(dx, dy, hx, hy);
    s.key[j] = b;
    sense_sort_add(s, j, b);
    s.lo[j] = b - s.cang[k] * .5f;
    s.hi[j] = b + s.cang[k] * .5f;
    s.rng[j] = sqrtf(dx * dx + dy * dy);
  }
  BARRIER();
  sense_rank_sort(s.key, n, s.order, s);
  PAR_FOR(t, n) {
    bool join = false;
    if (t > 0) {
      const int j = s.order[t], q = s.order[t - 1];
      join = s.lo[j] <= s.hi[q] && fabsf(s.rng[j] - s.rng[q]) <= .20f;
    }
    s.flag[t] = join ? 0 : 1;
  }
  BARRIER();
  int groups = sense_compact(s.flag, n, s.gstart, s.misc + SM_WARP);
  if (groups > P) groups = P;
  SERIAL_BEGIN
  s.gstart[groups] = (int16_t)n;
  SERIAL_END
  BARRIER();
  PAR_FOR(gi, groups) {
    const int t1 = gi + 1 < groups ? s.gstart[gi + 1] : n;
    int members = 0;
    bool merged = false;
    float ws = 0.f, sx = 0.f, sy = 0.f, vx = 0.f, vy = 0.f, conf = 0.f;
    float mnx = kInf, mny = kInf, mxx = -kInf, mxy = -kInf, mna = kInf, mxa = -kInf;
    for (int t = s.gstart[gi]; t < t1; ++t) {
      const int j = s.order[t], k = s.cidx[j];
      const float wt = fmaxf(s.cconf[k], .001f);
      ++members;
      ws += wt;
      sx += s.cx[k] * wt;
      sy += s.cy[k] * wt;
      vx += s.cvx[k] * wt;
      vy += s.cvy[k] * wt;
      conf = fmaxf(conf, s.cconf[k]);
      merged = merged || s.cmerged[k];
      mnx = fminf(mnx, s.cx[k] - s.csx[k] * .5f);
      mny = fminf(mny, s.cy[k] - s.csy[k] * .5f);
      mxx = fmaxf(mxx, s.cx[k] + s.csx[k] * .5f);
      mxy = fmaxf(mxy, s.cy[k] + s.csy[k] * .5f);
      mna = fminf(mna, s.lo[j]);
      mxa = fmaxf(mxa, s.hi[j]);
    }
    const int o = out + gi;
    s.fx[o] = sx / ws;
    s.fy[o] = sy / ws;
    s.fvx[o] = vx / ws;
    s.fvy[o] = vy / ws;
    s.fconf[o] = conf;
    s.fsx[o] = mxx - mnx;
    s.fsy[o] = mxy - mny;
    s.fang[o] = mxa - mna;
    s.fbear[o] = (mna + mxa) * .5f;
    s.fmerged[o] = (merged || members > 1) ? 1 : 0;
  }
  BARRIER();
  SENSE_MARK(s, 5);
  return groups;
}

// Full sensor update of robot r of environment e (`force`: episode reset).
AD_HD void sense_row(World& w, const SimParams& sp, SenseScratch& s, int e, int r, bool force) {
  const int P = sp.P;
  const int steps = w.g_steps[(size_t)e * 2];
  if (!force && (steps % sp.perception_interval) != 0) return;
  const uint32_t tick_id = ((uint32_t)w.e_episode[e] << 14) ^ (force ? 0x3fffu : (uint32_t)steps);
  const Rng rng{sp.seed0, sp.seed1};
  const size_t base_p = (size_t)e * P;
  const size_t row = (size_t)e * sp.R + r;
  // piece state and the current-visibility reset
  PAR_FOR(i, P) {
    s.px[i] = w.f_pos[(size_t)e * 3 * P + i];
    s.py[i] = w.f_pos[(size_t)e * 3 * P + P + i];
    s.pfree[i] = (w.f_active[base_p + i] && w.f_owner[base_p + i] < 0) ? 1 : 0;
    w.t_visible[row * P + i] = 0;
  }
  PAR_FOR(b, kSortBuckets + 1) { s.sbucket[b] = 0; }
  BARRIER();
  SENSE_MARK(s, 0);
  // rear pair first, so the packed order (rear >= 0, front, rear < 0) is known
  int nside[2] = {0, 0};
  for (int side = 1; side >= 0; --side) {
    int m = sense_lens(w, sp, s, e, r, 2 * side, 0);
    m += sense_lens(w, sp, s, e, r, 2 * side + 1, m);
    nside[side] = sense_fuse(w, sp, s, e, r, side, m, side ? 0 : P);
  }
  // 4. packing: rear bearing >= 0, front, rear bearing < 0
  PAR_FOR(k, nside[1]) { s.flag[k] = s.fbear[k] >= 0.f ? 1 : 0; }
  BARRIER();
  const int n_pos = sense_compact(s.flag, nside[1], s.cidx, s.misc + SM_WARP);
  PAR_FOR(k, nside[1]) { s.flag[k] = s.fbear[k] < 0.f ? 1 : 0; }
  BARRIER();
  const int n_neg = sense_compact(s.flag, nside[1], s.order, s.misc + SM_WARP);
  const int ndet_all = n_pos + nside[0] + n_neg;
  const int ndet = ndet_all < P ? ndet_all : P;
  PAR_FOR(k, ndet) {
    int src;
    if (k < n_pos) src = s.cidx[k];
    else if (k < n_pos + nside[0]) src = P + (k - n_pos);
    else src = s.order[k - n_pos - nside[0]];
    s.det[k] = (int16_t)src;
  }
  BARRIER();
  SENSE_MARK(s, 6);
  // 5. association: live tracks in bearing order
  const float* own = w.r_pose + row * 3;
  const float* tpx = w.t_pos + row * 2 * P;
  const float* tpy = tpx + P;
  PAR_FOR(i, P) { s.flag[i] = w.t_mask[row * P + i]; }
  BARRIER();
  int16_t* tslot = s.gstart;  // compacted live slots
  const int nt = sense_compact(s.flag, P, tslot, s.misc + SM_WARP);
  const float ohx = cosf(own[2]), ohy = sinf(own[2]);
  PAR_FOR(j, nt) {
    const int k = tslot[j];
    s.key[j] = sense_bearing(tpx[k] - own[0], tpy[k] - own[1], ohx, ohy);
    sense_sort_add(s, j, s.key[j]);
  }
  BARRIER();
  int16_t* torder = s.gstart + P;  // rank -> compacted live slot
  sense_rank_sort(s.key, nt, torder, s);
  const float gate = .35f + 4.f * sp.position_noise;
  float* qstate = w.t_quality + row * P;
  PAR_FOR(i, P) { s.winner[i] = P + 1; }
  BARRIER();
  PAR_FOR(i, ndet) {
    bool observed = false;
    int cand = -1;
    const int f = s.det[i];
    const float dx = s.fx[f] - own[0], dy = s.fy[f] - own[1];
    const float dist = fmaxf(sqrtf(dx * dx + dy * dy), .05f);
    const float width = 2.f * atanf((sp.ball_diameter * .5f) / dist);
    const float inst = clampf(expf(-dist / 8.f) * fminf(width / .012f, 1.f), 0.f, 1.f) * s.fconf[f];
    const float q = (.8f * qstate[i] + .2f * inst) * s.fconf[f];
    qstate[i] = q;
    s.qual[i] = q;
    observed = rng.uniform((uint32_t)e, tick_id, RNG_SENSE, (uint32_t)(r * kMaxPieces + i)) <
               q * (1.f - sp.perception_dropout);
    if (observed) {
      float best = kInf;
      const int r0 = i - 1 < 0 ? 0 : i - 1, r1 = i + 1 < P - 1 ? i + 1 : P - 1;
      for (int rk = r0; rk <= r1; ++rk) {
        if (rk >= nt) continue;
        const int slot = tslot[torder[rk]];
        const float ex = tpx[slot] - s.fx[f], ey = tpy[slot] - s.fy[f];
        const float d = sqrtf(ex * ex + ey * ey);
        if (d < best) {
          best = d;
          cand = slot;
        }
      }
      if (cand >= 0 && best <= gate) {
#if defined(__CUDA_ARCH__)
        atomicMin(&s.winner[cand], i);
#else
        if (i < s.winner[cand]) s.winner[cand] = i;
#endif
      } else {
        cand = -1;
      }
    }
    s.cand[i] = (int16_t)cand;
    s.observed[i] = observed ? 1 : 0;
  }
  BARRIER();
  // matched detections keep their track; the rest take free slots in order
  PAR_FOR(i, ndet) {
    const int c = s.cand[i];
    const bool won = s.observed[i] && c >= 0 && s.winner[c] == i;
    s.accepted[i] = won ? 1 : 0;
    s.target[i] = (int16_t)(won ? c : -1);
    s.flag[i] = (s.observed[i] && !won) ? 1 : 0;  // needs a new slot
  }
  BARRIER();
  int16_t* needs = s.gstart;  // live-slot list no longer needed
  const int nneed = sense_compact(s.flag, ndet, needs, s.misc + SM_WARP);
  PAR_FOR(i, P) { s.flag[i] = w.t_mask[row * P + i] ? 0 : 1; }
  BARRIER();
  int16_t* freelist = s.gstart + P;
  const int nfree = sense_compact(s.flag, P, freelist, s.misc + SM_WARP);
  PAR_FOR(k, nneed) {
    if (k < nfree) {
      const int i = needs[k];
      s.target[i] = freelist[k];
      s.accepted[i] = 1;
    }
  }
  BARRIER();
  // track writes
  PAR_FOR(i, ndet) {
    if (!s.accepted[i]) continue;
    const int slot = s.target[i], f = s.det[i];
    const size_t k = row * P + slot;
    const float dx = s.fx[f] - own[0], dy = s.fy[f] - own[1];
    const float dist = fmaxf(sqrtf(dx * dx + dy * dy), .05f);
    const float width = 2.f * atanf((sp.ball_diameter * .5f) / dist);
    const float size_q = fmaxf(.15f, fminf(1.f, width / .012f));
    const float scale = sp.position_noise * (1.f + dist / 8.f) / sqrtf(size_q);
    const U4 u = rng.draw((uint32_t)e, tick_id, RNG_SENSE, 0x40000000u | (uint32_t)(r * kMaxPieces + i));
    const U4 u2 = rng.draw((uint32_t)e, tick_id, RNG_SENSE, 0x80000000u | (uint32_t)(r * kMaxPieces + i));
    const float mx = s.fx[f] + normal_from(u.x, u.y) * scale;
    const float my = s.fy[f] + normal_from(u.z, u.w) * scale;
    const float nvx = normal_from(u2.x, u2.y) * sp.velocity_noise;
    const float nvy = normal_from(u2.z, u2.w) * sp.velocity_noise;
    float* tx = w.t_pos + row * 2 * P + slot;
    float* ty = tx + P;
    float* tvx = w.t_vel + row * 2 * P + slot;
    float* tvy = tvx + P;
    const bool prior = w.t_mask[k] && w.t_age[k] <= sp.track_timeout;
    const float elapsed = fmaxf(w.t_age[k], sp.dt);
    const float vx = (prior ? *tvx + .5f * (mx - *tx) / elapsed : 0.f) + nvx;
    const float vy = (prior ? *tvy + .5f * (my - *ty) / elapsed : 0.f) + nvy;
    *tx = mx;
    *ty = my;
    *tvx = vx;
    *tvy = vy;
    w.t_age[k] = 0.f;
    w.t_mask[k] = 1;
    w.t_conf[k] = s.qual[i];
    w.t_spatial[row * 2 * P + slot] = s.fsx[f];
    w.t_spatial[row * 2 * P + P + slot] = s.fsy[f];
    w.t_angular[k] = s.fang[f];
    w.t_merged[k] = s.fmerged[f];
    w.t_visible[k] = 1;
  }
  BARRIER();
  SENSE_MARK(s, 7);
}

}  // namespace ad
