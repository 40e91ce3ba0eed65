// exact_sum.cuh -- the left-to-right fp32 sum of non-negative terms
// (s = 0; s = fl(s + a_j) for j = 0..n-1, the sum of squares of
// rms_norm_slice, src/ops/rms_norm.rs:97-100) computed by a whole CTA, with
// the same result bit for bit.
//
// Why it can be parallel. While the running sum s stays inside one ulp range
// (all values with the same spacing u = ulp(s): one binade, or the subnormals
// together with the first normal binade), s = N * u with N an integer below
// 2^24, and one step is integer arithmetic:
//   N' = N + floor(a / u) + r,  r = 1 if the remainder is above u/2, 0 below,
//   and for a remainder of exactly u/2 (round half to even) r makes N' even.
// So one step is the map N -> N + c[N & 1] (c depends on the term and u only),
// and such maps compose into maps of the same form: a run of steps inside one
// ulp range is one (c0, c1) pair, found with a segmented scan over the CTA.
//
// The plan. A parallel fp32 prefix sum P_j of the terms predicts the ulp range
// of every state. With terms of one sign, the left-to-right fp32 sum stays
// within j 2^-24 of the exact prefix, and P_j within (depth of its adds) 2^-24;
// d_j = (j + slack) 2^-23 covers both with a factor 2 to spare (slack = the
// scan depth plus the rounding of the bounds themselves). Steps whose interval
// [P_{j-1}(1-d_j), P_j(1+d_j)] lies in one ulp range are "range steps"; the
// others ("crossing steps", about a dozen for 2048 squares of normal values)
// are added by one thread in fp32. That thread walks the crossing steps in order and moves
// s over each run of range steps between them with the run's (c0, c1).
//
// Verification makes the result exact whatever the prediction did: a run is
// applied only if s really has the run's spacing u (s in the run's ulp range,
// or s == 0 with the subnormal spacing) and the run ends at N <= 2^24 (N never
// decreases, so no step of the run left the range except possibly by rounding
// up to exactly 2^24 u, which is also the fp32 result). Otherwise, and for
// non-finite terms or more crossing steps than the table holds, the CTA falls
// back to the plain serial loop.
#pragma once
#include <cstdint>

#ifndef __CUDACC__
#define __host__
#define __device__
#define __forceinline__ inline
#endif

#ifndef XSUM_STAMP
#define XSUM_STAMP(i) \
  do {                \
  } while (0)
#endif

namespace vtq {
namespace xsum {

constexpr int kNone = -100000;   // "no range step in this stretch"
constexpr int kMaxCross = 96;    // crossing steps the table holds
constexpr int kCap = 1 << 26;    // saturation of composed increments (any value > 2^24 fails)

struct Map {
  int c0, c1;  // increment of N for N even / odd
};

__host__ __device__ __forceinline__ uint32_t fbits(float x) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(x);
#else
  uint32_t u;
  __builtin_memcpy(&u, &x, 4);
  return u;
#endif
}

__host__ __device__ __forceinline__ float bitsf(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float x;
  __builtin_memcpy(&x, &u, 4);
  return x;
#endif
}

// Exponent of the fp32 spacing at a non-negative float x: -149 below 2^-125
// (subnormals and the first normal binade share it), else floor(log2 x) - 23;
// +inf gives 105, which no finite state has.
__host__ __device__ __forceinline__ int ulp_exp(float x) {
  const int ef = (int)(fbits(x) >> 23);
  return (ef > 1 ? ef : 1) - 150;
}

// A step of term a on the grid u = 2^ue, rounded by the adder itself: with
// M = 2^23 u (spacing u, N = 2^23 even) the increment of N for even N is the
// distance in ulps of fl(M + a) from M, and for odd N that of fl(M' + a) from
// M' = M + u: rounding inside one binade depends on the state only through
// its parity (round half to even). Increments of 2^23 and more (the sum left
// the binade; counted in coarser ulps past it) are clamped to kCap; any run
// containing one fails verification (N_end > 2^24), except the exact landing
// on 2^24 u, which is the fp32 result either way.
__host__ __device__ __forceinline__ Map term_map(float a, int ue) {
  const uint32_t mb = (uint32_t)(ue + 150) << 23;
#ifdef __CUDA_ARCH__
  const float e = __fadd_rn(bitsf(mb), a), o = __fadd_rn(bitsf(mb + 1), a);
#else
  const float e = bitsf(mb) + a, o = bitsf(mb + 1) + a;
#endif
  const uint32_t ce = fbits(e) - mb, co = fbits(o) - (mb + 1);
  return Map{ce > (uint32_t)kCap ? kCap : (int)ce, co > (uint32_t)kCap ? kCap : (int)co};
}

__host__ __device__ __forceinline__ int sat_add(int a, int b) {
  const int s = a + b;
  return s > kCap ? kCap : s;
}

// f, then g.
__host__ __device__ __forceinline__ Map compose(Map f, Map g) {
  const int g0 = ((f.c0 & 1) ? g.c1 : g.c0);      // N even: N + f.c0 has parity f.c0
  const int g1 = ((f.c1 + 1) & 1) ? g.c1 : g.c0;  // N odd
  return Map{sat_add(f.c0, g0), sat_add(f.c1, g1)};
}

// Apply a run with spacing 2^ue to s; false (s unchanged) when the run's
// assumptions fail. Branch-free.
__host__ __device__ __forceinline__ bool apply_run(float& s, Map m, int ue) {
  const uint32_t b = fbits(s);
  const uint32_t ef = b >> 23;  // s >= 0
  const int se = (ef > 1 ? (int)ef : 1) - 150;
  const uint32_t n = (b & 0x7fffff) | (ef ? 0x800000u : 0u);  // s == 0 gives 0
  const uint32_t ne = n + (uint32_t)((n & 1) ? m.c1 : m.c0);
  const bool ok = ef != 0xff && se == ue && ne <= (1u << 24) && (ne >= (1u << 23) || ue == -149);
  // 2^(ue + 24) for ne == 2^24 (ue + 151 == 255 gives +inf); subnormal; normal.
  const uint32_t nb = ne == (1u << 24) ? (uint32_t)(ue + 151) << 23
                      : ne < (1u << 23) ? ne
                                        : ((uint32_t)(ue + 150) << 23) | (ne & 0x7fffff);
  s = ok ? bitsf(nb) : s;
  return ok;
}

// Margin factors for steps up to index jmax: the bounds below use
// d = (jmax + slack) 2^-23 (a larger d only turns more steps into crossings).
struct Margin {
  float lo, hi;  // 1 - d, 1 + d
};
__host__ __device__ __forceinline__ Margin margin(int jmax, int slack) {
  const float d = (float)(jmax + slack) * 1.1920928955078125e-07f;
  return Margin{1.0f - d, 1.0f + d};
}

// Classify a step (state before it predicted as p_prev, after it as p): the
// spacing exponent of a range step, or kNone for a crossing step.
__host__ __device__ __forceinline__ int classify(float p_prev, float p, Margin mg) {
#ifdef __CUDA_ARCH__
  const int lo = ulp_exp(__fmul_rn(p_prev, mg.lo)), hi = ulp_exp(__fmul_rn(p, mg.hi));
#else
  const int lo = ulp_exp(p_prev * mg.lo), hi = ulp_exp(p * mg.hi);
#endif
  return lo == hi ? lo : kNone;
}

// Scan element: fl = a crossing step resets the stretch; us = spacing of the
// last range step after the last reset (kNone if none).
struct Seg {
  int fl;
  Map m;
  int us;
};

__host__ __device__ __forceinline__ Seg seg_combine(const Seg& a, const Seg& b) {
  Seg r;
  r.fl = a.fl | b.fl;
  r.m = b.fl ? b.m : compose(a.m, b.m);
  r.us = b.fl ? b.us : (b.us != kNone ? b.us : a.us);
  return r;
}

#ifdef __CUDACC__
// Shared-memory scratch of exact_serial_sum (one per CTA).
struct Scratch {
  float wsum[32];
  int wfl[32], wc0[32], wc1[32], wus[32], wcnt[32];
  float val[kMaxCross];  // the crossing steps' terms
  int rc0[kMaxCross], rc1[kMaxCross], rus[kMaxCross];
  int fc0, fc1, fus;
  int bad;
  float result;
};

__device__ __forceinline__ float serial_fold(const float* a, int n) {
  float s = 0.0f;
  for (int i = 0; i < n; i++) s = __fadd_rn(s, a[i]);
  return s;
}

// Warp-inclusive scan of Seg + crossing count (lanes below `lane`). The flag,
// the spacing (offset by 150: 1..255, 0 for kNone) and the count (n <= 16384 < 2^15)
// travel in one word: three shuffles a level.
__device__ __forceinline__ void seg_warp_scan(Seg& in, int& cnt, int lane) {
  uint32_t w = (uint32_t)cnt | ((uint32_t)(in.us == kNone ? 0 : in.us + 150) << 15) |
               ((uint32_t)in.fl << 23);
  int c0 = in.m.c0, c1 = in.m.c1;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t tw = __shfl_up_sync(0xffffffffu, w, o);
    const int t0 = __shfl_up_sync(0xffffffffu, c0, o), t1 = __shfl_up_sync(0xffffffffu, c1, o);
    if (lane >= o) {  // (earlier lanes: tw, t0, t1) then (this: w, c0, c1)
      const bool fl = (w >> 23) & 1;
      const Map m = fl ? Map{c0, c1} : compose(Map{t0, t1}, Map{c0, c1});
      const uint32_t us = (w >> 15) & 0xff, tus = (tw >> 15) & 0xff;
      const uint32_t rus = fl ? us : (us ? us : tus);
      w = ((w & 0x7fff) + (tw & 0x7fff)) | (rus << 15) | (((w | tw) & (1u << 23)));
      c0 = m.c0;
      c1 = m.c1;
    }
  }
  cnt = (int)(w & 0x7fff);
  const uint32_t us = (w >> 15) & 0xff;
  in = Seg{(int)((w >> 23) & 1), Map{c0, c1}, us ? (int)us - 150 : kNone};
}

// The left-to-right fp32 sum of a[0..n) (every a[j] >= 0 or not finite),
// computed by `nthr` threads (a multiple of 32, at most 1024; this thread is
// tid); sync() is their barrier. Each thread holds up to EPT consecutive terms
// in registers; for n > EPT * nthr one thread runs the plain loop. Returns the
// sum in every thread. `a` stays unchanged; the caller syncs before writing it
// again.
template <int EPT, class Sync>
__device__ float exact_serial_sum(const float* a, int n, Scratch* sc, int tid, int nthr,
                                  Sync sync) {
  static_assert(EPT >= 1 && EPT <= 16, "the scan's count field holds n <= 16 * 1024");
  const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
  if (n > EPT * nthr) {
    if (tid == 0) sc->result = serial_fold(a, n);
    sync();
    return sc->result;
  }
  const int ept = (n + nthr - 1) / nthr;
  const int b0 = min(tid * ept, n), cntl = min(ept, n - b0);
  XSUM_STAMP(0);
  // Depth of the prediction's adds: the chunk, two 5-level scans, 2 joins,
  // plus 8 for the rounding of the bounds.
  const Margin mg = margin(b0 + ept, ept + 20);
  // 1. The chunk in registers, its sum and prefix (fp32), non-finite check.
  float v[EPT];
#pragma unroll
  for (int i = 0; i < EPT; i++) v[i] = i < cntl ? a[b0 + i] : 0.0f;
  float cs = 0.0f;
  int nonfinite = 0;
#pragma unroll
  for (int i = 0; i < EPT; i++) {
    nonfinite |= (fbits(v[i]) >> 23) == 0xff;
    cs = __fadd_rn(cs, v[i]);
  }
  float inc = cs;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc = __fadd_rn(inc, t);
  }
  float lane_ex = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) lane_ex = 0.0f;
  nonfinite = __any_sync(0xffffffffu, nonfinite);
  if (tid == 0) sc->bad = 0;
  if (lane == 31) {
    sc->wsum[warp] = inc;
    sc->wfl[warp] = nonfinite;
  }
  sync();
  if (warp == 0) {
    float w = lane < nw ? sc->wsum[lane] : 0.0f;
    int nf = lane < nw ? sc->wfl[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w = __fadd_rn(w, t);
    }
    nf = __any_sync(0xffffffffu, nf);
    if (lane < nw) sc->wsum[lane] = w;
    if (lane == 0 && nf) sc->bad = 1;
  }
  sync();
  const bool fallback_nf = sc->bad != 0;
  const float p_base = __fadd_rn(lane_ex, warp ? sc->wsum[warp - 1] : 0.0f);
  XSUM_STAMP(1);
  // 2. Classify the steps (independent per term: unrolled), 3. segmented scan
  // of the run maps + crossing count.
  Seg acc{0, Map{0, 0}, kNone};
  int cnt = 0;
  {
    float pp = p_base;
#pragma unroll
    for (int i = 0; i < EPT; i++) {
      if (i >= cntl) break;
      const float p = __fadd_rn(pp, v[i]);
      const int us = classify(pp, p, mg);
      const Map m = term_map(v[i], us == kNone ? 0 : us);
      const bool valid = true, cross = us == kNone;
      const Seg comb = seg_combine(acc, Seg{0, m, us});
      acc.fl = cross ? 1 : (valid ? comb.fl : acc.fl);
      acc.m.c0 = cross ? 0 : (valid ? comb.m.c0 : acc.m.c0);
      acc.m.c1 = cross ? 0 : (valid ? comb.m.c1 : acc.m.c1);
      acc.us = cross ? kNone : (valid ? comb.us : acc.us);
      cnt += cross;
      pp = p;
    }
  }
  XSUM_STAMP(2);
  Seg in = acc;
  int icnt = cnt;
  seg_warp_scan(in, icnt, lane);
  sync();  // step 1's readers of wsum / wfl are done
  if (lane == 31) {
    sc->wfl[warp] = in.fl;
    sc->wc0[warp] = in.m.c0;
    sc->wc1[warp] = in.m.c1;
    sc->wus[warp] = in.us;
    sc->wcnt[warp] = icnt;
  }
  sync();
  if (warp == 0) {
    Seg w{0, Map{0, 0}, kNone};
    int wc = 0;
    if (lane < nw) {
      w = Seg{sc->wfl[lane], Map{sc->wc0[lane], sc->wc1[lane]}, sc->wus[lane]};
      wc = sc->wcnt[lane];
    }
    seg_warp_scan(w, wc, lane);
    if (lane < nw) {  // inclusive per warp
      sc->wfl[lane] = w.fl;
      sc->wc0[lane] = w.m.c0;
      sc->wc1[lane] = w.m.c1;
      sc->wus[lane] = w.us;
      sc->wcnt[lane] = wc;
    }
  }
  // The lane-exclusive part before the barrier (shuffles of `in`).
  Seg lx;
  lx.fl = __shfl_up_sync(0xffffffffu, in.fl, 1);
  lx.m.c0 = __shfl_up_sync(0xffffffffu, in.m.c0, 1);
  lx.m.c1 = __shfl_up_sync(0xffffffffu, in.m.c1, 1);
  lx.us = __shfl_up_sync(0xffffffffu, in.us, 1);
  const int lxc = __shfl_up_sync(0xffffffffu, icnt, 1);
  sync();
  XSUM_STAMP(3);
  // Exclusive prefix of this thread: the warps before, then the lanes before.
  Seg ex{0, Map{0, 0}, kNone};
  int exc = 0;
  if (warp > 0) {
    ex = Seg{sc->wfl[warp - 1], Map{sc->wc0[warp - 1], sc->wc1[warp - 1]}, sc->wus[warp - 1]};
    exc = sc->wcnt[warp - 1];
  }
  if (lane > 0) {
    ex = seg_combine(ex, lx);
    exc += lxc;
  }
  const int total = sc->wcnt[nw - 1];
  const bool fallback = fallback_nf || total > kMaxCross;
  // 4. Write the crossing table: each crossing's term and the run before it.
  if (!fallback) {
    Seg r = ex;
    int q = exc;
    float pp = p_base;
#pragma unroll
    for (int i = 0; i < EPT; i++) {
      if (i >= cntl) break;
      const float p = __fadd_rn(pp, v[i]);
      const int us = classify(pp, p, mg);
      const Map m = term_map(v[i], us == kNone ? 0 : us);
      const bool valid = true, cross = us == kNone;
      if (cross) {
        sc->val[q] = v[i];
        sc->rc0[q] = r.m.c0;
        sc->rc1[q] = r.m.c1;
        sc->rus[q] = r.us;
      }
      const Seg comb = seg_combine(r, Seg{0, m, us});
      r.fl = cross ? 1 : (valid ? comb.fl : r.fl);
      r.m.c0 = cross ? 0 : (valid ? comb.m.c0 : r.m.c0);
      r.m.c1 = cross ? 0 : (valid ? comb.m.c1 : r.m.c1);
      r.us = cross ? kNone : (valid ? comb.us : r.us);
      q += cross;
      pp = p;
    }
    if (cntl > 0 && b0 + cntl == n) {
      sc->fc0 = r.m.c0;
      sc->fc1 = r.m.c1;
      sc->fus = r.us;
    }
  }
  XSUM_STAMP(4);
  sync();
  XSUM_STAMP(5);
  // 5. One thread walks the crossings; the next entry is loaded while the
  // current one is applied, so the walk is the add chain alone.
  if (tid == 0) {
    float s = 0.0f;
    bool ok = !fallback;
    if (ok && total > 0) {
      int us = sc->rus[0], c0 = sc->rc0[0], c1 = sc->rc1[0];
      float val = sc->val[0];
      for (int q = 0; q < total; q++) {
        const int qn = q + 1 < total ? q + 1 : q;
        const int nus = sc->rus[qn], nc0 = sc->rc0[qn], nc1 = sc->rc1[qn];
        const float nval = sc->val[qn];
        if (us != kNone) ok = apply_run(s, Map{c0, c1}, us) && ok;  // one thread: no divergence
        s = __fadd_rn(s, val);
        us = nus;
        c0 = nc0;
        c1 = nc1;
        val = nval;
      }
    }
    if (ok && sc->fus != kNone) ok = apply_run(s, Map{sc->fc0, sc->fc1}, sc->fus);
    if (!ok) s = serial_fold(a, n);
    sc->result = s;
  }
  XSUM_STAMP(6);
  sync();
  return sc->result;
}
#endif

}  // namespace xsum
}  // namespace vtq
