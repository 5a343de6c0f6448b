// nls_scan.cuh -- exact parallel replay of a sequential fp32 accumulation.
//
// The reference accumulates softmax denominators, top-p running sums, draw
// totals and the draw itself one element at a time in fp32
// (src/nimllm/sampler.nim:54-56, 104-108, 115-120). A tree reduction rounds
// differently, and for long candidate lists (the full-sort path) the
// difference reaches 1e-4 relative (small terms are absorbed by the running
// sum). This file reproduces the sequential result bit for bit with a block
// scan.
//
// Method. While the running value v stays inside one binade [2^E, 2^(E+1))
// every representable result is a multiple of u = 2^(E-23). Adding a term a
// and rounding to nearest-even is then integer arithmetic on S = v/u:
//     S' = S + rne(a/u)              when frac(a/u) != 1/2   ("A" step)
//     S' = the even one of S+k, S+k+1 when a/u = k + 1/2       ("B" step)
// The maps {S -> S + c} and {S -> 2*ceil((S + c)/2) + d} are closed under
// composition (worked out below), so a block can scan them in parallel. A
// result that leaves the binade (the grid changes) is detected exactly on the
// u-grid and that one element is recomputed with a real fp32 add; the scan
// restarts from there with the new grid. Subtraction (the draw, r -= p) is the
// same with S = -r/u. Everything else -- the sums themselves -- is exact
// integer arithmetic.
#pragma once

#include <climits>
#include <cstdint>

namespace nls {

// f(S) = isB ? (S + a) + ((S + a) & 1) + b : S + a
struct Fn {
  long long a, b;
  int isB;
};

__device__ __forceinline__ Fn fn_identity() { return Fn{0, 0, 0}; }

// "f then g"
__device__ __forceinline__ Fn fn_compose(const Fn& f, const Fn& g) {
  if (!f.isB) {
    if (!g.isB) return Fn{f.a + g.a, 0, 0};
    return Fn{f.a + g.a, g.b, 1};
  }
  if (!g.isB) return Fn{f.a, f.b + g.a, 1};
  long long c = f.b + g.a;
  return Fn{f.a, c + (c & 1LL) + g.b, 1};
}

__device__ __forceinline__ long long fn_apply(const Fn& f, long long S) {
  long long t = S + f.a;
  return f.isB ? t + (t & 1LL) + f.b : t;
}

// The step for adding a >= 0 on the grid 2^ue. Values of a/u at or above
// 2^40 only ever occur at a binade change (they are clamped; the element is
// then recomputed exactly).
__device__ __forceinline__ Fn fn_of(float a, int ue) {
  double q = ldexp((double)a, -ue);  // exact: a power-of-two scaling
  const double kBig = 1099511627776.0;  // 2^40
  if (q >= kBig) return Fn{1LL << 40, 0, 0};
  double kf = floor(q);
  double f = q - kf;
  long long k = (long long)kf;
  if (f < 0.5) return Fn{k, 0, 0};
  if (f > 0.5) return Fn{k + 1, 0, 0};
  return Fn{k, 0, 1};
}

// 2^ue as a float (ue >= -149; below -126 a denormal)
__device__ __forceinline__ float grid_unit(int ue) {
  return ue >= -126 ? __int_as_float((ue + 127) << 23) : __int_as_float(1 << (ue + 149));
}

// fl(S * 2^ue) for |S| < 2^25 and ue >= -149: (float)S rounds once, and the
// power-of-two scaling is exact (a product below 2^-126 is a multiple of
// 2^-149 under 2^-126, which a denormal holds exactly), so this is the
// correctly rounded value -- exact for |S| <= 2^24.
__device__ __forceinline__ float grid_value(long long S, int ue) {
  return __fmul_rn((float)S, grid_unit(ue));
}

__device__ __forceinline__ int binade_exp(float v);

// v / 2^(binade_exp(v) - 23), exactly: v's significand with its hidden bit
// (denormals and zero, on the grid 2^-149: the significand alone)
__device__ __forceinline__ long long grid_S(float v) {
  const uint32_t vb = __float_as_uint(v) & 0x7fffffffu;
  return (vb >> 23) ? (long long)((vb & 0x7fffffu) | 0x800000u) : (long long)vb;
}

// half a step of the grid 2^ue as a float (0 below the denormal range: then
// no term counts as absorbed, which only costs work)
__device__ __forceinline__ float half_grid(int ue) { return __fmul_rn(grid_unit(ue), 0.5f); }

__device__ __forceinline__ int binade_exp(float v) {
  // exponent of |v| for normals; denormals and zero share the grid of
  // [2^-126, 2^-125), i.e. E = -126.
  uint32_t u = __float_as_uint(v) & 0x7fffffffu;
  int e = (int)(u >> 23) - 127;
  return e < -126 ? -126 : e;
}

// Contribution of a >= 0 (finite) on the grid 2^ue, from its bits: returns
// rne(a / 2^ue) with ties reported separately (tie = true means a/2^ue is
// k + 1/2 and the returned value is k). Values at or above 2^40 are clamped;
// they only occur at a binade change, which the caller recomputes exactly.
__device__ __forceinline__ long long grid_units(float a, int ue, bool* tie) {
  const uint32_t bits = __float_as_uint(a);
  *tie = false;
  if (bits == 0u) return 0;
  const int be = (int)(bits >> 23);
  const uint32_t m = (bits & 0x7fffffu) | (be ? 0x800000u : 0u);
  const int d = (be ? be : 1) - 150 - ue;  // a = m * 2^(d + ue)
  if (d >= 0) return d >= 17 ? (1LL << 40) : ((long long)m << d);
  const int sh = -d;
  if (sh > 25) return 0;
  const uint32_t q = m >> sh;
  const uint32_t rem = m & ((1u << sh) - 1u);
  const uint32_t half = 1u << (sh - 1);
  if (rem == half) { *tie = true; return q; }
  return q + (rem > half ? 1u : 0u);
}

struct ScanShared {
  Fn warp_tot[32];
  long long S_end;
  float v;
  int trig;
  int stopped;
  int walk_j;
  int walk_stop;
};

template <int NT>
__device__ __forceinline__ Fn block_exclusive_scan_fn(Fn x, ScanShared& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  Fn incl = x;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    Fn o;
    o.a = __shfl_up_sync(0xffffffffu, incl.a, off);
    o.b = __shfl_up_sync(0xffffffffu, incl.b, off);
    o.isB = __shfl_up_sync(0xffffffffu, incl.isB, off);
    if (lane >= off) incl = fn_compose(o, incl);
  }
  Fn excl;
  excl.a = __shfl_up_sync(0xffffffffu, incl.a, 1);
  excl.b = __shfl_up_sync(0xffffffffu, incl.b, 1);
  excl.isB = __shfl_up_sync(0xffffffffu, incl.isB, 1);
  if (lane == 0) excl = fn_identity();
  if (lane == 31) sm.warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    constexpr int NW = NT / 32;
    Fn w = (lane < NW) ? sm.warp_tot[lane] : fn_identity();
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      Fn o;
      o.a = __shfl_up_sync(0xffffffffu, w.a, off);
      o.b = __shfl_up_sync(0xffffffffu, w.b, off);
      o.isB = __shfl_up_sync(0xffffffffu, w.isB, off);
      if (lane >= off) w = fn_compose(o, w);
    }
    // exclusive per warp
    Fn e;
    e.a = __shfl_up_sync(0xffffffffu, w.a, 1);
    e.b = __shfl_up_sync(0xffffffffu, w.b, 1);
    e.isB = __shfl_up_sync(0xffffffffu, w.isB, 1);
    if (lane == 0) e = fn_identity();
    if (lane < NW) sm.warp_tot[lane] = e;
  }
  __syncthreads();
  Fn wp = sm.warp_tot[warp];
  __syncthreads();
  return fn_compose(wp, excl);
}

struct ScanResult {
  float v;     // final (or stopping) value
  int stop_j;  // element at which `stop` fired, or -1
};

struct WalkResult {
  float v;     // value after the last replayed element
  int j;       // next element to replay
  int stop_j;  // element at which `stop` fired, or -1
};

// One warp replays elements [j, j1) of the same accumulation as exact_scan,
// 32 at a time: a warp scan of the grid steps, the first element whose
// result leaves the binade or stops is redone with a real fp32 operation,
// and the next group starts right after it. Returns at the stop, at j1,
// after `max_groups` groups, or after two groups in a row without such an
// element (the caller's block scan is cheaper from there). Lanes of one warp
// only; no block barrier.
template <bool DEC, class Elem, class Stop>
__device__ WalkResult warp_walk(int j, int j1, float v, Elem elem, Stop stop, bool has_stop,
                                int max_groups) {
  const int lane = threadIdx.x & 31;
  int quiet = 0;
  for (int g = 0; g < max_groups && j < j1 && quiet < 2; ++g) {
    const int E = binade_exp(v);
    const int ue = E - 23;
    long long S0 = grid_S(v);
    if (DEC) S0 = -S0;
    const int jj = j + lane;
    const bool in = jj < j1;
    const float a = in ? elem(jj) : 0.0f;
    bool tie = false;
    const long long k = in ? grid_units(a, ue, &tie) : 0;
    long long Sb, Sn;
    if (!__any_sync(0xffffffffu, tie)) {
      // no tie: every step adds its units, so a plain prefix sum. Units are
      // clamped to 2^25 + 1 for 32-bit arithmetic: an element that large
      // leaves the binade by itself, so every element before the first
      // trigger is unclamped and the value before the trigger is exact.
      const int kc = (int)(k < (1LL << 25) ? k : (1LL << 25) + 1);
      int incl = kc;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      Sb = S0 + (long long)(incl - kc);
      Sn = Sb + kc;
    } else {
      const Fn f = in ? Fn{k, 0, tie ? 1 : 0} : fn_identity();
      Fn incl = f;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        Fn o;
        o.a = __shfl_up_sync(0xffffffffu, incl.a, off);
        o.b = __shfl_up_sync(0xffffffffu, incl.b, off);
        o.isB = __shfl_up_sync(0xffffffffu, incl.isB, off);
        if (lane >= off) incl = fn_compose(o, incl);
      }
      Fn excl;
      excl.a = __shfl_up_sync(0xffffffffu, incl.a, 1);
      excl.b = __shfl_up_sync(0xffffffffu, incl.b, 1);
      excl.isB = __shfl_up_sync(0xffffffffu, incl.isB, 1);
      if (lane == 0) excl = fn_identity();
      Sb = fn_apply(excl, S0);  // before element jj
      Sn = fn_apply(f, Sb);     // after it
    }
    bool t = false;
    if (in) {
      if (!DEC) t = (Sn >= (1LL << 24));
      else t = (Sn >= 0) || (E > -126 && Sn >= -(1LL << 23));
      if (!t && has_stop) t = stop(grid_value(DEC ? -Sn : Sn, ue));
    }
    const unsigned m = __ballot_sync(0xffffffffu, t);
    if (m == 0u) {
      const int cnt = (j1 - j < 32) ? j1 - j : 32;
      const long long Se = __shfl_sync(0xffffffffu, Sn, cnt - 1);
      v = grid_value(DEC ? -Se : Se, ue);
      j += cnt;
      ++quiet;
      continue;
    }
    quiet = 0;
    const int tl = __ffs(m) - 1;
    const long long Sp = __shfl_sync(0xffffffffu, Sb, tl);
    const float at = __shfl_sync(0xffffffffu, a, tl);
    const float vprev = grid_value(DEC ? -Sp : Sp, ue);
    v = DEC ? __fsub_rn(vprev, at) : __fadd_rn(vprev, at);
    if (has_stop && stop(v)) return WalkResult{v, j + tl + 1, j + tl};
    j += tl + 1;
  }
  return WalkResult{v, j, -1};
}

// Replays v <- fl(v + a_j) (DEC: v <- fl(v - a_j)) for j in [j0, j1), with
// a_j = elem(j) >= 0 and finite. Stops at the first j whose new value makes
// stop(value) true (the value after that element is returned). When `absorb`
// is set (increasing sums over non-increasing terms only) the scan ends as
// soon as the next term is below half a grid step: every later term then
// rounds away. All threads of the block must call; NT = blockDim.x.
template <int NT, int EPT, bool DEC, class Elem, class Stop>
__device__ ScanResult exact_scan(int j0, int j1, float v0, Elem elem, Stop stop, bool has_stop,
                                 bool absorb, ScanShared& sm) {
  const int tid = threadIdx.x;
  constexpr int CH = NT * EPT;
  float v = v0;
  int j = j0;
  while (j < j1) {
    const int E = binade_exp(v);
    const int ue = E - 23;
    long long S0 = grid_S(v);
    if (DEC) S0 = -S0;
    if (!DEC && absorb) {
      float a0 = elem(j);
      if (a0 < half_grid(ue)) break;
    }
    const int cend = (j1 - j > CH) ? j + CH : j1;
    Fn fe[EPT];
    Fn F = fn_identity();
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      int jj = j + tid * EPT + e;
      fe[e] = fn_identity();
      if (jj < cend) {
        bool tie;
        const long long k = grid_units(elem(jj), ue, &tie);
        fe[e] = Fn{k, 0, tie ? 1 : 0};
        F = fn_compose(F, fe[e]);
      }
    }
    Fn P = block_exclusive_scan_fn<NT>(F, sm);
    long long S = fn_apply(P, S0);
    int trig = INT_MAX;
    long long Strig = 0;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      int jj = j + tid * EPT + e;
      if (jj < cend && trig == INT_MAX) {
        long long Sn = fn_apply(fe[e], S);
        bool t;
        if (!DEC) t = (Sn >= (1LL << 24));
        else t = (Sn >= 0) || (E > -126 && Sn >= -(1LL << 23));
        if (!t && has_stop) t = stop(grid_value(DEC ? -Sn : Sn, ue));
        if (t) { trig = jj; Strig = S; }
        S = Sn;
      }
    }
    if (tid == 0) sm.trig = INT_MAX;
    __syncthreads();
    if (trig != INT_MAX) atomicMin(&sm.trig, trig);
    int last_owner = (cend - 1 - j) / EPT;
    if (tid == last_owner) sm.S_end = S;
    __syncthreads();
    const int tmin = sm.trig;
    if (tmin == INT_MAX) {
      long long Se = sm.S_end;
      v = grid_value(DEC ? -Se : Se, ue);
      j = cend;
      __syncthreads();
      continue;
    }
    if (trig == tmin) {
      float vprev = grid_value(DEC ? -Strig : Strig, ue);
      float a = elem(tmin);
      float vn = DEC ? __fsub_rn(vprev, a) : __fadd_rn(vprev, a);
      sm.v = vn;
      sm.stopped = has_stop ? (stop(vn) ? 1 : 0) : 0;
    }
    __syncthreads();
    v = sm.v;
    int st = sm.stopped;
    __syncthreads();
    if (st) return ScanResult{v, tmin};
    j = tmin + 1;
    // Binade changes come in runs (the first doublings of a sum, the last
    // halvings of the draw): one warp takes the elements right after this
    // one, far cheaper per change than a block scan.
    if ((threadIdx.x >> 5) == 0) {
      const WalkResult w = warp_walk<DEC>(j, j1, v, elem, stop, has_stop, 8);
      if ((threadIdx.x & 31) == 0) {
        sm.v = w.v;
        sm.walk_j = w.j;
        sm.walk_stop = w.stop_j;
      }
    }
    __syncthreads();
    v = sm.v;
    j = sm.walk_j;
    const int wstop = sm.walk_stop;
    __syncthreads();
    if (wstop >= 0) return ScanResult{v, wstop};
  }
  return ScanResult{v, -1};
}


struct FastScanShared {
  long long red[32];
  int flag[32];
};

// Same contract as exact_scan, for long sequences: each chunk first takes the
// fast path -- the sum of its elements' grid units, one block reduction -- and
// only a chunk that holds a tie, a binade change or the stop takes the
// element-by-element path of exact_scan. `stop` must be monotone along the
// sequence (true from some element on); elem(j) is called once per element
// and chunk attempt.
//
// prep(j, jend) is called by every thread at the start of each chunk, before
// any elem() of it: a block-wide hook that may fill a cache elem() reads
// (it must end with a barrier if it writes).
template <int NT, int EPT, bool DEC, class Elem, class Stop, class Prep>
__device__ ScanResult exact_scan_fast(int j0, int j1, float v0, Elem elem, Stop stop,
                                      bool has_stop, bool absorb, ScanShared& sm,
                                      FastScanShared& fs, Prep prep) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int CH = NT * EPT;
  float v = v0;
  int j = j0;
  while (j < j1) {
    const int E = binade_exp(v);
    const int ue = E - 23;
    long long S0 = grid_S(v);
    if (DEC) S0 = -S0;
    const int cend = (j1 - j > CH) ? j + CH : j1;
    prep(j, cend);
    if (!DEC && absorb) {
      const float a0 = elem(j);
      if (a0 < half_grid(ue)) break;
    }
    long long sum = 0;
    bool tie = false;
#pragma unroll
    for (int e = 0; e < EPT; ++e) {
      const int jj = j + e * NT + tid;  // strided: coalesced loads
      if (jj < cend) {
        bool t;
        sum += grid_units(elem(jj), ue, &t);
        tie |= t;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    const unsigned anytie = __ballot_sync(0xffffffffu, tie);
    if (lane == 0) { fs.red[warp] = sum; fs.flag[warp] = anytie != 0u; }
    __syncthreads();
    long long tot = (lane < NT / 32) ? fs.red[lane] : 0;
    const int any = __any_sync(0xffffffffu, (lane < NT / 32) ? fs.flag[lane] : 0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    __syncthreads();
    const long long Se = S0 + tot;
    bool fast = !any;
    if (fast) {
      if (!DEC) fast = Se < (1LL << 24);
      else fast = (E == -126) ? (Se < 0) : (Se < -(1LL << 23));
    }
    if (fast && has_stop) fast = !stop(grid_value(DEC ? -Se : Se, ue));
    if (fast) {
      v = grid_value(DEC ? -Se : Se, ue);
      j = cend;
      continue;
    }
    // Something happens inside this chunk: retry its sub-chunks of NT
    // elements on the fast path and replay only the failing ones element by
    // element.
    for (int sj = j; sj < cend; sj += NT) {
      const int send = (cend - sj > NT) ? sj + NT : cend;
      const int E2 = binade_exp(v);
      const int ue2 = E2 - 23;
      long long S2 = grid_S(v);
      if (DEC) S2 = -S2;
      bool t2 = false;
      long long sum2 = 0;
      if (sj + tid < send) sum2 = grid_units(elem(sj + tid), ue2, &t2);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum2 += __shfl_xor_sync(0xffffffffu, sum2, o);
      const unsigned tie2 = __ballot_sync(0xffffffffu, t2);
      if (lane == 0) { fs.red[warp] = sum2; fs.flag[warp] = tie2 != 0u; }
      __syncthreads();
      long long tot2 = (lane < NT / 32) ? fs.red[lane] : 0;
      const int any2 = __any_sync(0xffffffffu, (lane < NT / 32) ? fs.flag[lane] : 0);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tot2 += __shfl_xor_sync(0xffffffffu, tot2, o);
      __syncthreads();
      const long long Se2 = S2 + tot2;
      bool fast2 = !any2;
      if (fast2) {
        if (!DEC) fast2 = Se2 < (1LL << 24);
        else fast2 = (E2 == -126) ? (Se2 < 0) : (Se2 < -(1LL << 23));
      }
      if (fast2 && has_stop) fast2 = !stop(grid_value(DEC ? -Se2 : Se2, ue2));
      if (fast2) {
        v = grid_value(DEC ? -Se2 : Se2, ue2);
        continue;
      }
      ScanResult r = exact_scan<NT, 1, DEC>(sj, send, v, elem, stop, has_stop, false, sm);
      if (r.stop_j >= 0) return r;
      v = r.v;
    }
    j = cend;
  }
  return ScanResult{v, -1};
}
}  // namespace nls
