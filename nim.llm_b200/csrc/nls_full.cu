// nls_full.cu -- rows that need more than a small top-k: top_k <= 0 or
// top_k >= vocab (the reference's full stable sort, sampler.nim:96-97),
// 256 < top_k < vocab (the heap path with a large k, sampler.nim:86-95), and
// rows the streaming kernel handed over (candidate buffers overflowed, an
// optimistic threshold that proved too high, or a penalty window with too
// many distinct ids for its table). A row whose window and bias list exceed
// this kernel's own table too is patched whole in the row's scratch slot.
//
// One 1024-thread CTA per row, persistent over its work (rows claimed from
// the batch, or the list the streaming kernel handed over), with its own
// scratch slot of 4 x vocab words in HBM/L2:
//   KY[i]  order key of logit i (index order),
//   SK[j]  (key << 32 | index) grouped by value bucket, candidate order
//          between windows, sorted inside a window once a scan needs it,
//   TT[j]  x_j = y_j - max (written with SK) until its window is sorted,
//          then t_j = expf(x_j) exactly.
// Steps:
//   1. transform: penalties and bias (precomputed per patched position),
//      temperature; KY gets each logit's key, whose ascending order is the
//      reference's candidate order (descending value);
//   2. coarse bucketing: 256 buckets linear in (max - y) -- monotone, so
//      bucket order is candidate order -- filled tile by tile through a
//      shared-memory counting sort, so SK is written in contiguous runs.
//      Windows are runs of whole buckets of at most 8191 positions. A row
//      with a bucket beyond 4096 (heavily repeated values) is sorted by the
//      LSD radix fallback instead;
//   3. the reference's sequential fp32 sums -- softmax denominator, top-p
//      running sum, draw total and the draw -- replayed exactly
//      (nls_scan.cuh), window by window. Inside one binade of the running
//      value, with no rounding tie and no stop, a window's effect is the sum
//      of its terms' grid units whatever their order, so such a window is
//      summed in bucket order from exp estimates (exact where an estimate
//      is too close to a rounding boundary), two adjacent windows in one
//      pass when the previous window predicts that the binade holds over
//      both. Only a window where
//      something order-sensitive happens is sorted in shared memory (fine
//      buckets and insertion sorts on (key, index)) and replayed in order
//      from a shared-memory copy of its exact t values. The min-p cut is a
//      key threshold and is counted without sorting;
//   4. the drawn position is mapped back to a token id with the reference's
//      tie order (ascending index for the stable sort; for the heap path,
//      descending index and the heap's survivor rule among ties at the k-th
//      value).
#include <climits>
#include <atomic>
#include <type_traits>

#include <cooperative_groups.h>

#include "nls_common.cuh"
#include "nls_kernels.h"
#include "nls_scan.cuh"
#include "nls_tma.cuh"

namespace nls {

constexpr int FT_THREADS = 1024;
constexpr int FT_EPT = 4;
constexpr int FT_TILE = FT_THREADS * FT_EPT;
constexpr int FT_WARPS = FT_THREADS / 32;
static_assert(FT_WARPS == 32, "a warp reduces one per-warp partial per lane");
static_assert(FT_WARPS <= 32, "block reductions keep one warp partial per lane");
constexpr int FT_HASH_LOG2 = 12;
constexpr int FT_GSHIFT = 2;
constexpr int FT_NB = 256;         // coarse value buckets (first level)
constexpr int FT_TILE1 = 8192;     // elements per scatter tile
constexpr int FT_WIN = 4096;       // a window holds the buckets starting in FT_WIN positions
constexpr int FT_BUCKET_MAX = 4096;  // larger coarse buckets take the LSD fallback
constexpr int FT_BIG = 8192;       // window capacity (FT_WIN + FT_BUCKET_MAX)
constexpr int FT_NB2 = 4096;       // fine buckets per window (second level)
constexpr int FT_INS_MAX = 64;     // fine buckets up to this size: one-thread insertion sort
constexpr int FT_BIGLIST = 64;
constexpr int FT_MAXWIN = kMaxVocab / FT_WIN;  // windows of the largest vocabulary
constexpr float FT_DCAP = 110.0f;  // expf(-110) is 0: beyond this t_j is 0

// one replay iteration's outcome, from warp 0
struct ReplayShared {
  float v;    // the running value after the iteration
  int j;      // the next position
  int stop;   // the position where the stop fired, or -1
  int event;  // whether a group held an event (else the span grows)
};

struct FullShared {
  union {  // the patch table is dead once the row is transformed
    struct {
      int hkey[1 << FT_HASH_LOG2];
      int hcnt[1 << FT_HASH_LOG2];
      float hbias[1 << FT_HASH_LOG2];
      int hflag[1 << FT_HASH_LOG2];
    } pt;
    unsigned long long bufB[FT_BIG];
  } ph;
  uint32_t hist2[FT_NB2];
  uint32_t off2[FT_NB2];
  union {
    unsigned long long big[FT_BIG];  // window buffer A / tile staging / block-sort buffer
    int wcnt[FT_WARPS][257];
  } u;
  uint32_t h1[FT_NB];
  uint32_t s1[FT_NB];
  uint32_t c1[FT_NB];
  uint32_t lc[FT_NB];
  uint32_t lo1[FT_NB];
  uint32_t gb1[FT_NB];
  uint32_t base[256];
  uint32_t tilecnt[256];
  ScanShared scan;
  FastScanShared fscan;
  int ired[FT_WARPS];
  float fred[FT_WARPS];
  uint32_t ured[FT_WARPS];
  uint32_t ured2[FT_WARPS];
  // an order-independent pass's per-warp partials (sum, largest term's
  // bits, tie), two sets used alternately
  uint32_t pp[2][3][FT_WARPS];
  int ibuf[8];
  float fbuf[8];
  int biglist[FT_BIGLIST];
  int nbig;
  // windows: window c spans SK positions [wstart[c], wstart[c+1]) and the
  // coarse buckets [wbkt[c], wbkt[c+1]); wstate[c] = 0 bucket order, 2 sorted
  // with TT (exact t per position) filled
  int wstart[FT_MAXWIN + 1];
  int wbkt[FT_MAXWIN + 1];
  int wstate[FT_MAXWIN];
  int cwin;  // window whose exact t values sit in u.big (as floats), or -1
  // replay of a sorted window: grid-unit sums of its 32-position groups and
  // their ties, two sets used alternately
  uint32_t gsum[2][FT_BIG / 32];
  int gtie[2][FT_BIG / 32];
  ReplayShared rpl[2];
  long long gS;
  int gev;
  // a cluster pair's first row: values pushed here by the partner CTA
  int x_row;
  int x_nan;
  uint32_t x_kmin, x_kmax;
  uint32_t x_h1[FT_NB];
  int counter, patch_overflow, dup, nan;
};

size_t full_smem_bytes(int V) {
  size_t groups = ((size_t)V + (1u << FT_GSHIFT) - 1) >> FT_GSHIFT;
  size_t bm_words = (groups + 31) / 32;
  bm_words = (bm_words + 3) & ~(size_t)3;
  return ((sizeof(FullShared) + 15) & ~(size_t)15) + bm_words * 4;
}

// ---- small block utilities ------------------------------------------------
__device__ int block_sum_int(int v, FullShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_add_sync(0xffffffffu, v);
  if (lane == 0) S.ired[warp] = v;
  __syncthreads();
  const int tot = __reduce_add_sync(0xffffffffu, lane < FT_WARPS ? S.ired[lane] : 0);
  __syncthreads();
  return tot;
}

__device__ int block_max_int(int v, FullShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_max_sync(0xffffffffu, v);
  if (lane == 0) S.ired[warp] = v;
  __syncthreads();
  const int m = __reduce_max_sync(0xffffffffu, lane < FT_WARPS ? S.ired[lane] : INT_MIN);
  __syncthreads();
  return m;
}

__device__ int block_excl_sum_int(int v, int* total, FullShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) S.ired[warp] = incl;
  __syncthreads();
  const int c = lane < FT_WARPS ? S.ired[lane] : 0;  // total of warp `lane`
  const int wpre = __reduce_add_sync(0xffffffffu, lane < warp ? c : 0);
  const int tot = __reduce_add_sync(0xffffffffu, c);
  __syncthreads();
  *total = tot;
  return wpre + incl - v;
}

// Index of the nth (0-based) position i in [0, limit) with pred(i), in
// ascending order; -1 if there is none.
template <class Pred>
__device__ int block_find_nth(int limit, int nth, Pred pred, FullShared& S) {
  int running = 0;
  for (int c0 = 0; c0 < limit; c0 += FT_TILE) {
    int cnt = 0;
#pragma unroll
    for (int e = 0; e < FT_EPT; ++e) {
      int i = c0 + threadIdx.x * FT_EPT + e;
      if (i < limit && pred(i)) ++cnt;
    }
    int tot;
    int ex = block_excl_sum_int(cnt, &tot, S);
    if (running + tot > nth) {
      const int want = nth - running;
      if (want >= ex && want < ex + cnt) {
        int k = want - ex;
#pragma unroll
        for (int e = 0; e < FT_EPT; ++e) {
          int i = c0 + threadIdx.x * FT_EPT + e;
          if (i < limit && pred(i)) {
            if (k == 0) S.ibuf[0] = i;
            --k;
          }
        }
      }
      __syncthreads();
      int r = S.ibuf[0];
      __syncthreads();
      return r;
    }
    running += tot;
  }
  return -1;
}

template <class Pred>
__device__ int block_count(int limit, Pred pred, FullShared& S) {
  int c = 0;
  for (int i = threadIdx.x; i < limit; i += FT_THREADS) c += pred(i) ? 1 : 0;
  return block_sum_int(c, S);
}

// first position in the ascending array `B` with B[i] >= key (or > key)
__device__ __forceinline__ int lower_bound_u32(const uint32_t* B, int n, uint32_t key) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (B[mid] < key) lo = mid + 1; else hi = mid;
  }
  return lo;
}
__device__ __forceinline__ int upper_bound_u32(const uint32_t* B, int n, uint32_t key) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if (B[mid] <= key) lo = mid + 1; else hi = mid;
  }
  return lo;
}
// the same on the key (high word) of sorted (key << 32 | index) pairs
__device__ __forceinline__ int lower_bound_key(const unsigned long long* B, int n, uint32_t key) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if ((uint32_t)(B[mid] >> 32) < key) lo = mid + 1; else hi = mid;
  }
  return lo;
}
__device__ __forceinline__ int upper_bound_key(const unsigned long long* B, int n, uint32_t key) {
  int lo = 0, hi = n;
  while (lo < hi) {
    int mid = (lo + hi) >> 1;
    if ((uint32_t)(B[mid] >> 32) <= key) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// ---- LSD radix sort passes (keys only, stable): the fallback sort ----------
__device__ void lsd_count(const uint32_t* src, int n, int sh, FullShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int d = lane; d < 257; d += 32) S.u.wcnt[warp][d] = 0;
  __syncwarp();
  for (int t0 = 0; t0 < n; t0 += FT_TILE) {
#pragma unroll
    for (int j = 0; j < FT_EPT; ++j) {
      const int i = t0 + warp * (32 * FT_EPT) + j * 32 + lane;
      const int d = (i < n) ? (int)((src[i] >> sh) & 255u) : 256;
      const unsigned peers = __match_any_sync(0xffffffffu, d);
      if (lane == __ffs(peers) - 1 && d < 256) S.u.wcnt[warp][d] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  if (threadIdx.x < 256) {
    int c = 0;
    for (int w = 0; w < FT_WARPS; ++w) c += S.u.wcnt[w][threadIdx.x];
    S.tilecnt[threadIdx.x] = (uint32_t)c;
  }
  __syncthreads();
  if (warp == 0) {
    uint32_t loc[8];
    uint32_t sum = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) { loc[b] = S.tilecnt[lane * 8 + b]; sum += loc[b]; }
    uint32_t incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += o;
    }
    uint32_t run = incl - sum;
#pragma unroll
    for (int b = 0; b < 8; ++b) { S.base[lane * 8 + b] = run; run += loc[b]; }
  }
  __syncthreads();
}

__device__ void lsd_scatter(const uint32_t* src, uint32_t* dst, int n, int sh, FullShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned ltmask = lanemask_lt();
  for (int t0 = 0; t0 < n; t0 += FT_TILE) {
    for (int d = lane; d < 257; d += 32) S.u.wcnt[warp][d] = 0;
    __syncwarp();
    uint32_t k[FT_EPT];
    int dg[FT_EPT], rk[FT_EPT];
#pragma unroll
    for (int j = 0; j < FT_EPT; ++j) {
      const int i = t0 + warp * (32 * FT_EPT) + j * 32 + lane;
      k[j] = (i < n) ? src[i] : 0u;
      dg[j] = (i < n) ? (int)((k[j] >> sh) & 255u) : 256;
      const unsigned peers = __match_any_sync(0xffffffffu, dg[j]);
      const int before = S.u.wcnt[warp][dg[j]];
      __syncwarp();
      rk[j] = before + __popc(peers & ltmask);
      if (lane == __ffs(peers) - 1) S.u.wcnt[warp][dg[j]] = before + __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    if (threadIdx.x < 256) {
      int run = 0;
      for (int w = 0; w < FT_WARPS; ++w) {
        int c = S.u.wcnt[w][threadIdx.x];
        S.u.wcnt[w][threadIdx.x] = run;
        run += c;
      }
      S.tilecnt[threadIdx.x] = (uint32_t)run;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < FT_EPT; ++j) {
      if (dg[j] < 256) dst[S.base[dg[j]] + S.u.wcnt[warp][dg[j]] + rk[j]] = k[j];
    }
    __syncthreads();
    if (threadIdx.x < 256) S.base[threadIdx.x] += S.tilecnt[threadIdx.x];
    __syncthreads();
  }
}

// ---- sorting small segments -------------------------------------------------
// Ascending bitonic sort of 32*E keys held by one warp, element lane*E + e in
// v[e] (E a power of two).
template <int E>
__device__ __forceinline__ void warp_bitonic_asc(unsigned long long (&v)[E]) {
  const int lane = threadIdx.x & 31;
  constexpr int N = 32 * E;
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= E) {
        const int lm = j / E;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const unsigned long long o = __shfl_xor_sync(0xffffffffu, v[e], lm);
          const int i = lane * E + e;
          const bool up = (i & k) == 0;
          const bool lower = (lane & lm) == 0;
          const unsigned long long mn = v[e] < o ? v[e] : o;
          const unsigned long long mx = v[e] < o ? o : v[e];
          v[e] = (lower == up) ? mn : mx;
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if ((e & j) == 0) {
            const int e2 = e | j;
            const int i = lane * E + e;
            const bool up = (i & k) == 0;
            if ((v[e] > v[e2]) == up) {
              const unsigned long long t = v[e];
              v[e] = v[e2];
              v[e2] = t;
            }
          }
        }
      }
    }
  }
}

template <int E>
__device__ __forceinline__ void warp_sort_segment(unsigned long long* seg, int n) {
  const int lane = threadIdx.x & 31;
  unsigned long long v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    v[e] = i < n ? seg[i] : ~0ull;
  }
  warp_bitonic_asc<E>(v);
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int i = lane * E + e;
    if (i < n) seg[i] = v[e];
  }
}

// Block-wide ascending bitonic sort of n64 (power of two) keys in shared memory.
__device__ void block_bitonic_asc(unsigned long long* v, int n64) {
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int size = 2; size <= n64; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n64 / 2; i += nt) {
        int lo = 2 * i - (i & (stride - 1));
        int hi = lo + stride;
        bool asc = ((lo & size) == 0);
        unsigned long long x = v[lo], y = v[hi];
        if ((x > y) == asc) { v[lo] = y; v[hi] = x; }
      }
      __syncthreads();
    }
  }
}

// Order key of the full-sort path: ascending key == the reference's
// candidate order by value (descending logit).
__device__ __forceinline__ uint32_t desc_key(float y) { return ~fkey(y); }
__device__ __forceinline__ float desc_key_value(uint32_t kd) { return fkey_inv(~kd); }

// Value bucket of a key: linear in d = max - y, monotone, so bucket order is
// candidate order. d >= the cut (or +inf/NaN) goes to the last bucket.
struct Bucketer {
  float mx, scale, dcut;
  __device__ __forceinline__ int operator()(uint32_t kd) const {
    const float d = __fsub_rn(mx, desc_key_value(kd));
    if (!(d < dcut)) return FT_NB - 1;
    const int b = __float2int_rz(__fmul_rn(d, scale));
    return b < 0 ? 0 : (b > FT_NB - 1 ? FT_NB - 1 : b);
  }
};

// Terms of the three accumulations as functions of t = expf(y - max): the
// softmax denominator sums t itself, the top-p / total / draw sums sum
// p = t / s. exact() is the reference's arithmetic; lo()/hi() map a lower /
// upper bound of t to a lower / upper bound of the term (monotone).
// mid(a) for a = texp_estimate(x) estimates the exact term (from
// t = ref_expf(x)) to a relative error: TermT within kBracketRel = 2^-20;
// TermP adds the roundings of 1/s, of the product and of the reference's
// quotient, within 1.2 * 2^-20. `margin` is at least twice that.
struct TermT {
  static constexpr float margin = 0x1p-19f;
  __device__ float exact(float t) const { return t; }
  __device__ float mid(float a) const { return a; }
};
struct TermP {
  static constexpr float margin = 0x1p-18f;
  float s, rinv;  // rinv = 1/s rounded to nearest
  __device__ float exact(float t) const { return __fdiv_rn(t, s); }
  __device__ float mid(float a) const { return __fmul_rn(a, rinv); }
};

// ---- a top-k row with a NaN among its first k positions ------------------
// The reference's heap (sampler.nim:88-95) run as written, by one warp. Nim's
// tuple `<` on (float32, int) goes through cmp field by field (equal: next
// field; x < y: less; anything else, NaN included: not less), so a NaN is
// neither below nor above any item. A NaN pushed in the first k pushes never
// leaves the heap (only the root is replaced, and `x > h[0][0]` is false
// for a NaN root), so it is a candidate: the softmax sum is NaN and so is
// every probability (sampler.nim:51-57,100). Then top-p never stops
// (`cum >= topP` is false, :107), min-p keeps one candidate (:111-114) and
// the draw falls through to idx[n - 1] (:118-121): the token is idx[0], the
// last item popped, when min_p > 0, else idx[k - 1], the first item popped
// (the root). Its probability is NaN. Items: value bits << 32 | index.
__device__ __forceinline__ float nheap_val(unsigned long long it) {
  return __uint_as_float((uint32_t)(it >> 32));
}
__device__ __forceinline__ bool nheap_less(unsigned long long a, unsigned long long b) {
  const float va = nheap_val(a), vb = nheap_val(b);
  if (va == vb) return (uint32_t)a < (uint32_t)b;
  return va < vb;
}
// heapq's _siftdown and _siftup (the steps of std/heapqueue)
__device__ void nheap_siftdown(unsigned long long* h, int startpos, int pos) {
  const unsigned long long item = h[pos];
  while (pos > startpos) {
    const int parentpos = (pos - 1) >> 1;
    const unsigned long long parent = h[parentpos];
    if (!nheap_less(item, parent)) break;
    h[pos] = parent;
    pos = parentpos;
  }
  h[pos] = item;
}
__device__ void nheap_siftup(unsigned long long* h, int len, int pos) {
  const int startpos = pos;
  const unsigned long long item = h[pos];
  int child = 2 * pos + 1;
  while (child < len) {
    const int right = child + 1;
    if (right < len && !nheap_less(h[child], h[right])) child = right;
    h[pos] = h[child];
    pos = child;
    child = 2 * pos + 1;
  }
  h[pos] = item;
  nheap_siftdown(h, startpos, pos);
}
// Called by the 32 lanes of one warp. y(i) is the row's value at position i
// after penalties, bias and temperature. The heap lives in `sh` (shared
// memory, FT_BIG items) when k fits, else in the CTA's global scratch `gl`
// (vocab items). Lane 0 runs every heap step; the warp only looks ahead for
// the next position that the current root lets in (re-tested after every
// step, so the order of steps is the reference's).
template <class LogitFn>
__device__ void nan_heap_row(const BatchArgs& a, int row, const nls_row_params& p, int V, int K,
                             float invT, LogitFn logit, unsigned long long* sh,
                             unsigned long long* gl) {
  const int lane = threadIdx.x & 31;
  unsigned long long* h = (K <= FT_BIG) ? sh : gl;
  int len = 0;
  float root = 0.0f;  // value of h[0], valid once len == K (lane 0)
  for (int base = 0; base < V; base += 32) {
    const int i = base + lane;
    const float y = (i < V) ? __fmul_rn(logit(i), invT) : 0.0f;
    int j = -1;
    for (;;) {
      const float rv = __shfl_sync(0xffffffffu, root, 0);
      const unsigned m = __ballot_sync(0xffffffffu, lane > j && i < V && (i < K || y > rv));
      if (!m) break;
      j = __ffs(m) - 1;
      const float yj = __shfl_sync(0xffffffffu, y, j);
      if (lane == 0) {
        const unsigned long long it = ((unsigned long long)__float_as_uint(yj) << 32) | (uint32_t)(base + j);
        if (len < K) {          // h.push((x, i))
          h[len] = it;
          ++len;
          nheap_siftdown(h, 0, len - 1);
        } else if (yj > nheap_val(h[0])) {  // discard h.replace((x, i))
          h[0] = it;
          nheap_siftup(h, len, 0);
        }
        root = nheap_val(h[0]);
      }
    }
  }
  if (lane == 0) {
    unsigned long long pick = h[0];  // the first pop: idx[k - 1]
    if (p.min_p > 0.0) {             // the last pop: idx[0]
      int n = len;
      while (n > 0) {
        const unsigned long long last = h[n - 1];
        --n;
        if (n > 0) {
          pick = h[0];
          h[0] = last;
          nheap_siftup(h, n, 0);
        } else {
          pick = last;
        }
      }
    }
    a.out_ids[row] = (int64_t)(uint32_t)pick;
    if (a.out_probs) a.out_probs[row] = __uint_as_float(0x7fc00000u);
  }
  __syncwarp();
}

// The next row whose parameters select the full path, for a row-claiming
// launch (a.rows when none is left): from the classification's list (one
// atomic) when there is one, else by walking the rows from the shared
// counter (batches of a few hundred rows, where listing them first would
// only delay the claims).
__device__ __forceinline__ int claim_row(const BatchArgs& a, int V) {
  if (a.claim_list != nullptr) {
    const int i = atomicAdd(a.row_claim, 1);
    return (i < *a.claim_count) ? a.claim_list[i] : a.rows;
  }
  int r;
  while ((r = atomicAdd(a.row_claim, 1)) < a.rows) {
    int64_t kk;
    if (row_mode(a.params[r], V, &kk) == kModeFull) break;
  }
  return r;
}

// A row whose penalty window and bias list hold more distinct ids than the
// shared patch table: the patched row is written whole to `out` (the CTA's
// TT slot, unused until the scans), the window counted in `cnt` and each
// bias entry marked in `bmark` (its index in the list + 1), both dense over
// the vocabulary (the KY and SK slots, unused until the transform).
// Block-wide; returns false (block-uniform) on a duplicate bias id.
__device__ bool dense_patch_row(const BatchArgs& a, int row, const nls_row_params& p,
                                const float* rowp, int V, int* cnt, int* bmark, float* out,
                                int* s_dup) {
  const int tid = threadIdx.x;
  int64_t h0, h1, b0, b1;
  patch_lists(a, row, p, &h0, &h1, &b0, &b1);
  const int64_t nh = h1 - h0, ntot = nh + (b1 - b0);
  for (int i = tid; i < V; i += FT_THREADS) {
    cnt[i] = 0;
    bmark[i] = 0;
    out[i] = __ldcs(rowp + i);
  }
  if (tid == 0) *s_dup = 0;
  __syncthreads();
  for (int64_t j = tid; j < ntot; j += FT_THREADS) {
    if (j < nh) {
      const int64_t t = a.hist_ids[h0 + j];
      if (t >= 0 && t < V) atomicAdd(&cnt[t], 1);
    } else {
      const int64_t t = a.bias_ids[b0 + (j - nh)];
      if (t >= 0 && t < V && atomicExch(&bmark[t], (int)(j - nh) + 1) != 0) atomicExch(s_dup, 1);
    }
  }
  __syncthreads();
  if (*s_dup) return false;
  // each listed id gets its patched logit (an id listed twice writes the same
  // value twice)
  for (int64_t j = tid; j < ntot; j += FT_THREADS) {
    const int64_t t = (j < nh) ? a.hist_ids[h0 + j] : a.bias_ids[b0 + (j - nh)];
    if (t < 0 || t >= V) continue;
    const int m = bmark[t];
    const float b = m ? __double2float_rn(a.bias_vals[b0 + (m - 1)]) : 0.0f;  // b.float32 (:76)
    out[t] = penalise(rowp[t], cnt[t], m != 0, b, p);
  }
  __syncthreads();
  return true;
}

// PAIR: launched as clusters of two CTAs (row-claiming launches of batches
// larger than the GPU). The pair shares the first phase of the first row it
// claims -- transform, histogram and scatter, each CTA taking one half of the
// row in CTA 0's scratch slot, the extremes and bucket counts pushed into the
// partner's shared memory before each cluster barrier -- then CTA 0 finishes
// that row and each CTA claims further rows alone; CTA 1's SM is free early
// for the streaming kernel. Without PAIR none of this is compiled.
template <bool PAIR>
__global__ void __launch_bounds__(FT_THREADS, 1)
full_kernel(BatchArgs a, uint32_t* scratch, int vpad) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FullShared& S = *reinterpret_cast<FullShared*>(smem_raw);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem_raw + ((sizeof(FullShared) + 15) & ~(size_t)15));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int V = a.V;
  uint32_t* KY = scratch + (size_t)blockIdx.x * 4 * (size_t)vpad;
  unsigned long long* SK = reinterpret_cast<unsigned long long*>(KY + vpad);
  float* TT = reinterpret_cast<float*>(KY + 3 * (size_t)vpad);
  // LSD fallback: two key arrays in the SK region
  uint32_t* LA = KY + vpad;
  uint32_t* LB = KY + 2 * (size_t)vpad;
  const bool claim = (a.row_claim != nullptr);
  namespace cg = cooperative_groups;
  bool pair = PAIR && claim && cg::this_cluster().num_blocks() == 2;
  // this CTA's rank in the pair and the partner's shared memory, read where
  // used (no register held across a row)
  auto crank_now = []() { return (int)cg::this_cluster().block_rank(); };
  auto partner = [&]() { return cg::this_cluster().map_shared_rank(&S, crank_now() ^ 1); };
  auto cluster_sync = []() { cg::this_cluster().sync(); };
  // Launched as a programmatic dependent of the streaming kernel (small
  // batches): wait until that grid has finished and its writes (the hand-back
  // list) are visible. Without such a launch this returns at once.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int nwork = claim ? 0 : *a.full_count;
  int w = blockIdx.x;

  for (;;) {
    int row;
    if (PAIR && pair) {  // CTA 0 claims for both
      if (crank_now() == 0 && tid == 0) {
        const int r = claim_row(a, V);
        S.ibuf[0] = r;
        partner()->x_row = r;
      }
      cluster_sync();
      row = (crank_now() == 0) ? S.ibuf[0] : S.x_row;
      if (row >= a.rows) break;
    } else if (claim) {  // next row whose parameters select the full path
      if (tid == 0) S.ibuf[0] = claim_row(a, V);
      __syncthreads();
      row = S.ibuf[0];
      __syncthreads();
      if (row >= a.rows) break;
    } else {
      if (w >= nwork) break;
      row = a.full_list[w];
      w += gridDim.x;
    }
    const nls_row_params p = a.params[row];
    int64_t K64;
    const int mode = row_mode(p, V, &K64);
    const bool greedy = (mode == kModeGreedy);
    // the pair's CTA 1 writes no results
    const bool lead = !PAIR || !pair || crank_now() == 0;
    if (!greedy && a.uniforms == nullptr) {
      if (tid == 0 && lead) { a.out_ids[row] = -1; record_status(a.status, NLS_ERR_INVALID_ARG); }
      if (PAIR) pair = false;  // (both CTAs alike: no more cluster barriers)
      continue;
    }
    // heap path iff k < V (sampler.nim:86)
    const bool heap = (K64 < V);
    const int ncand = heap ? (int)K64 : V;
    const float* rowp = a.logits + (int64_t)row * a.ld;

    PatchTable T{S.ph.pt.hkey, S.ph.pt.hcnt, S.ph.pt.hbias, S.ph.pt.hflag, bitmap, FT_HASH_LOG2, 0, V, FT_GSHIFT};
    int npatch = build_patches(a, row, p, T, rowp, &S.counter, &S.patch_overflow, &S.dup);
    if (S.patch_overflow && !S.dup) {
      // More distinct ids than the table holds: the row is patched whole in
      // this CTA's TT slot and read from there; CTA 0 of a pair takes the
      // row alone.
      __syncthreads();
      if (PAIR && pair) {
        pair = false;
        if (crank_now() == 1) continue;
      }
      if (dense_patch_row(a, row, p, rowp, V, reinterpret_cast<int*>(KY), reinterpret_cast<int*>(LA),
                          TT, &S.dup)) {
        rowp = TT;
        npatch = 0;
      }
    }
    if (S.dup) {
      if (tid == 0 && lead) {
        a.out_ids[row] = -1;
        record_status(a.status, NLS_ERR_INVALID_ARG);
      }
      __syncthreads();
      if (PAIR) pair = false;
      continue;
    }
    if (npatch > 0) precompute_patches(T, p);
    if (tid == 0) S.nan = 0;
    __syncthreads();
    auto logit = [&](int i) -> float {
      float x = rowp[i];
      if (npatch > 0 && patch_bit(T, i)) {
        const int slot = patch_find(T, i);
        if (slot >= 0) x = patched_value(T, slot);
      }
      return x;
    };

    if (greedy) {
      // argmax over the patched row (sampler.nim:45-49, 77-78)
      float gb = 0.0f;
      int gi = INT_MAX;
      for (int i = tid; i < V; i += FT_THREADS) {
        const float x = logit(i);
        if (i == 0 && x != x) S.nan = 1;
        if (!(x != x) && (gi == INT_MAX || x > gb)) { gb = x; gi = i; }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        float ob = __shfl_down_sync(0xffffffffu, gb, off);
        int oi = __shfl_down_sync(0xffffffffu, gi, off);
        if (oi != INT_MAX && (gi == INT_MAX || ob > gb || (ob == gb && oi < gi))) { gb = ob; gi = oi; }
      }
      if (lane == 0) { S.fred[warp] = gb; S.ired[warp] = gi; }
      __syncthreads();
      if (tid == 0) {
        float b = 0.0f;
        int bi = INT_MAX;
        for (int k = 0; k < FT_WARPS; ++k) {
          float ob = S.fred[k];
          int oi = S.ired[k];
          if (oi != INT_MAX && (bi == INT_MAX || ob > b || (ob == b && oi < bi))) { b = ob; bi = oi; }
        }
        a.out_ids[row] = S.nan ? 0 : (bi == INT_MAX ? 0 : bi);
        if (a.out_probs) a.out_probs[row] = 1.0f;
      }
      __syncthreads();
      continue;
    }

    // 1. transform: KY[i] = key of y_i; track the extreme keys and NaNs
    const float invT = __double2float_rn(__ddiv_rn(1.0, p.temperature));
    uint32_t kmin = 0xffffffffu, kmax = 0u;
    int anynan = 0;
    const bool vec = ((reinterpret_cast<uintptr_t>(rowp) & 15u) == 0);
    const int nv4 = vec ? (V >> 2) : 0;
    // this CTA's positions [e0, e1) of the first phase (a pair splits the row
    // at a multiple of 4), written to the pair's shared slot (CTA 0's)
    const int half = (PAIR && pair) ? min(V, ((V >> 1) + 3) & ~3) : V;
    const int e0 = (PAIR && pair && crank_now() == 1) ? half : 0;
    const int e1 = (PAIR && pair && crank_now() == 0) ? half : V;
    uint32_t* const KYp = PAIR ? KY - (pair ? (size_t)crank_now() * 4 * (size_t)vpad : 0) : KY;
    unsigned long long* const SKp = PAIR ? reinterpret_cast<unsigned long long*>(KYp + vpad) : SK;
    float* const TTp = PAIR ? reinterpret_cast<float*>(KYp + 3 * (size_t)vpad) : TT;
    auto transform4 = [&](int g, const float4 q) {
      float x[4] = {q.x, q.y, q.z, q.w};
      if (npatch > 0 && patch_bit(T, 4 * g)) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int slot = patch_find(T, 4 * g + e);
          if (slot >= 0) x[e] = patched_value(T, slot);
        }
      }
      uint32_t k[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float y = __fmul_rn(x[e], invT);
        if (y != y) {
          // heap rows: a NaN past the first k positions is never pushed
          // (sampler.nim:91, `x > h[0][0]` is false), exactly like -inf there
          if (heap && 4 * g + e >= ncand) y = -INFINITY;
          else anynan = 1;
        }
        k[e] = desc_key(y);
        kmin = min(kmin, k[e]);
        kmax = max(kmax, k[e]);
      }
      reinterpret_cast<uint4*>(KYp)[g] = make_uint4(k[0], k[1], k[2], k[3]);
    };
    {
      // four loads in flight per thread before any of them is used
      constexpr int TU = 4;
      const float4* src = reinterpret_cast<const float4*>(rowp);
      const int g1 = PAIR ? min(e1 >> 2, nv4) : nv4;
      int g = PAIR ? (e0 >> 2) + tid : tid;
      for (; g + (TU - 1) * FT_THREADS < g1; g += TU * FT_THREADS) {
        float4 q[TU];
#pragma unroll
        for (int u = 0; u < TU; ++u) q[u] = __ldcs(src + g + u * FT_THREADS);
#pragma unroll
        for (int u = 0; u < TU; ++u) transform4(g + u * FT_THREADS, q[u]);
      }
      for (; g < g1; g += FT_THREADS) transform4(g, __ldcs(src + g));
    }
    for (int i = (PAIR ? max(e0, 4 * nv4) : 4 * nv4) + tid; i < e1; i += FT_THREADS) {
      float y = __fmul_rn(logit(i), invT);
      if (y != y) {
        if (heap && i >= ncand) y = -INFINITY;
        else anynan = 1;
      }
      const uint32_t k = desc_key(y);
      kmin = min(kmin, k);
      kmax = max(kmax, k);
      KYp[i] = k;
    }
    kmin = __reduce_min_sync(0xffffffffu, kmin);
    kmax = __reduce_max_sync(0xffffffffu, kmax);
    if (lane == 0) { S.ured[warp] = kmin; S.ured2[warp] = kmax; }
    if constexpr (PAIR) {
      int nnan = block_sum_int(anynan, S);  // (its barrier also publishes ured)
      kmin = 0xffffffffu;
      kmax = 0u;
#pragma unroll 8
      for (int k = 0; k < FT_WARPS; ++k) { kmin = min(kmin, S.ured[k]); kmax = max(kmax, S.ured2[k]); }
      if (pair) {  // the other half's extremes and NaNs (KY complete after the barrier)
        if (tid == 0) {
          partner()->x_kmin = kmin;
          partner()->x_kmax = kmax;
          partner()->x_nan = nnan;
        }
        cluster_sync();
        kmin = min(kmin, S.x_kmin);
        kmax = max(kmax, S.x_kmax);
        nnan += S.x_nan;
      }
      if (nnan > 0) {
        if (heap) {
          if (lead && warp == 0) nan_heap_row(a, row, p, V, ncand, invT, logit, S.u.big, SK);
          __syncthreads();  // warp 0 read the patch table the next row rebuilds
        } else if (tid == 0 && lead) {
          a.out_ids[row] = -1;
          if (a.out_probs) a.out_probs[row] = 0.0f;
          record_status(a.status, NLS_ERR_NAN_LOGITS);
        }
        pair = false;
        continue;
      }
    } else {
      if (block_sum_int(anynan, S) > 0) {   // (its barrier also publishes ured)
        if (heap) {
          if (warp == 0) nan_heap_row(a, row, p, V, ncand, invT, logit, S.u.big, SK);
          __syncthreads();  // warp 0 read the patch table the next row rebuilds
        } else if (tid == 0) {
          a.out_ids[row] = -1;
          if (a.out_probs) a.out_probs[row] = 0.0f;
          record_status(a.status, NLS_ERR_NAN_LOGITS);
        }
        continue;
      }
      kmin = 0xffffffffu;
      kmax = 0u;
#pragma unroll 8
      for (int k = 0; k < FT_WARPS; ++k) { kmin = min(kmin, S.ured[k]); kmax = max(kmax, S.ured2[k]); }
    }
    const float mx = desc_key_value(kmin);
    const float ymin = desc_key_value(kmax);

    // 2. sort into SK: coarse buckets linear in (max - y), scattered through
    //    shared-memory tiles (coalesced runs); then each window of whole
    //    coarse buckets is refined in shared memory into fine buckets of about
    //    one element, finished by insertion sorts on (key, index).
    Bucketer bk;
    bk.mx = mx;
    {
      const float range = __fsub_rn(mx, ymin);  // +inf when ymin is -inf
      const float span = (range < FT_DCAP) ? range : FT_DCAP;
      bk.dcut = (range < FT_DCAP) ? INFINITY : FT_DCAP;
      bk.scale = (span > 0.0f && isfinite(mx)) ? (float)(FT_NB - 1) / span : 0.0f;
      if (!isfinite(mx)) bk.dcut = INFINITY;
    }
    // the row's coarse histogram (a pair: the totals of both halves in both
    // CTAs, each holding the other's counts in x_h1)
    auto histogram = [&]() {
      for (int b = tid; b < FT_NB; b += FT_THREADS) S.h1[b] = 0u;
      __syncthreads();
      {
        // this CTA's positions [e0, e1); e0 is a multiple of 4, KY 16-byte aligned
        const int gk1 = PAIR ? e1 >> 2 : V >> 2;
        for (int g = (PAIR ? (e0 >> 2) : 0) + tid; g < gk1; g += FT_THREADS) {
          const uint4 k = reinterpret_cast<const uint4*>(KYp)[g];
          atomicAdd(&S.h1[bk(k.x)], 1u);
          atomicAdd(&S.h1[bk(k.y)], 1u);
          atomicAdd(&S.h1[bk(k.z)], 1u);
          atomicAdd(&S.h1[bk(k.w)], 1u);
        }
        for (int i = (PAIR ? max(e0, 4 * gk1) : 4 * gk1) + tid; i < e1; i += FT_THREADS) atomicAdd(&S.h1[bk(KYp[i])], 1u);
      }
      __syncthreads();
      if constexpr (PAIR) {
        if (pair) {  // totals; CTA 1 writes each bucket's run after CTA 0's
          for (int b = tid; b < FT_NB; b += FT_THREADS) partner()->x_h1[b] = S.h1[b];
          cluster_sync();
          for (int b = tid; b < FT_NB; b += FT_THREADS) S.h1[b] += S.x_h1[b];
          __syncthreads();
        }
      }
    };
    histogram();
    {
      // A few far outliers -- a banned token (-inf bias), a heavy tail --
      // stretch the value-linear buckets until the bulk of the row shares a
      // few of them, more than a window holds. Then the span is narrowed to
      // leave at most FT_BUCKET_MAX logits beyond it (they share the last
      // bucket, which a window sorts as one block) and the row is counted
      // again; only repeated values still take the radix-sort fallback.
      int bm = 0;
      for (int b = tid; b < FT_NB; b += FT_THREADS) bm = max(bm, (int)S.h1[b]);
      bm = block_max_int(bm, S);  // (its barriers order the reads of h1 below)
      if (bm > FT_BUCKET_MAX && isfinite(mx) && bk.scale > 0.0f) {
        if (warp == 0) {
          // the smallest b* whose suffix sum_{b >= b*} h1[b] is at most
          // FT_BUCKET_MAX (lane l holds buckets 8l .. 8l+7)
          uint32_t loc[FT_NB / 32], sum = 0;
#pragma unroll
          for (int r = 0; r < FT_NB / 32; ++r) { loc[r] = S.h1[lane * (FT_NB / 32) + r]; sum += loc[r]; }
          uint32_t suf = sum;  // inclusive suffix over lanes >= this one
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_down_sync(0xffffffffu, suf, o);
            if (lane + o < 32) suf += v;
          }
          uint32_t after = suf - sum;  // buckets of the lanes above
          int bs = FT_NB;
#pragma unroll
          for (int r = FT_NB / 32 - 1; r >= 0; --r) {
            after += loc[r];
            if (after <= (uint32_t)FT_BUCKET_MAX) bs = lane * (FT_NB / 32) + r;
          }
          bs = __reduce_min_sync(0xffffffffu, bs);
          if (lane == 0) S.ibuf[4] = bs;
        }
        __syncthreads();
        const int bstar = S.ibuf[4];
        __syncthreads();
        if (bstar >= 2 && bstar < FT_NB) {
          const float D = __fdiv_rn((float)bstar, bk.scale);  // d at bucket b*'s lower edge
          if (D > 0.0f) {
            bk.dcut = D;
            bk.scale = (float)(FT_NB - 1) / D;
            histogram();
          }
        }
      }
    }
    if (warp == 0) {  // exclusive scan of the 256 coarse counts (8 per lane)
      uint32_t loc[FT_NB / 32], sum = 0;
#pragma unroll
      for (int r = 0; r < FT_NB / 32; ++r) { loc[r] = S.h1[lane * (FT_NB / 32) + r]; sum += loc[r]; }
      uint32_t incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      uint32_t run = incl - sum;
#pragma unroll
      for (int r = 0; r < FT_NB / 32; ++r) {
        const int b = lane * (FT_NB / 32) + r;
        S.s1[b] = run;
        S.c1[b] = run + ((PAIR && pair && crank_now() == 1) ? S.x_h1[b] : 0u);
        run += loc[r];
      }
    }
    int bigmax = 0;
    for (int b = tid; b < FT_NB; b += FT_THREADS) bigmax = max(bigmax, (int)S.h1[b]);
    bigmax = block_max_int(bigmax, S);
    const bool bucketed = bigmax <= FT_BUCKET_MAX;
    if constexpr (PAIR) {
      if (pair && !bucketed) {  // CTA 0 radix-sorts the whole (complete) KY alone
        pair = false;
        if (crank_now() == 1) continue;
      }
    }
    const int nwin = (V + FT_WIN - 1) / FT_WIN;
    unsigned long long* bufA = S.u.big;
    unsigned long long* bufB = S.ph.bufB;
    // the sorted window under replay: exact t per position, in shared memory
    float* tcache = reinterpret_cast<float*>(S.u.big);
    auto texp_key = [&](uint32_t kdv) { return ref_expf(__fsub_rn(desc_key_value(kdv), mx)); };
    // Sort window c in shared memory: fine buckets of about one element
    // (value-linear inside each coarse bucket), insertion sorts on
    // (key, index), a block sort for the rare large fine bucket; then TT.
    auto sort_window = [&](int c) {
      const int bA = S.wbkt[c], bB = S.wbkt[c + 1], ws = S.wstart[c], we = S.wstart[c + 1];
      const int n = we - ws;
      // a thread may still read the previous window's exact t (u.big, e.g.
      // the absorption check after a replay) while another starts here
      __syncthreads();
      if (n > 1) {
        const int F = FT_NB2 / max(1, bB - bA);  // fine buckets per coarse bucket
        auto fine = [&](uint32_t kdv) {
          const int b = bk(kdv);
          const float d = __fsub_rn(mx, desc_key_value(kdv));
          int sub = F - 1;
          if (d < bk.dcut) {
            const float x = __fmul_rn(d, bk.scale);
            const int f = __float2int_rz(__fmul_rn(__fsub_rn(x, (float)b), (float)F));
            sub = f < 0 ? 0 : (f > F - 1 ? F - 1 : f);
          }
          return (b - bA) * F + sub;
        };
        for (int i = tid; i < FT_NB2; i += FT_THREADS) S.hist2[i] = 0u;
        for (int i = tid; i < n; i += FT_THREADS) bufA[i] = SK[ws + i];
        __syncthreads();
        for (int i = tid; i < n; i += FT_THREADS) atomicAdd(&S.hist2[fine((uint32_t)(bufA[i] >> 32))], 1u);
        __syncthreads();
        {  // exclusive scan of the fine counts (FT_NB2 / FT_THREADS per thread)
          uint32_t cc[FT_NB2 / FT_THREADS];
          int loc = 0;
#pragma unroll
          for (int r = 0; r < FT_NB2 / FT_THREADS; ++r) { cc[r] = S.hist2[tid * (FT_NB2 / FT_THREADS) + r]; loc += (int)cc[r]; }
          int tot;
          int ex = block_excl_sum_int(loc, &tot, S);
#pragma unroll
          for (int r = 0; r < FT_NB2 / FT_THREADS; ++r) {
            S.off2[tid * (FT_NB2 / FT_THREADS) + r] = (uint32_t)ex;
            ex += (int)cc[r];
          }
        }
        if (tid == 0) S.nbig = 0;
        __syncthreads();
        for (int i = tid; i < n; i += FT_THREADS) {
          const unsigned long long v = bufA[i];
          bufB[atomicAdd(&S.off2[fine((uint32_t)(v >> 32))], 1u)] = v;
        }
        __syncthreads();
        // off2[f] is now the end of fine bucket f: insertion-sort the small
        // ones, list the rare large ones for the block sort
        for (int f = tid; f < FT_NB2; f += FT_THREADS) {
          const int m = (int)S.hist2[f];
          if (m <= 1) continue;
          unsigned long long* seg = bufB + (S.off2[f] - (uint32_t)m);
          if (m <= FT_INS_MAX) {
            for (int x = 1; x < m; ++x) {
              const unsigned long long v = seg[x];
              int y = x - 1;
              while (y >= 0 && seg[y] > v) { seg[y + 1] = seg[y]; --y; }
              seg[y + 1] = v;
            }
          } else {
            const int slot = atomicAdd(&S.nbig, 1);
            if (slot < FT_BIGLIST) S.biglist[slot] = f;
          }
        }
        __syncthreads();
        const int nbig = min(S.nbig, FT_BIGLIST);
        const bool all_listed = S.nbig <= FT_BIGLIST;
        for (int q = 0; q < FT_NB2 && q < (all_listed ? nbig : FT_NB2); ++q) {
          const int f = all_listed ? S.biglist[q] : q;
          const int m = (int)S.hist2[f];
          if (m <= FT_INS_MAX) continue;  // (only when scanning every fine bucket)
          unsigned long long* seg = bufB + (S.off2[f] - (uint32_t)m);
          int m64 = 1;
          while (m64 < m) m64 <<= 1;
          for (int i = tid; i < m64; i += FT_THREADS) bufA[i] = i < m ? seg[i] : ~0ull;
          __syncthreads();
          block_bitonic_asc(bufA, m64);
          for (int i = tid; i < m; i += FT_THREADS) seg[i] = bufA[i];
          __syncthreads();
        }
        for (int i = tid; i < n; i += FT_THREADS) {
          const unsigned long long v = bufB[i];
          const float t = texp_key((uint32_t)(v >> 32));
          SK[ws + i] = v;
          TT[ws + i] = t;
          tcache[i] = t;
        }
      } else if (n == 1) {
        if (tid == 0) {
          const float t = texp_key((uint32_t)(SK[ws] >> 32));
          TT[ws] = t;
          tcache[0] = t;
        }
      }
      if (tid == 0) {
        S.wstate[c] = 2;
        S.cwin = c;
      }
      __syncthreads();
    };
    // make window c's exact t values resident in tcache (c sorted)
    auto cache_window = [&](int c) {
      if (S.cwin == c) return;
      const int ws = S.wstart[c], n = S.wstart[c + 1] - ws;
      __syncthreads();
      for (int i = tid; i < n; i += FT_THREADS) tcache[i] = TT[ws + i];
      if (tid == 0) S.cwin = c;
      __syncthreads();
    };
    // window holding SK position j (the same in every thread)
    auto window_of = [&](int j) {
      int lo = 0, hi = nwin - 1;  // last c with wstart[c] <= j
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (S.wstart[mid] <= j) lo = mid; else hi = mid - 1;
      }
      return lo;
    };
    auto ensure_sorted = [&](int j) {
      const int c = window_of(j);
      if (S.wstate[c] != 2) sort_window(c);
    };
    if (bucketed) {
      // coarse scatter, one tile at a time: counting sort of the tile in
      // shared memory, then each bucket's run goes out contiguously
      unsigned long long* stage = S.u.big;
      constexpr int PT = FT_TILE1 / FT_THREADS;
      for (int b = tid; b < FT_NB; b += FT_THREADS) S.lc[b] = 0u;
      uint32_t kd[PT];  // this tile's keys, loaded one tile ahead
#pragma unroll
      for (int r = 0; r < PT; ++r) {
        const int i = e0 + tid + r * FT_THREADS;
        kd[r] = (i < e1) ? KYp[i] : 0u;
      }
      __syncthreads();
      for (int t0 = e0; t0 < e1; t0 += FT_TILE1) {
        const int nt = min(FT_TILE1, e1 - t0);
        int bb[PT];
        uint32_t rk[PT];  // rank inside the tile's bucket
#pragma unroll
        for (int r = 0; r < PT; ++r) {
          const int i = tid + r * FT_THREADS;
          bb[r] = (i < nt) ? bk(kd[r]) : -1;
          rk[r] = (bb[r] >= 0) ? atomicAdd(&S.lc[bb[r]], 1u) : 0u;
        }
        __syncthreads();
        if (warp == 0) {
          uint32_t loc[FT_NB / 32], sum = 0;
#pragma unroll
          for (int r = 0; r < FT_NB / 32; ++r) { loc[r] = S.lc[lane * (FT_NB / 32) + r]; sum += loc[r]; }
          uint32_t incl = sum;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
          }
          uint32_t run = incl - sum;
#pragma unroll
          for (int r = 0; r < FT_NB / 32; ++r) {
            const int b = lane * (FT_NB / 32) + r;
            S.lo1[b] = run;       // the bucket's run inside the staged tile
            S.gb1[b] = S.c1[b];   // and its destination in SK
            S.c1[b] += loc[r];
            S.lc[b] = 0u;
            run += loc[r];
          }
        }
        __syncthreads();
#pragma unroll
        for (int r = 0; r < PT; ++r) {
          if (bb[r] >= 0)
            stage[S.lo1[bb[r]] + rk[r]] = ((unsigned long long)kd[r] << 32) | (uint32_t)(t0 + tid + r * FT_THREADS);
        }
#pragma unroll
        for (int r = 0; r < PT; ++r) {
          const int i = t0 + FT_TILE1 + tid + r * FT_THREADS;
          kd[r] = (i < e1) ? KYp[i] : 0u;
        }
        __syncthreads();
        // (the next tile touches lo1/gb1/stage only after its first barrier)
        for (int q = tid; q < nt; q += FT_THREADS) {
          const unsigned long long v = stage[q];
          const uint32_t kdv = (uint32_t)(v >> 32);
          const int b = bk(kdv);
          const uint32_t j = S.gb1[b] + ((uint32_t)q - S.lo1[b]);
          SKp[j] = v;
          TTp[j] = __fsub_rn(desc_key_value(kdv), mx);  // x = y - max, for the passes
        }
      }
      __syncthreads();
      if constexpr (PAIR) {
        if (pair) {  // every SK entry of the row is written; CTA 1 moves on
          cluster_sync();
          pair = false;
          if (crank_now() == 1) continue;
        }
      }
      // windows: the coarse buckets whose start lies in [c*FT_WIN, (c+1)*FT_WIN)
      for (int c = tid; c <= nwin; c += FT_THREADS) {
        const int x = c * FT_WIN;
        int lo = 0, hi = FT_NB;  // first bucket starting at or after x
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if ((int)S.s1[mid] >= x) hi = mid; else lo = mid + 1;
        }
        S.wbkt[c] = lo;
        S.wstart[c] = (c == nwin || lo >= FT_NB) ? V : (int)S.s1[lo];
        if (c < nwin) S.wstate[c] = 0;
      }
      if (tid == 0) S.cwin = -1;  // u.big held the scatter stage
    } else {
      // repeated values overflow one bucket: LSD radix sort of the keys
      lsd_count(KY, V, 0, S);
      lsd_scatter(KY, LA, V, 0, S);
      lsd_count(LA, V, 8, S);
      lsd_scatter(LA, LB, V, 8, S);
      lsd_count(LB, V, 16, S);
      lsd_scatter(LB, LA, V, 16, S);
      lsd_count(LA, V, 24, S);
      lsd_scatter(LA, LB, V, 24, S);
    }
    __syncthreads();
    // sorted key of candidate position j
    auto skey = [&](int j) -> uint32_t { return bucketed ? (uint32_t)(SK[j] >> 32) : LB[j]; };

    const double u_draw = a.uniforms[row];
    int pos;
    float prob;
    if (!isfinite(mx)) {
      // Non-finite maximum: the reference's arithmetic produces NaNs that a
      // grid replay cannot represent; run its loops literally (one thread).
      if (bucketed)
        for (int c = 0; c < nwin; ++c)
          if (S.wstate[c] != 2) sort_window(c);
      if (tid == 0) {
        float m = -INFINITY;
        for (int j = 0; j < ncand; ++j) {
          float y = desc_key_value(skey(j));
          m = (m <= y) ? y : m;
        }
        float ss = 0.0f;
        for (int j = 0; j < ncand; ++j) {
          float tj = ref_expf(__fsub_rn(desc_key_value(skey(j)), m));
          TT[j] = tj;
          ss = __fadd_rn(ss, tj);
        }
        for (int j = 0; j < ncand; ++j) TT[j] = __fdiv_rn(TT[j], ss);
        int n = ncand;
        if (p.top_p > 0.0 && p.top_p < 1.0) {
          float cum = 0.0f;
          for (int j = 0; j < n; ++j) {
            cum = __fadd_rn(cum, TT[j]);
            if ((double)cum >= p.top_p) { n = j + 1; break; }
          }
        }
        if (p.min_p > 0.0) {
          const float thr = __fmul_rn(TT[0], __double2float_rn(p.min_p));
          int m2 = 1;
          while (m2 < n && TT[m2] >= thr) ++m2;
          n = m2;
        }
        float total = 0.0f;
        for (int j = 0; j < n; ++j) total = __fadd_rn(total, TT[j]);
        float r = __fmul_rn(__double2float_rn(u_draw), total);
        int ps = n - 1;
        for (int j = 0; j < n; ++j) {
          r = __fsub_rn(r, TT[j]);
          if (r <= 0.0f) { ps = j; break; }
        }
        S.ibuf[1] = ps;
        S.fbuf[1] = TT[ps];
      }
      __syncthreads();
      pos = S.ibuf[1];
      prob = S.fbuf[1];
      __syncthreads();
    } else {
      // 3. t_j = expf(y_j - max) in candidate order (TT), then the three
      //    sequential sums of the reference replayed exactly.
      int tt_valid = 0;  // LSD path: TT holds [0, tt_valid); the same in every thread
      auto texp = [&](int j) { return texp_key(skey(j)); };
      auto prep = [&](int j0, int j1) {
        if (j1 > tt_valid) {
          for (int j = max(j0, tt_valid) + tid; j < j1; j += FT_THREADS) TT[j] = texp(j);
          tt_valid = j1;
          __syncthreads();
        }
      };
      auto nostop = [](float) { return false; };
      // One sequential fp32 accumulation over candidate positions [0, j1)
      // whose j-th term is fromt(t_j). Bucketed path: a window whose
      // elements leave the running value in its binade with no rounding tie
      // and no stop contributes an order-independent integer sum, so it is
      // summed in bucket order without sorting; any other window (and one
      // cut by j1) is sorted first and replayed in order.
      // Exact replay of positions [j0, j1) of one sorted window (terms from
      // shared memory): every warp sums the grid units of 32-position groups,
      // warp 0 finds the first group where a tie, a binade change or the stop
      // happens, everything before it is taken at once, and one warp replays
      // from that group; then again with the new grid.
      // the set of group sums the next replay iteration writes (alternating
      // across all the row's replays)
      int rset = 0;
      auto window_replay = [&](auto decc, int j0, int j1, float v0, auto elem, auto stop,
                               bool has_stop, bool absorb) -> ScanResult {
        constexpr bool DEC = decltype(decc)::value;
        float v = v0;
        int j = j0;
        // Positions summed per pass. The terms do not grow along the sorted
        // order, so the running value cannot leave its binade within
        // (distance to the binade edge) / elem(j) positions. While that bound
        // is under one group per warp, a pass takes one group per warp
        // (binade changes near a sum's start come 1, 2, 4, ... positions
        // apart); beyond it, FT_BIG positions at once (a pass costs mostly its
        // barriers). Doubled while passes find no event.
        auto first_span = [&](int jj, float vv) -> int {
          const float tj = elem(jj);
          const int E = binade_exp(vv);
          // (exact: v and the binade's edge are within a factor of two)
          const float edge = (E >= -126) ? __int_as_float((E + 127 + (DEC ? 0 : 1)) << 23) : 0.0f;
          const float room = DEC ? __fsub_rn(vv, edge) : __fsub_rn(edge, vv);
          return (tj > 0.0f && room < tj * (float)(32 * FT_WARPS)) ? 32 * FT_WARPS : FT_BIG;
        };
        int span = first_span(j, v);
        while (j < j1) {
          const int E = binade_exp(v);
          const int ue = E - 23;
          if (!DEC && absorb && elem(j) < half_grid(ue)) break;
          long long S0 = grid_S(v);
          if (DEC) S0 = -S0;
          const int jend = (j1 - j > span) ? j + span : j1;
          const int ng = (jend - j + 31) >> 5;  // <= FT_BIG / 32
          // (set `rset` of the group sums and of the results below: the
          // next iteration writes the other set, so readers need no second
          // barrier)
          uint32_t* const gsum = S.gsum[rset];
          int* const gtie = S.gtie[rset];
          ReplayShared& rs = S.rpl[rset];
          rset ^= 1;
          for (int g = warp; g < ng; g += FT_WARPS) {
            const int jj = j + 32 * g + lane;
            long long u = 0;
            bool tie = false;
            if (jj < jend) u = grid_units(elem(jj), ue, &tie);
            // units clamped at 2^25: such an element leaves the binade by
            // itself, so the first event and the sums before it are exact
            const uint32_t gs = __reduce_add_sync(0xffffffffu, (uint32_t)min(u, 1LL << 25));
            const bool gt = __any_sync(0xffffffffu, tie);
            if (lane == 0) {
              gsum[g] = gs;
              gtie[g] = gt;
            }
          }
          __syncthreads();
          // warp 0: the first group holding a tie, a binade change or the
          // stop (lane l scans groups l*per .. l*per+per-1)
          if (warp == 0) {
            const int per = (ng + 31) >> 5;  // groups per lane, <= 8
            long long loc = 0;
            for (int r = 0; r < per; ++r) {
              const int g = lane * per + r;
              if (g < ng) loc += gsum[g];
            }
            long long incl = loc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const long long y = __shfl_up_sync(0xffffffffu, incl, o);
              if (lane >= o) incl += y;
            }
            long long run = S0 + incl - loc;  // value before this lane's first group
            int ev = INT_MAX;
            long long sb = 0;
            for (int r = 0; r < per; ++r) {
              const int g = lane * per + r;
              if (g >= ng) break;
              const long long after = run + gsum[g];
              bool e = gtie[g] != 0;
              if (!e) {
                if (!DEC) e = after >= (1LL << 24);
                else e = (E == -126) ? (after >= 0) : (after >= -(1LL << 23));
              }
              if (!e && has_stop) e = stop(grid_value(DEC ? -after : after, ue));
              if (e) {
                ev = g;
                sb = run;
                break;
              }
              run = after;
            }
            const unsigned eb = __ballot_sync(0xffffffffu, ev != INT_MAX);
            int gev = -1;
            long long gS = S0 + __shfl_sync(0xffffffffu, incl, 31);
            if (eb) {
              const int L = __ffs(eb) - 1;
              gev = __shfl_sync(0xffffffffu, ev, L);
              gS = __shfl_sync(0xffffffffu, sb, L);
            }
            float wv = grid_value(DEC ? -gS : gS, ue);
            int wj = jend, wstop = -1;
            if (gev >= 0) {  // replay from that group, one warp
              const WalkResult w = warp_walk<DEC>(j + 32 * gev, j1, wv, elem, stop, has_stop, 8);
              wv = w.v;
              wj = w.j;
              wstop = w.stop_j;
            }
            if (lane == 0) {
              rs.v = wv;
              rs.j = wj;
              rs.stop = wstop;
              rs.event = gev >= 0;
            }
          }
          __syncthreads();
          v = rs.v;
          j = rs.j;
          if (rs.stop >= 0) return ScanResult{v, rs.stop};
          if (!rs.event) {  // no event in the span: taken in one step
            span = (span < FT_BIG) ? span * 2 : span;
            continue;
          }
          if (j < j1) span = first_span(j, v);
        }
        return ScanResult{v, -1};
      };
      // the set of pass partials the next order-independent pass writes
      // (alternating across all the row's scans)
      int pset = 0;
      auto run_scan = [&](auto decc, int j1, float v0, auto fromt, auto stop, bool has_stop,
                          bool absorb) -> ScanResult {
        constexpr bool DEC = decltype(decc)::value;
        auto elem = [&](int j) { return fromt.exact(TT[j]); };
        if (!bucketed)
          return exact_scan_fast<FT_THREADS, FT_EPT, DEC>(0, j1, v0, elem, stop, has_stop, absorb,
                                                          S.scan, S.fscan, prep);
        float v = v0;
        constexpr int WPT = FT_BIG / FT_THREADS;  // a pass covers at most FT_BIG positions
        // The last window the order-independent pass settled: its grid, grid
        // units and size predict whether the next two windows fit one pass.
        int last_ue = INT_MIN, last_n = 1;
        long long last_units = 0;
        int alone = -1;  // a window whose two-window pass failed: taken alone
        for (int c = 0; c < nwin; ++c) {
          const int ws = S.wstart[c];
          if (ws >= j1) break;
          const int we0 = S.wstart[c + 1];
          if (we0 <= ws) continue;
          const int we = min(we0, j1);
          const int st = S.wstate[c];
          if (st != 2 && we == we0) {
            // Order-independent pass. An element's grid units follow from the
            // estimate texp_estimate(x) of its term (x from TT) unless a
            // rounding boundary lies within the estimate's error; then
            // ref_expf is evaluated.
            // v's binade, its grid 2^ue and v on that grid (from v's bits:
            // the significand with its hidden bit; denormals share E = -126)
            const uint32_t vb = __float_as_uint(v) & 0x7fffffffu;
            const int E = binade_exp(v);
            const int ue = E - 23;
            long long S0 = (vb >> 23) ? (long long)((vb & 0x7fffffu) | 0x800000u) : (long long)vb;
            if (DEC) S0 = -S0;
            // a grid value S * 2^ue as a float (|S| <= 2^24: exact)
            const float gunit = (ue >= -126) ? __int_as_float((ue + 127) << 23) : __int_as_float(1 << (ue + 149));
            auto gval = [&](long long Sv) { return __fmul_rn((float)(DEC ? -Sv : Sv), gunit); };
            // Windows c and c+1 in one pass when the last settled window, on
            // this grid, predicts (terms do not grow along the sorted order)
            // that the running value stays inside its binade and short of the
            // stop over both. A wrong guess costs one pass: window c is then
            // taken alone. Either way the checks below decide.
            int wend = we;
            if (c != alone && last_ue == ue && c + 1 < nwin && S.wstate[c + 1] != 2) {
              const int we2 = S.wstart[c + 2];
              if (we2 > we && we2 <= j1 && we2 - ws <= FT_BIG) {
                const float pred = 1.25f * (float)last_units * (float)(we2 - ws) / (float)last_n;
                const float sp = (float)S0 + pred;
                bool two = !DEC ? sp < 0x1p24f : (E != -126 && sp < -0x1p23f);
                if (two && has_stop) two = !stop(gval((long long)sp));
                if (two) wend = we2;
              }
            }
            // grid 2^ue as a float scale (when representable)
            const bool scale_ok = (ue >= -120 && ue <= 126);  // terms near a grid step stay normal
            const float gscale = scale_ok ? __int_as_float((127 - ue) << 23) : 0.0f;
            const int rounds = (wend - ws + FT_THREADS - 1) / FT_THREADS;  // same in every thread
            float xv[WPT];  // x = y - max per position, all loads first: one memory latency per pass
#pragma unroll
            for (int r = 0; r < WPT; ++r) {
              const int j = ws + tid + r * FT_THREADS;
              xv[r] = (j < wend) ? TT[j] : 0.0f;
            }
            // the next pass most likely starts at wend: its estimates into L1
#pragma unroll
            for (int r = 0; r < WPT; ++r) {
              const int j = wend + tid + r * FT_THREADS;
              if (j < j1) asm volatile("prefetch.global.L1 [%0];" ::"l"(TT + j));
            }
            float sumf = 0.0f;  // settled units, each < 2^18: at most 2^21, exact in fp32
            uint32_t usum = 0u;  // units of the elements redone exactly (saturated)
            bool tie = false;
            float amax = 0.0f;
            unsigned pending = 0u;  // elements the estimate does not settle
            // q = term / grid; the exact term lies within q * margin / 2 of q,
            // so if no half-integer is that close, rne(q) is its grid value
            // and it is no tie. Straight-line code: the unrolled elements
            // overlap; the rare unsettled ones are redone exactly below.
#pragma unroll
            for (int r = 0; r < WPT; ++r) {
              if (r >= rounds) break;
              const bool valid = ws + tid + r * FT_THREADS < wend;
              const float a = texp_estimate(xv[r]);
              const float emid = fromt.mid(a);
              const float q = __fmul_rn(emid, gscale);
              const float k = rintf(q);
              const float f = fabsf(__fsub_rn(q, k));
              const bool ok = (a >= kBracketMin) && scale_ok && (__fsub_rn(0.5f, f) > __fmul_rn(q, fromt.margin));
              sumf = __fadd_rn(sumf, (valid && ok) ? k : 0.0f);
              amax = fmaxf(amax, valid ? emid : 0.0f);
              pending |= (valid && !ok) ? (1u << r) : 0u;
            }
#pragma unroll
            for (int r = 0; r < WPT; ++r) {
              if (!(pending & (1u << r))) continue;
              const float e = fromt.exact(ref_expf(xv[r]));
              bool tj;
              const long long gu = grid_units(e, ue, &tj);
              usum = min(usum + (uint32_t)min(gu, 1LL << 24), 1u << 24);
              tie |= tj;
              amax = fmaxf(amax, e);
            }
            // Sums saturate at 2^24 units: a pass that reaches them leaves the
            // binade anyway (|S0| < 2^24 on the same side), so the checks
            // below still fail it; below that every sum is exact in 32 bits
            // (32 x 2^24 < 2^32).
            usum = min(usum + (uint32_t)sumf, 1u << 24);
            const uint32_t wsum = min(__reduce_add_sync(0xffffffffu, usum), 1u << 24);
            const uint32_t wmaxb = __reduce_max_sync(0xffffffffu, __float_as_uint(amax));  // amax >= 0
            const unsigned anytie = __ballot_sync(0xffffffffu, tie);
            // (set `pset` of the partials: the previous pass read the other
            // one, so one barrier per pass suffices)
            uint32_t(*const pp)[FT_WARPS] = S.pp[pset];
            pset ^= 1;
            if (lane == 0) { pp[0][warp] = wsum; pp[1][warp] = wmaxb; pp[2][warp] = anytie != 0u; }
            __syncthreads();
            const long long tot = (long long)__reduce_add_sync(0xffffffffu, pp[0][lane]);
            const float wmax = __uint_as_float(__reduce_max_sync(0xffffffffu, pp[1][lane]));
            const int any = __any_sync(0xffffffffu, pp[2][lane] != 0u);
            // every later term is at most this pass's largest
            // (wmax estimates the largest term within 2^-18; 2^-12 covers it;
            // half a grid step below the float range reads 0: no early end)
            if (!DEC && absorb && __fmul_rn(wmax, 1.0f + 0x1p-12f) < __fmul_rn(gunit, 0.5f))
              return ScanResult{v, -1};
            const long long Se = S0 + tot;
            bool fast = !any;
            if (fast) {
              if (!DEC) fast = Se < (1LL << 24);
              else fast = (E == -126) ? (Se < 0) : (Se < -(1LL << 23));
            }
            if (fast && has_stop) fast = !stop(gval(Se));
            if (fast) {
              v = gval(Se);
              last_ue = ue;  // v stayed in its binade
              last_units = tot;
              last_n = wend - ws;
              if (wend != we) ++c;  // window c+1 was in the pass too
              continue;
            }
            if (wend != we) {  // take window c alone
              alone = c;
              --c;
              continue;
            }
          }
          last_ue = INT_MIN;
          if (S.wstate[c] != 2) sort_window(c);
          else cache_window(c);
          auto elemc = [&](int j) { return fromt.exact(tcache[j - ws]); };
          const ScanResult r = window_replay(decc, ws, we, v, elemc, stop, has_stop, absorb);
          if (r.stop_j >= 0) return r;
          v = r.v;
          if (!DEC && absorb && elemc(we - 1) < half_grid(binade_exp(v) - 23))
            return ScanResult{v, -1};
        }
        return ScanResult{v, -1};
      };
      using inc_t = std::integral_constant<bool, false>;
      using dec_t = std::integral_constant<bool, true>;
      if (bucketed && heap) ensure_sorted(ncand - 1);
      // softmax denominator (sampler.nim:54-56)
      const float s = run_scan(inc_t{}, ncand, 0.0f, TermT{}, nostop, false, true).v;
      const TermP pfrom{s, __frcp_rn(s)};
      // min-p first cut (sampler.nim:110-113): first j >= 1 with p_j < thr.
      // p is a non-increasing function of the candidate's key, so the kept
      // prefix is {key <= K*} for the largest key K* with p(K*) >= thr.
      int nlim = ncand;
      if (p.min_p > 0.0) {
        if (!bucketed) {
          auto pval_any = [&](int j) { return __fdiv_rn(j < tt_valid ? TT[j] : texp(j), s); };
          if (tid == 0) {
            const float thr = __fmul_rn(pval_any(0), __double2float_rn(p.min_p));
            int lo = 1, hi = ncand;
            while (lo < hi) {
              const int mid = (lo + hi) >> 1;
              if (pval_any(mid) < thr) hi = mid; else lo = mid + 1;
            }
            S.ibuf[2] = lo;
          }
          __syncthreads();
          nlim = S.ibuf[2];
          __syncthreads();
        } else {
          // t of the maximum is expf(0) = 1
          const float thr = __fmul_rn(__fdiv_rn(1.0f, s), __double2float_rn(p.min_p));
          auto pk = [&](uint32_t kdv) { return __fdiv_rn(texp_key(kdv), s); };
          if (tid == 0) {
            uint32_t lo = kmin, hi = kmax;  // pk(lo) >= thr unless min_p > 1
            if (!(pk(lo) >= thr)) {
              S.ibuf[2] = -1;
            } else {
              while (lo < hi) {  // largest key with pk >= thr
                const uint32_t mid = lo + (uint32_t)((hi - lo + 1u) >> 1);
                if (pk(mid) >= thr) lo = mid; else hi = mid - 1u;
              }
              S.ibuf[2] = bk(lo);
              S.ibuf[3] = (int)lo;
            }
          }
          __syncthreads();
          const int bs = S.ibuf[2];
          const uint32_t kstar = (uint32_t)S.ibuf[3];
          __syncthreads();
          if (bs < 0) {
            nlim = 1;
          } else {
            // buckets before bs hold keys <= K*, buckets after it keys > K*
            const int b0 = (int)S.s1[bs], b1 = b0 + (int)S.h1[bs];
            int cnt = 0;
            for (int j = b0 + tid; j < b1; j += FT_THREADS) cnt += (uint32_t)(SK[j] >> 32) <= kstar;
            cnt = block_sum_int(cnt, S);
            nlim = max(1, min(ncand, b0 + cnt));
          }
        }
      }
      // top-p (sampler.nim:103-108) and the draw total (:115-116)
      int n;
      float total;
      if (p.top_p > 0.0 && p.top_p < 1.0) {
        const double tp = p.top_p;
        const ScanResult r = run_scan(inc_t{}, nlim, 0.0f, pfrom, [tp](float v) { return (double)v >= tp; },
                                      true, false);
        n = (r.stop_j >= 0) ? r.stop_j + 1 : nlim;
        total = r.v;
      } else {
        n = nlim;
        total = run_scan(inc_t{}, nlim, 0.0f, pfrom, nostop, false, true).v;
      }
      // draw (sampler.nim:117-121)
      const float r0 = __fmul_rn(__double2float_rn(u_draw), total);
      const ScanResult d = run_scan(dec_t{}, n, r0, pfrom, [](float v) { return v <= 0.0f; }, true, false);
      pos = (d.stop_j >= 0) ? d.stop_j : n - 1;
      if (bucketed) {
        ensure_sorted(pos);
      } else if (pos >= tt_valid) {
        if (tid == 0) TT[pos] = texp(pos);
        __syncthreads();
      }
      prob = __fdiv_rn(TT[pos], s);
      __syncthreads();
    }

    // 4. token id of the drawn position
    int id = -1;
    if (bucketed) {
      if (tid == 0) {
        const uint32_t kpos = (uint32_t)(SK[pos] >> 32);
        if (!heap) {
          id = (int)(uint32_t)SK[pos];
        } else {
          // equal keys share a coarse bucket, hence a (sorted) window
          const int c = window_of(pos);
          const int w0 = S.wstart[c], wn = S.wstart[c + 1] - w0;
          const int lb = w0 + lower_bound_key(SK + w0, wn, kpos);
          const int o = pos - lb;
          const uint32_t tkey = (uint32_t)(SK[ncand - 1] >> 32);
          if (kpos != tkey) {
            const int g = w0 + upper_bound_key(SK + w0, wn, kpos) - lb;
            id = (int)(uint32_t)SK[lb + g - 1 - o];  // ties in descending index
          } else {
            id = -2;  // needs tau (below)
          }
        }
        S.ibuf[3] = id;
      }
      __syncthreads();
      id = S.ibuf[3];
      __syncthreads();
      if (id == -2) {
        // the heap keeps the highest-indexed ties <= tau, where tau is the
        // index at which the count of values >= t reaches k
        const uint32_t tkey = (uint32_t)(SK[ncand - 1] >> 32);
        const int tau = block_find_nth(V, ncand - 1, [&](int i) { return KY[i] <= tkey; }, S);
        if (tid == 0) {
          const int c = window_of(ncand - 1);
          const int w0 = S.wstart[c], wn = S.wstart[c + 1] - w0;
          const int lb = w0 + lower_bound_key(SK + w0, wn, tkey);
          const int ub = w0 + upper_bound_key(SK + w0, wn, tkey);
          // ties <= tau form a prefix of the tie group (ascending index)
          int lo2 = lb, hi2 = ub;
          while (lo2 < hi2) {
            const int mid = (lo2 + hi2) >> 1;
            if ((int)(uint32_t)SK[mid] <= tau) lo2 = mid + 1; else hi2 = mid;
          }
          const int o = pos - lb;
          S.ibuf[3] = (int)(uint32_t)SK[lo2 - 1 - o];
        }
        __syncthreads();
        id = S.ibuf[3];
        __syncthreads();
      }
    } else {
      const uint32_t kpos = LB[pos];
      const int lb = lower_bound_u32(LB, V, kpos);
      const int o = pos - lb;
      if (!heap) {
        id = block_find_nth(V, o, [&](int i) { return KY[i] == kpos; }, S);
      } else {
        const uint32_t tkey = LB[ncand - 1];
        if (kpos != tkey) {
          const int g = upper_bound_u32(LB, V, kpos) - lb;
          id = block_find_nth(V, g - 1 - o, [&](int i) { return KY[i] == kpos; }, S);
        } else {
          const int tau = block_find_nth(V, ncand - 1, [&](int i) { return KY[i] <= tkey; }, S);
          const int mt = block_count(tau + 1, [&](int i) { return KY[i] == tkey; }, S);
          id = block_find_nth(tau + 1, mt - 1 - o, [&](int i) { return KY[i] == tkey; }, S);
        }
      }
    }
    if (tid == 0) {
      a.out_ids[row] = id;
      if (a.out_probs) a.out_probs[row] = prob;
    }
    __syncthreads();
  }
}

// The rows whose parameters select the full path, in ascending order, for a
// row-claiming full-sort launch: one block, an ordered compaction of the
// row classification (sampler.nim:77-78, 85-86).
__global__ void __launch_bounds__(1024) classify_full_rows(BatchArgs a, int* list, int* count) {
  __shared__ int wsum[32];
  __shared__ int base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) base = 0;
  __syncthreads();
  for (int r0 = 0; r0 < a.rows; r0 += 1024) {
    const int r = r0 + tid;
    int64_t kk;
    const bool full = r < a.rows && row_mode(a.params[r], a.V, &kk) == kModeFull;
    const unsigned m = __ballot_sync(0xffffffffu, full);
    if (lane == 0) wsum[warp] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < 32; ++w) {
      const int c = wsum[w];
      before += (w < warp) ? c : 0;
      total += c;
    }
    if (full) list[base + before + __popc(m & lanemask_lt())] = r;
    __syncthreads();
    if (tid == 0) base += total;
    __syncthreads();
  }
  if (tid == 0) *count = base;
}

cudaError_t launch_classify(const BatchArgs& a, int* list, int* count, cudaStream_t stream) {
  classify_full_rows<<<1, 1024, 0, stream>>>(a, list, count);
  return cudaGetLastError();
}

static std::atomic<int> g_full_smem_set[kMaxDevicesAttr];
static std::atomic<int> g_full_pair_smem_set[kMaxDevicesAttr];

cudaError_t launch_full(const BatchArgs& a, uint32_t* scratch, int vpad, int slots,
                        cudaStream_t stream, bool after_light) {
  const size_t smem = full_smem_bytes(a.V);
  int grid = (a.rows < slots) ? a.rows : slots;  // a CTA takes at most one row at a time
  // A row-claiming launch runs as cluster pairs (an even grid within the
  // scratch slots, two CTAs per row where the slots allow): a pair shares its
  // first row's first phase, and CTA 1 then claims rows alone or leaves its
  // SM to the concurrent streaming kernel.
  const bool pairs = a.row_claim != nullptr && !after_light && slots >= 2 && a.rows >= 1;
  if (pairs) grid = ((2 * a.rows < slots) ? 2 * a.rows : slots) & ~1;
  const void* fn = pairs ? reinterpret_cast<const void*>(full_kernel<true>)
                         : reinterpret_cast<const void*>(full_kernel<false>);
  cudaError_t e = ensure_smem_attr(fn, (int)smem, pairs ? g_full_pair_smem_set : g_full_smem_set);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(FT_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (pairs) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, full_kernel<true>, a, scratch, vpad);
    if (e == cudaSuccess) return e;
    // no room for a cluster pair right now (another context holds the SMs):
    // the single-CTA kernel over the same grid does the same work
    (void)cudaGetLastError();
    e = ensure_smem_attr(reinterpret_cast<const void*>(full_kernel<false>), (int)smem, g_full_smem_set);
    if (e != cudaSuccess) return e;
    cfg.attrs = nullptr;
    cfg.numAttrs = 0;
    return cudaLaunchKernelEx(&cfg, full_kernel<false>, a, scratch, vpad);
  }
  if (after_light) {
    // may start before the streaming kernel ends (its launch latency hides
    // behind that kernel); griddepcontrol.wait orders the reads
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, full_kernel<false>, a, scratch, vpad);
}

}  // namespace nls
