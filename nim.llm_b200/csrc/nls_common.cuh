// nls_common.cuh -- device helpers shared by the sampler kernels (sm_100a).
//
// Numerics follow src/nimllm/sampler.nim (reference repository) exactly:
// every parity-relevant float op uses an explicit round-to-nearest intrinsic
// (__fadd_rn, __fmul_rn, __fdiv_rn, __dmul_rn, ...) and the library is built
// with -fmad=false, so nothing is contracted into an FMA.
#pragma once

#include <atomic>

#include <cstdint>
#include <cuda_runtime.h>

#include "nimllm_sample.h"

namespace nls {

// Raise a kernel's dynamic shared-memory limit on the current device only
// when a launch needs more than was set before (the attribute call costs
// host time on every launch otherwise). `done` holds, per device, the largest
// value set so far.
constexpr int kMaxDevicesAttr = 64;
inline cudaError_t ensure_smem_attr(const void* fn, int bytes, std::atomic<int>* done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDevicesAttr && done[dev].load(std::memory_order_relaxed) >= bytes)
    return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDevicesAttr) {
    int cur = done[dev].load(std::memory_order_relaxed);
    while (cur < bytes && !done[dev].compare_exchange_weak(cur, bytes)) {
    }
  }
  return cudaSuccess;
}

constexpr int kMaxVocab = 1 << 18;   // token ids fit in 18 bits (composite sort keys)
constexpr int kLightKMax = 256;      // top-k rows with k <= this take the streaming path

enum RowMode : int { kModeGreedy = 0, kModeTopK = 1, kModeFull = 2 };

// Per-call arguments, passed by value to every kernel.
struct BatchArgs {
  const float* logits;
  int64_t ld;
  int rows;
  int V;
  const nls_row_params* params;
  const int64_t* hist_ids;   // may be null
  const int64_t* hist_off;
  const int64_t* bias_ids;   // may be null
  const double* bias_vals;
  const int64_t* bias_off;
  const double* uniforms;    // may be null when every row is greedy
  int64_t* out_ids;
  float* out_probs;          // may be null
  int* full_list;            // rows handed to the full-sort kernel
  int* full_count;
  int* status;               // first error code recorded by any kernel
  int argmax_only;           // nls_argmax_batch: plain argmax, no params
  // Full-sort kernel: when set, it claims the rows whose parameters select
  // the full path through this counter from claim_list[0 .. *claim_count)
  // (written by classify_full_rows), instead of reading full_list (lets it
  // run concurrently with the streaming kernel).
  int* row_claim;
  const int* claim_list;
  const int* claim_count;
  // Streaming kernel: leave full-path rows alone (a concurrent full-sort
  // launch claims them) instead of appending them to full_list.
  int skip_full;
  // Limit of the streaming kernel's waits for its bulk copies (ns; 0 gives
  // up at once). The drain of copies in flight before a CTA exits always
  // waits up to kWaitLimitNs.
  unsigned long long wait_ns;
};

__device__ __forceinline__ void record_status(int* st, int code) { atomicCAS(st, 0, code); }

// Order-preserving map of an fp32 value onto uint32 (ascending key ==
// ascending value). -0.0 maps to the key of +0.0: Nim's cmp and tuple `<`
// treat the two zeros as equal, so they must tie here too.
__device__ __forceinline__ uint32_t fkey(float y) {
  uint32_t u = __float_as_uint(y);
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}
// Float threshold equivalent to "key >= k" for non-NaN values. Keys below the
// key of -Inf decode to negative NaNs; every non-NaN value passes them.
__device__ __forceinline__ float key_threshold_float(uint32_t k) {
  const float f = fkey_inv(k);
  return (f != f) ? -INFINITY : f;
}

// expf as the reference computes it. Nim's exp(float32) is C expf
// (sampler.nim:56); on x86-64 Linux that is glibc's expf (glibc >= 2.28),
// which implements the method published in Arm's optimized-routines
// (math/expf.c, Szabolcs Nagy, 2017) and is NOT correctly rounded: on
// 97,052 of the floats in [-104, 0] it differs from the correctly rounded
// exponential by one ulp. This is that method, restated operation by
// operation in double precision, with the multiply-adds fused as in glibc's
// x86-64 FMA build (the variant its resolver picks on any CPU with FMA):
//   z  = x * 32/ln2;  k = round(z) (by adding 1.5 * 2^52);  r = z - k, with
//   the product and the subtraction in one fused multiply-add;
//   2^(k/32) = 2^(k >> 5) * T[k & 31]  (T[j] = 2^(j/32) rounded to double,
//   stored with j/32 taken out of its exponent field);
//   2^(r/32) ~ 1 + c2 r + c1 r^2 + c0 r^3 (the published minimax cubic);
//   the double result rounded once to float.
// Inputs below -0x1.9fe368p6 give 0, above 0x1.62e42ep6 +inf, NaN gives NaN.
// Checked bit for bit against the host's glibc expf over every float (host
// restatement) and on the GPU over [-104, 0].
// (global memory, read through the read-only cache: a warp's 32 lanes index
// it at different places, which constant memory would serialise)
__device__ static const unsigned long long kExp2Tab[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};
__device__ __forceinline__ float ref_expf(float x) {
  constexpr double kInvLn2N = 0x1.71547652b82fep0 * 32.0;
  constexpr double kShift = 0x1.8p+52;
  constexpr double kC0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
  constexpr double kC1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
  constexpr double kC2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  if (x != x) return x;
  if (x < -0x1.9fe368p6f) return 0.0f;
  if (x > 0x1.62e42ep6f) return INFINITY;
  const double xd = (double)x;
  double kd = __fma_rn(kInvLn2N, xd, kShift);
  const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
  kd = __dsub_rn(kd, kShift);
  const double r = __fma_rn(kInvLn2N, xd, -kd);
  const unsigned long long t = __ldg(&kExp2Tab[ki & 31ull]) + (ki << 47);
  const double s = __longlong_as_double((long long)t);
  const double z = __fma_rn(kC0, r, kC1);
  double y = __fma_rn(kC2, r, 1.0);
  y = __fma_rn(z, __dmul_rn(r, r), y);
  return __double2float_rn(__dmul_rn(y, s));
}

// Estimate of ref_expf(x): expf, documented at 2 ulp, is within
// kBracketRel = 2^-20 relative of ref_expf(x) where expf(x) >= 2^-120
// (checked on the GPU for every float in [-110, 0]). Below 2^-120 the
// estimate is not used.
constexpr float kBracketMin = 0x1p-120f;
constexpr float kBracketRel = 0x1p-20f;
__device__ __forceinline__ float texp_estimate(float x) { return expf(x); }

// Row classification (sampler.nim:77-78, 85-86).
__device__ __forceinline__ int row_mode(const nls_row_params& p, int V, int64_t* k_out) {
  int64_t k = (p.top_k > 0) ? (p.top_k < V ? p.top_k : (int64_t)V) : (int64_t)V;
  *k_out = k;
  if (p.temperature <= 0.0) return kModeGreedy;
  if (k < V && k <= kLightKMax) return kModeTopK;
  return kModeFull;
}

// Penalty condition of sampler.nim:64-65.
__device__ __forceinline__ bool penalties_active(const nls_row_params& p, int64_t hist_len) {
  return hist_len > 0 &&
         (p.repeat_penalty != 1.0 || p.presence_penalty != 0.0 || p.frequency_penalty != 0.0);
}

// ---------------------------------------------------------------------------
// Patch table: the positions of one row (or chunk of a row) that penalties
// or bias modify, with the count of each id in the penalty window and its
// bias. A shared-memory open-addressing hash (keys = token id, -1 = empty)
// plus a bitmap over the chunk so the streaming loop tests one bit per
// element and probes the hash only on a hit.
// ---------------------------------------------------------------------------
struct PatchTable {
  int* key;
  int* cnt;        // count in the penalty window | kPatchHasBias
  float* bias;     // the position's logit as read; after precompute_patches: the patched value
  int* flag;       // the bias as float32 bits (valid when cnt has kPatchHasBias)
  uint32_t* bits;  // bitmap over [lo, hi): bit (pos - lo) >> gshift
  int log2size;
  int lo, hi;
  int gshift;      // positions per bit = 1 << gshift
};

__device__ __forceinline__ int patch_bitmap_words(int len, int gshift) {
  return ((((len + (1 << gshift) - 1) >> gshift)) + 31) >> 5;
}
__device__ __forceinline__ bool patch_bit(const PatchTable& T, int off) {
  const int g = off >> T.gshift;
  return (T.bits[g >> 5] >> (g & 31)) & 1u;
}

__device__ __forceinline__ uint32_t patch_hash(int tok, int log2size) {
  return ((uint32_t)tok * 0x9E3779B1u) >> (32 - log2size);
}

constexpr int kPatchHasBias = 1 << 30;
constexpr int kPatchCountMask = kPatchHasBias - 1;

// Insert `tok` (with its logit `raw`, read by the caller): the thread that
// creates the slot stores raw. Returns false when the table is full.
__device__ __forceinline__ bool patch_insert(PatchTable& T, int tok, int cnt_add,
                                             bool has_bias, float b, float raw, int* dup_flag) {
  const uint32_t mask = (1u << T.log2size) - 1u;
  uint32_t h = patch_hash(tok, T.log2size);
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    int prev = atomicCAS(&T.key[h], -1, tok);
    if (prev == -1 || prev == tok) {
      if (prev == -1) T.bias[h] = raw;
      if (cnt_add) atomicAdd(&T.cnt[h], cnt_add);
      if (has_bias) {
        int old = atomicOr(&T.cnt[h], kPatchHasBias);
        if (old & kPatchHasBias) atomicExch(dup_flag, 1);
        T.flag[h] = __float_as_int(b);
      }
      return true;
    }
    h = (h + 1u) & mask;
  }
  return false;
}

// Slot of `tok`, or -1. Linear probing without deletions: an empty slot ends
// the probe sequence of a key that is not in the table.
__device__ __forceinline__ int patch_find(const PatchTable& T, int tok) {
  const uint32_t mask = (1u << T.log2size) - 1u;
  uint32_t h = patch_hash(tok, T.log2size);
  for (uint32_t probe = 0; probe <= mask; ++probe) {
    const int k = T.key[h];
    if (k == tok) return (int)h;
    if (k == -1) return -1;
    h = (h + 1u) & mask;
  }
  return -1;
}

// Penalties then bias for one logit (sampler.nim:71-76): `cnt` occurrences
// in the penalty window (> 0 only when the penalty block is active for the
// row), then the bias b.float32 when the id has one.
__device__ __forceinline__ float penalise(float x, int cnt, bool has_bias, float b,
                                          const nls_row_params& p) {
  if (cnt > 0) {
    if (p.repeat_penalty != 1.0) {
      float rp = __double2float_rn(p.repeat_penalty);
      x = (x > 0.0f) ? __fdiv_rn(x, rp) : __fmul_rn(x, rp);
    }
    double d = __dadd_rn(__dmul_rn((double)cnt, p.frequency_penalty), p.presence_penalty);
    x = __fsub_rn(x, __double2float_rn(d));
  }
  if (has_bias) x = __fadd_rn(x, b);
  return x;
}
__device__ __forceinline__ float patch_apply(float x, const PatchTable& T, int slot,
                                             const nls_row_params& p) {
  const int word = T.cnt[slot];
  return penalise(x, word & kPatchCountMask, (word & kPatchHasBias) != 0,
                  __int_as_float(T.flag[slot]), p);
}

// The row's penalty window [h0, h1) in hist_ids (empty when the penalty block
// is inactive; the last repeat_last_n ids when that is > 0, sampler.nim:67)
// and its bias list [b0, b1).
__device__ __forceinline__ void patch_lists(const BatchArgs& a, int row, const nls_row_params& p,
                                            int64_t* h0, int64_t* h1, int64_t* b0, int64_t* b1) {
  *h0 = *h1 = *b0 = *b1 = 0;
  if (a.hist_ids != nullptr) {
    *h0 = a.hist_off[row];
    *h1 = a.hist_off[row + 1];
    if (!penalties_active(p, *h1 - *h0)) *h1 = *h0;
    else if (p.repeat_last_n > 0 && *h1 - *h0 > p.repeat_last_n) *h0 = *h1 - p.repeat_last_n;
  }
  if (a.bias_ids != nullptr) {
    *b0 = a.bias_off[row];
    *b1 = a.bias_off[row + 1];
  }
}

// Replace each slot's logit by the final patched logit of its position.
// Block-wide; after it, patched_value() gives the logit the reference sees at
// a patched position. (The logits were read while the table was built.)
__device__ inline void precompute_patches(PatchTable& T, const nls_row_params& p) {
  const int hs = 1 << T.log2size;
  for (int i = threadIdx.x; i < hs; i += blockDim.x) {
    const int k = T.key[i];
    if (k >= 0) T.bias[i] = patch_apply(T.bias[i], T, i, p);
  }
  __syncthreads();
}
__device__ __forceinline__ float patched_value(const PatchTable& T, int slot) { return T.bias[slot]; }

// Block-wide construction of the patch table for positions [lo, hi) of `row`;
// `chunk` is the row's logits from position lo. Every id's logit is read as
// its id is read (four ids per thread in flight), so the scattered loads
// overlap each other and the table's initialisation -- unless read_logits is
// false: then the caller fills each slot's logit itself before
// precompute_patches. Returns the number of patched positions
// (block-uniform). Sets *overflow / *dup (shared ints) on a full table / a
// duplicate bias id. hs must be a multiple of blockDim.x.
__device__ inline int build_patches(const BatchArgs& a, int row, const nls_row_params& p,
                                    PatchTable& T, const float* chunk, int* s_counter,
                                    int* s_overflow, int* s_dup, bool read_logits = true) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int hs = 1 << T.log2size;
  constexpr int U = 4;
  // the ids of the penalty window and of the bias list, and their logits
  int64_t h0, h1, b0, b1;
  patch_lists(a, row, p, &h0, &h1, &b0, &b1);
  const int64_t nh = h1 - h0, ntot = nh + (b1 - b0);
  for (int i = tid; i < hs; i += nt) { T.key[i] = -1; T.cnt[i] = 0; }
  const int nwords = patch_bitmap_words(T.hi - T.lo, T.gshift);
  for (int i = tid; i < nwords; i += nt) T.bits[i] = 0u;
  if (tid == 0) { *s_counter = 0; *s_overflow = 0; *s_dup = 0; }
  for (int64_t base = 0; base < ntot; base += (int64_t)U * nt) {
    int tok[U];
    float raw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = base + tid + (int64_t)u * nt;
      int64_t t = -1;
      if (j < nh) t = a.hist_ids[h0 + j];
      else if (j < ntot) t = a.bias_ids[b0 + (j - nh)];
      tok[u] = (t >= T.lo && t < T.hi) ? (int)t : -1;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) raw[u] = (read_logits && tok[u] >= 0) ? __ldg(chunk + (tok[u] - T.lo)) : 0.0f;
    if (base == 0) __syncthreads();  // the table is initialised
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t j = base + tid + (int64_t)u * nt;
      if (tok[u] < 0) continue;
      bool ok;
      if (j < nh) {
        ok = patch_insert(T, tok[u], 1, false, 0.0f, raw[u], s_dup);
      } else {
        const float b = __double2float_rn(a.bias_vals[b0 + (j - nh)]);  // b.float32 (:76)
        ok = patch_insert(T, tok[u], 0, true, b, raw[u], s_dup);
      }
      if (!ok) atomicExch(s_overflow, 1);
    }
  }
  __syncthreads();
  const int lane = tid & 31;
  for (int i = tid; i < hs; i += nt) {
    const int k = T.key[i];
    if (k >= 0) {
      const int off = (k - T.lo) >> T.gshift;
      atomicOr(&T.bits[off >> 5], 1u << (off & 31));
    }
    const unsigned m = __ballot_sync(0xffffffffu, k >= 0);
    if (lane == 0 && m) atomicAdd(s_counter, __popc(m));
  }
  __syncthreads();
  return *s_counter;
}

// ---------------------------------------------------------------------------
// Block-wide radix select: the K-th largest key (1-based) among the entries i
// in [0, n) for which get(i, &key) returns true. 8-bit digits, 4 rounds; the
// shared histogram is filled with warp-aggregated atomics (__match_any_sync),
// since sampler keys are heavily skewed onto a few top-byte values.
// `hist` is 256 shared words, `sh` at least 4 shared words. All threads call;
// blockDim.x must be a multiple of 32.
// ---------------------------------------------------------------------------
//
// With rounds < 4 only the top 8*rounds bits are resolved: the result is then
// that prefix with the low bits zero, a lower bound of the K-th largest key,
// and sh[2] receives the number of entries at or above it.
template <class Get>
__device__ uint32_t block_select_kth_largest(int n, uint32_t K, Get get, uint32_t* hist,
                                             uint32_t* sh, int rounds = 4) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31;
  uint32_t prefix = 0, pmask = 0;
  if (tid == 0) { sh[0] = 0; sh[1] = K; sh[2] = 0; sh[3] = 0; }
  const int nround = (n + nt - 1) / nt * nt;
  const int last_shift = 32 - 8 * rounds;
  for (int shift = 24; shift >= last_shift; shift -= 8) {
    for (int i = tid; i < 256; i += nt) hist[i] = 0u;
    __syncthreads();
    for (int i = tid; i < nround; i += nt) {
      uint32_t k = 0;
      const bool ok = (i < n) && get(i, &k) && ((k & pmask) == prefix);
      const int bin = ok ? (int)((k >> shift) & 255u) : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (ok && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (tid < 32) {
      uint32_t rem = sh[1];
      // lane l owns bins 255-8l .. 248-8l (descending)
      uint32_t c = 0;
#pragma unroll
      for (int b = 0; b < 8; ++b) c += hist[255 - 8 * lane - b];
      uint32_t incl = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        uint32_t v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
      }
      uint32_t ball = __ballot_sync(0xffffffffu, incl >= rem);
      int L = __ffs(ball) - 1;
      if (lane == L) {
        uint32_t above = incl - c;
        int d = 0;
        for (int b = 0; b < 8; ++b) {
          int bin = 255 - 8 * lane - b;
          uint32_t hc = hist[bin];
          if (above + hc >= rem) { d = bin; break; }
          above += hc;
        }
        sh[0] = (uint32_t)d;
        sh[1] = rem - above;
        sh[2] = sh[3] + above + hist[d];  // entries >= the new prefix
        sh[3] += above;                   // entries strictly above the prefix
      }
    }
    __syncthreads();
    prefix |= sh[0] << shift;
    pmask |= 255u << shift;
    // (within the loop the next round's first barrier already separates
    // these reads of sh[0] from warp 0's next write of it; after the last
    // round a barrier keeps a following call's reset of sh behind them)
    if (shift == last_shift) __syncthreads();
  }
  return prefix;
}

// One warp's version of block_select_kth_largest for small n: the K-th
// largest key among the accepted entries (get() as above), by four rounds of
// an 8-bit radix select over a 256-bin shared histogram. Returns the key;
// *n_ge = entries >= it, *n_gt = entries > it (-1/-1 when fewer than K).
// Warp-synchronous: all 32 lanes call it, no block barrier.
template <class Get>
__device__ uint32_t warp_select_kth_largest(int n, uint32_t K, Get get, uint32_t* hist, int* n_ge,
                                            int* n_gt) {
  const int lane = threadIdx.x & 31;
  uint32_t prefix = 0, pmask = 0, rem = K, above = 0;
  // The accepted keys often share their top bytes (a row's best candidates):
  // the rounds start at the first byte where the smallest and the largest
  // differ (the last round always runs: it counts n_ge and n_gt).
  int start = 24;
  {
    uint32_t kmn = 0xffffffffu, kmx = 0u;
    for (int i = lane; i < n; i += 32) {
      uint32_t k = 0;
      if (get(i, &k)) {
        kmn = min(kmn, k);
        kmx = max(kmx, k);
      }
    }
    kmn = __reduce_min_sync(0xffffffffu, kmn);
    kmx = __reduce_max_sync(0xffffffffu, kmx);
    if (kmn <= kmx) {
      const int skip = min(__clz(kmn ^ kmx) / 8, 3);  // whole bytes shared
      start = 24 - 8 * skip;
      pmask = skip ? (0xffffffffu << (32 - 8 * skip)) : 0u;
      prefix = kmn & pmask;
    }
  }
  for (int shift = start; shift >= 0; shift -= 8) {
#pragma unroll
    for (int b = 0; b < 8; ++b) hist[lane * 8 + b] = 0u;
    __syncwarp();
    for (int i = lane; i < n; i += 32) {
      uint32_t k = 0;
      if (get(i, &k) && (k & pmask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
    }
    __syncwarp();
    // lane l owns bins 255-8l .. 248-8l (descending key order)
    uint32_t cnt[8], c = 0;
#pragma unroll
    for (int b = 0; b < 8; ++b) { cnt[b] = hist[255 - 8 * lane - b]; c += cnt[b]; }
    uint32_t incl = c;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    const unsigned ball = __ballot_sync(0xffffffffu, incl >= rem);
    if (!ball) {  // fewer than K accepted entries
      *n_ge = -1;
      *n_gt = -1;
      return 0u;
    }
    const int L = __ffs(ball) - 1;
    uint32_t d = 0, a2 = 0, hd = 0;
    if (lane == L) {
      uint32_t ab = incl - c;
#pragma unroll
      for (int b = 0; b < 8; ++b) {
        if (ab + cnt[b] >= rem) { d = 255u - 8u * (uint32_t)lane - (uint32_t)b; hd = cnt[b]; break; }
        ab += cnt[b];
      }
      a2 = ab;
    }
    d = __shfl_sync(0xffffffffu, d, L);
    a2 = __shfl_sync(0xffffffffu, a2, L);
    hd = __shfl_sync(0xffffffffu, hd, L);
    rem -= a2;
    above += a2;
    prefix |= d << shift;
    pmask |= 255u << shift;
    if (shift == 0) {
      *n_gt = (int)above;
      *n_ge = (int)(above + hd);
    }
    __syncwarp();
  }
  return prefix;
}

// One warp's bitonic sort of n64 (power of two, >= 2) uint64 keys in shared
// memory, descending.
__device__ inline void warp_bitonic_desc(unsigned long long* v, int n64) {
  const int lane = threadIdx.x & 31;
  for (int size = 2; size <= n64; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = lane; i < n64 / 2; i += 32) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const unsigned long long x = v[lo], y = v[hi];
        if ((x < y) == desc) { v[lo] = y; v[hi] = x; }
      }
      __syncwarp();
    }
  }
}

// Block-wide bitonic sort of n64 (power of two) uint64 keys, descending.
__device__ inline void block_bitonic_desc(unsigned long long* v, int n64) {
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int size = 2; size <= n64; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < n64 / 2; i += nt) {
        int lo = 2 * i - (i & (stride - 1));
        int hi = lo + stride;
        bool desc = ((lo & size) == 0);
        unsigned long long x = v[lo], y = v[hi];
        if ((x < y) == desc) { v[lo] = y; v[hi] = x; }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

}  // namespace nls
