// nls_top.cu -- topTokens (src/nimllm/sampler.nim:123-130 in the reference):
// the n most probable tokens of a row with their probabilities.
//
// The reference copies the row, runs softmaxInPlace over it (:51-57: max,
// then v = expf(v - max) and a sequential fp32 sum in INDEX order, then
// v /= s), and stable-sorts the indices by probability, descending (equal
// probabilities keep ascending index). Here, one 1024-thread CTA per row:
//   1. the row's maximum (a NaN or a non-finite maximum is reported as an
//      error: the reference's probabilities are NaN there);
//   2. s replayed exactly in index order by exact_scan_fast, with the terms
//      t_i = expf(x_i - max) cached in the CTA's scratch;
//   3. the n-th largest key (radix select), then the largest key whose
//      probability still equals the n-th one's (probabilities are a
//      non-increasing function of the key, but rounding can make distinct
//      logits equally probable, and those then order by index);
//   4. those candidates (at most kTopCap) sorted by (probability desc, index
//      asc) in shared memory; the first n are the result.
#include <atomic>
#include <climits>

#include "nls_common.cuh"
#include "nls_kernels.h"
#include "nls_scan.cuh"

namespace nls {

namespace {

constexpr int TP_THREADS = 1024;
constexpr int TP_EPT = 4;
constexpr int kTopCap = 2048;  // candidates sorted per row

struct TopShared {
  ScanShared scan;
  FastScanShared fscan;
  uint32_t hist[256];
  uint32_t sel[4];
  float fred[32];
  int ired[32];
  int nan;
  int ncand;
  uint32_t kstar;
  unsigned long long cand[kTopCap];
};

__device__ float block_max_f(float v, int* nanflag, TopShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if (lane == 0) S.fred[warp] = v;
  __syncthreads();
  float m = (lane < TP_THREADS / 32) ? S.fred[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int nf = *nanflag;
  __syncthreads();
  *nanflag = nf;
  return m;
}

// exclusive prefix sum of v over the block (thread order); *total gets the sum
__device__ int block_scan_excl(int v, int* total, TopShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) S.ired[warp] = incl;
  __syncthreads();
  const int c = (lane < TP_THREADS / 32) ? S.ired[lane] : 0;
  const int pre = __reduce_add_sync(0xffffffffu, lane < warp ? c : 0);
  *total = __reduce_add_sync(0xffffffffu, c);
  __syncthreads();
  return pre + incl - v;
}

__global__ void __launch_bounds__(TP_THREADS, 1)
top_kernel(const float* logits, int64_t ld, int rows, int V, int n, int64_t* out_ids,
           float* out_probs, int* status, uint32_t* scratch, int vpad) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TopShared& S = *reinterpret_cast<TopShared*>(smem_raw);
  const int tid = threadIdx.x;
  float* TT = reinterpret_cast<float*>(scratch + (size_t)blockIdx.x * 4 * (size_t)vpad);
  const int nout = n < V ? n : V;

  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* x = logits + (int64_t)row * ld;
    int64_t* oid = out_ids + (int64_t)row * n;
    float* opr = out_probs ? out_probs + (int64_t)row * n : nullptr;
    // 1. maximum and NaN
    if (tid == 0) S.nan = 0;
    __syncthreads();
    float m = -INFINITY;
    bool nan = false;
    for (int i = tid; i < V; i += TP_THREADS) {
      const float v = x[i];
      nan |= (v != v);
      m = fmaxf(m, v);
    }
    if (__any_sync(0xffffffffu, nan) && (tid & 31) == 0) S.nan = 1;
    int nf = 0;
    const float mx = block_max_f(m, &nf, S);
    const int anynan = S.nan;
    __syncthreads();
    if (anynan || !isfinite(mx)) {
      for (int i = tid; i < n; i += TP_THREADS) {
        oid[i] = -1;
        if (opr) opr[i] = 0.0f;
      }
      if (tid == 0) record_status(status, NLS_ERR_NAN_LOGITS);
      __syncthreads();
      continue;
    }
    // 2. s in index order, exactly (no absorption: index order is not sorted)
    int tt_valid = 0;
    auto prep = [&](int j0, int j1) {
      if (j1 > tt_valid) {
        for (int j = (j0 > tt_valid ? j0 : tt_valid) + tid; j < j1; j += TP_THREADS)
          TT[j] = ref_expf(__fsub_rn(x[j], mx));
        tt_valid = j1;
        __syncthreads();
      }
    };
    auto tval = [&](int j) { return TT[j]; };
    auto nostop = [](float) { return false; };
    const float s = exact_scan_fast<TP_THREADS, TP_EPT, false>(0, V, 0.0f, tval, nostop, false, false,
                                                               S.scan, S.fscan, prep).v;
    // 3. the n-th largest key (descending value: ascending ~fkey) and its
    //    probability pn; probabilities are a non-increasing function of the
    //    key, so {p > pn} is the key range below kA and {p == pn} is
    //    [kA, kB]. Rounding can make distinct logits equally probable, and
    //    equal probabilities order by index, so the tie group contributes its
    //    lowest indices.
    auto pk = [&](uint32_t kd) { return __fdiv_rn(ref_expf(__fsub_rn(fkey_inv(~kd), mx)), s); };
    const uint32_t kth = ~block_select_kth_largest(
        V, (uint32_t)nout, [&](int i, uint32_t* k) { *k = fkey(x[i]); return true; }, S.hist, S.sel);
    if (tid == 0) {
      const float pn = pk(kth);
      const uint32_t kinf = ~fkey(-INFINITY);  // the largest key of a non-NaN value
      uint32_t lo = kth, hi = kinf;           // largest key with pk >= pn
      while (lo < hi) {
        const uint32_t mid = lo + ((hi - lo + 1u) >> 1);
        if (pk(mid) >= pn) lo = mid; else hi = mid - 1u;
      }
      S.kstar = lo;  // kB
      uint32_t lo2 = 0u, hi2 = kth;           // smallest key with pk <= pn
      while (lo2 < hi2) {
        const uint32_t mid = lo2 + ((hi2 - lo2) >> 1);
        if (pk(mid) <= pn) hi2 = mid; else lo2 = mid + 1u;
      }
      S.sel[3] = lo2;  // kA
      S.ncand = 0;
    }
    __syncthreads();
    const uint32_t kB = S.kstar, kA = S.sel[3];
    __syncthreads();
    // 4a. everything strictly more probable than pn (fewer than n elements)
    for (int i = tid; i < V; i += TP_THREADS) {
      const uint32_t kd = ~fkey(x[i]);
      if (kd < kA) {
        const int pos = atomicAdd(&S.ncand, 1);
        if (pos < kTopCap) {
          const float p = __fdiv_rn(ref_expf(__fsub_rn(x[i], mx)), s);
          S.cand[pos] = ((unsigned long long)(~fkey(p)) << 32) | (uint32_t)i;
        }
      }
    }
    __syncthreads();
    // 4b. the lowest indices of the tie group, in index order
    {
      int need = nout - S.ncand;  // same in every thread
      __syncthreads();
      for (int t0 = 0; t0 < V && need > 0; t0 += TP_THREADS) {
        const int i = t0 + tid;
        const bool tie = i < V && ~fkey(x[i]) >= kA && ~fkey(x[i]) <= kB;
        int tot;
        const int rank = block_scan_excl(tie ? 1 : 0, &tot, S);
        if (tie && rank < need) {
          const int pos = atomicAdd(&S.ncand, 1);
          if (pos < kTopCap) {
            const float p = __fdiv_rn(ref_expf(__fsub_rn(x[i], mx)), s);
            S.cand[pos] = ((unsigned long long)(~fkey(p)) << 32) | (uint32_t)i;
          }
        }
        need -= tot;
      }
    }
    __syncthreads();
    const int nc = S.ncand;
    if (nc > kTopCap) {
      for (int i = tid; i < n; i += TP_THREADS) {
        oid[i] = -1;
        if (opr) opr[i] = 0.0f;
      }
      if (tid == 0) record_status(status, NLS_ERR_CAPACITY);
      __syncthreads();
      continue;
    }
    int n64 = 32;
    while (n64 < nc) n64 <<= 1;
    for (int i = nc + tid; i < n64; i += TP_THREADS) S.cand[i] = ~0ull;
    __syncthreads();
    // ascending (~fkey(p), index) = probability descending, index ascending
    block_bitonic_desc(S.cand, n64);  // descending sort ...
    for (int i = tid; i < n; i += TP_THREADS) {
      if (i < nout) {
        const unsigned long long v = S.cand[n64 - 1 - i];  // ... read from the back
        oid[i] = (int64_t)(uint32_t)(v & 0xffffffffull);
        if (opr) opr[i] = fkey_inv(~(uint32_t)(v >> 32));
      } else {
        oid[i] = -1;
        if (opr) opr[i] = 0.0f;
      }
    }
    __syncthreads();
  }
}

}  // namespace

size_t top_smem_bytes() { return sizeof(TopShared); }

cudaError_t launch_top(const float* logits, int64_t ld, int rows, int V, int n, int64_t* out_ids,
                       float* out_probs, int* status, uint32_t* scratch, int vpad, int slots,
                       cudaStream_t stream) {
  const size_t smem = top_smem_bytes();
  static std::atomic<int> done[kMaxDevicesAttr];
  cudaError_t e = ensure_smem_attr(reinterpret_cast<const void*>(top_kernel), (int)smem, done);
  if (e != cudaSuccess) return e;
  const int grid = rows < slots ? rows : slots;
  top_kernel<<<grid, TP_THREADS, smem, stream>>>(logits, ld, rows, V, n, out_ids, out_probs, status,
                                                 scratch, vpad);
  return cudaGetLastError();
}

}  // namespace nls
