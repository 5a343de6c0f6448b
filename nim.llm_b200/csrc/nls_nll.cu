// nls_nll.cu -- the per-position negative log-likelihood of perplexity
// (src/nimllm/model.nim:570-589 in the reference).
//
// For position t the reference takes mx = the fp32 maximum of the row
// (:581), s = sum over k of exp(float64(x_k - mx)) with the difference in
// fp32 and the exponential and the sum in float64 (:582-583), and adds
// -(float64(x_target - mx) - ln(s)) to its running total (:584). This kernel
// writes that term per row; the caller sums the terms and takes
// exp(total / count) (:589).
//
// One CTA per row (grid-stride over rows): a max pass with four float4 loads
// in flight per thread, then a pass summing the float64 terms (the second
// read of the row is mostly served by L2). The float64 sum runs in a tree
// order instead of the reference's index order: the two differ by rounding
// only (a few units of 2^-53 relative per term), far inside the tolerance the
// tests state. A row with a NaN or a non-finite maximum gets NaN and
// NLS_ERR_NAN_LOGITS; a target outside [0, V) gets NaN and
// NLS_ERR_INVALID_ARG (the reference would raise IndexDefect there).
#include <atomic>
#include <cmath>

#include "nls_common.cuh"
#include "nls_kernels.h"

namespace nls {

namespace {

constexpr int NL_THREADS = 512;
constexpr int NL_WARPS = NL_THREADS / 32;

struct NllShared {
  float fmax[NL_WARPS];
  double dsum[NL_WARPS];
  int nan;
};

__global__ void __launch_bounds__(NL_THREADS)
nll_kernel(const float* logits, int64_t ld, int rows, int V, const int64_t* targets, double* out,
           int* status) {
  __shared__ NllShared S;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* x = logits + (int64_t)row * ld;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
    const int nv4 = vec ? (V >> 2) : 0;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    // 1. the maximum (model.nim:581) and whether any logit is NaN
    float m = -INFINITY;
    bool nan = false;
    {
      constexpr int U = 4;
      int g = tid;
      for (; g + (U - 1) * NL_THREADS < nv4; g += U * NL_THREADS) {
        float4 q[U];
#pragma unroll
        for (int u = 0; u < U; ++u) q[u] = x4[g + u * NL_THREADS];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          nan |= (q[u].x != q[u].x) | (q[u].y != q[u].y) | (q[u].z != q[u].z) | (q[u].w != q[u].w);
          m = fmaxf(m, fmaxf(fmaxf(q[u].x, q[u].y), fmaxf(q[u].z, q[u].w)));
        }
      }
      for (; g < nv4; g += NL_THREADS) {
        const float4 q = x4[g];
        nan |= (q.x != q.x) | (q.y != q.y) | (q.z != q.z) | (q.w != q.w);
        m = fmaxf(m, fmaxf(fmaxf(q.x, q.y), fmaxf(q.z, q.w)));
      }
      for (int i = 4 * nv4 + tid; i < V; i += NL_THREADS) {
        const float v = x[i];
        nan |= (v != v);
        m = fmaxf(m, v);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const bool wnan = __any_sync(0xffffffffu, nan);
    if (tid == 0) S.nan = 0;
    __syncthreads();
    if (lane == 0) {
      S.fmax[warp] = m;
      if (wnan) S.nan = 1;
    }
    __syncthreads();
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NL_WARPS; ++w) mx = fmaxf(mx, S.fmax[w]);
    const int64_t tgt = targets[row];
    if (S.nan || !isfinite(mx) || tgt < 0 || tgt >= V) {
      if (tid == 0) {
        out[row] = __longlong_as_double(0x7ff8000000000000ll);  // NaN
        record_status(status, (S.nan || !isfinite(mx)) ? NLS_ERR_NAN_LOGITS : NLS_ERR_INVALID_ARG);
      }
      __syncthreads();
      continue;
    }
    // 2. s = sum of exp(float64(x_k - mx)) (model.nim:582-583)
    double s = 0.0;
    {
      constexpr int U = 4;
      int g = tid;
      for (; g + (U - 1) * NL_THREADS < nv4; g += U * NL_THREADS) {
        float4 q[U];
#pragma unroll
        for (int u = 0; u < U; ++u) q[u] = x4[g + u * NL_THREADS];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          s += exp((double)__fsub_rn(q[u].x, mx));
          s += exp((double)__fsub_rn(q[u].y, mx));
          s += exp((double)__fsub_rn(q[u].z, mx));
          s += exp((double)__fsub_rn(q[u].w, mx));
        }
      }
      for (; g < nv4; g += NL_THREADS) {
        const float4 q = x4[g];
        s += exp((double)__fsub_rn(q.x, mx));
        s += exp((double)__fsub_rn(q.y, mx));
        s += exp((double)__fsub_rn(q.z, mx));
        s += exp((double)__fsub_rn(q.w, mx));
      }
      for (int i = 4 * nv4 + tid; i < V; i += NL_THREADS) s += exp((double)__fsub_rn(x[i], mx));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) S.dsum[warp] = s;
    __syncthreads();
    if (tid == 0) {
      double tot = 0.0;
#pragma unroll
      for (int w = 0; w < NL_WARPS; ++w) tot += S.dsum[w];
      // model.nim:584
      out[row] = -((double)__fsub_rn(x[tgt], mx) - log(tot));
    }
    __syncthreads();
  }
}

}  // namespace

cudaError_t launch_nll(const float* logits, int64_t ld, int rows, int V, const int64_t* targets,
                       double* out, int* status, int sm_count, cudaStream_t stream) {
  int grid = rows < 4 * sm_count ? rows : 4 * sm_count;
  if (grid < 1) grid = 1;
  nll_kernel<<<grid, NL_THREADS, 0, stream>>>(logits, ld, rows, V, targets, out, status);
  return cudaGetLastError();
}

}  // namespace nls
