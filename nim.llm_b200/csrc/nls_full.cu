// nls_full.cu -- rows that need more than a small top-k: top_k <= 0 or
// top_k >= vocab (the reference's full stable sort, sampler.nim:96-97),
// 256 < top_k < vocab (the heap path with a large k, sampler.nim:86-95), and
// rows the streaming kernel handed over (buffers overflowed by ties, or a
// penalty window with too many distinct ids for its table).
//
// One 1024-thread CTA per row, persistent over the work list, with its own
// scratch slot of 3 x vocab words in HBM:
//   1. transform: penalties, bias, temperature; each logit becomes a 32-bit
//      key that sorts ascending in the reference's candidate order;
//   2. LSD radix sort of the keys (4 x 8-bit digits, stable warp ranking);
//   3. t_j = expf(y_j - max), then the reference's sequential fp32 sums --
//      softmax denominator, top-p running sum, min-p cut, draw total and the
//      draw itself -- replayed exactly by the block scan in nls_scan.cuh;
//   4. the drawn position is mapped back to a token id with the reference's
//      tie order (ascending index for the stable sort; for the heap path,
//      descending index and the heap's survivor rule among ties at the k-th
//      value).
#include <climits>

#include "nls_common.cuh"
#include "nls_kernels.h"
#include "nls_scan.cuh"

namespace nls {

constexpr int FT_THREADS = 1024;
constexpr int FT_EPT = 4;
constexpr int FT_TILE = FT_THREADS * FT_EPT;
constexpr int FT_WARPS = FT_THREADS / 32;
constexpr int FT_HASH_LOG2 = 12;

struct FullShared {
  int hkey[1 << FT_HASH_LOG2];
  int hcnt[1 << FT_HASH_LOG2];
  float hbias[1 << FT_HASH_LOG2];
  int hflag[1 << FT_HASH_LOG2];
  int wcnt[FT_WARPS][257];
  uint32_t base[256];
  uint32_t tilecnt[256];
  ScanShared scan;
  int ired[FT_WARPS];
  float fred[FT_WARPS];
  int ibuf[8];
  float fbuf[8];
  int counter, patch_overflow, dup, nan;
};

size_t full_smem_bytes(int V) {
  size_t bm_words = ((size_t)V + 31) / 32;
  bm_words = (bm_words + 3) & ~(size_t)3;
  return ((sizeof(FullShared) + 15) & ~(size_t)15) + bm_words * 4;
}

// ---- small block utilities ------------------------------------------------
__device__ int block_sum_int(int v, FullShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_add_sync(0xffffffffu, v);
  if (lane == 0) S.ired[warp] = v;
  __syncthreads();
  int tot = 0;
#pragma unroll 8
  for (int w = 0; w < FT_WARPS; ++w) tot += S.ired[w];
  __syncthreads();
  return tot;
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
  int wpre = 0, tot = 0;
  for (int w = 0; w < FT_WARPS; ++w) {
    int c = S.ired[w];
    if (w < warp) wpre += c;
    tot += c;
  }
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

// ---- LSD radix sort passes (keys only, stable) -----------------------------
__device__ void lsd_count(const uint32_t* src, int n, int sh, FullShared& S) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int d = lane; d < 257; d += 32) S.wcnt[warp][d] = 0;
  __syncwarp();
  for (int t0 = 0; t0 < n; t0 += FT_TILE) {
#pragma unroll
    for (int j = 0; j < FT_EPT; ++j) {
      const int i = t0 + warp * (32 * FT_EPT) + j * 32 + lane;
      const int d = (i < n) ? (int)((src[i] >> sh) & 255u) : 256;
      const unsigned peers = __match_any_sync(0xffffffffu, d);
      if (lane == __ffs(peers) - 1 && d < 256) S.wcnt[warp][d] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  if (threadIdx.x < 256) {
    int c = 0;
    for (int w = 0; w < FT_WARPS; ++w) c += S.wcnt[w][threadIdx.x];
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
    for (int d = lane; d < 257; d += 32) S.wcnt[warp][d] = 0;
    __syncwarp();
    uint32_t k[FT_EPT];
    int dg[FT_EPT], rk[FT_EPT];
#pragma unroll
    for (int j = 0; j < FT_EPT; ++j) {
      const int i = t0 + warp * (32 * FT_EPT) + j * 32 + lane;
      k[j] = (i < n) ? src[i] : 0u;
      dg[j] = (i < n) ? (int)((k[j] >> sh) & 255u) : 256;
      const unsigned peers = __match_any_sync(0xffffffffu, dg[j]);
      const int before = S.wcnt[warp][dg[j]];
      __syncwarp();
      rk[j] = before + __popc(peers & ltmask);
      if (lane == __ffs(peers) - 1) S.wcnt[warp][dg[j]] = before + __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    if (threadIdx.x < 256) {
      int run = 0;
      for (int w = 0; w < FT_WARPS; ++w) {
        int c = S.wcnt[w][threadIdx.x];
        S.wcnt[w][threadIdx.x] = run;
        run += c;
      }
      S.tilecnt[threadIdx.x] = (uint32_t)run;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < FT_EPT; ++j) {
      if (dg[j] < 256) dst[S.base[dg[j]] + S.wcnt[warp][dg[j]] + rk[j]] = k[j];
    }
    __syncthreads();
    if (threadIdx.x < 256) S.base[threadIdx.x] += S.tilecnt[threadIdx.x];
    __syncthreads();
  }
}

// Order key of the full-sort path: ascending key == the reference's
// candidate order by value (descending logit).
__device__ __forceinline__ uint32_t desc_key(float y) { return ~fkey(y); }
__device__ __forceinline__ float desc_key_value(uint32_t kd) { return fkey_inv(~kd); }

__global__ void __launch_bounds__(FT_THREADS, 1)
full_kernel(BatchArgs a, uint32_t* scratch, int vpad) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FullShared& S = *reinterpret_cast<FullShared*>(smem_raw);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem_raw + ((sizeof(FullShared) + 15) & ~(size_t)15));
  const int tid = threadIdx.x;
  const int V = a.V;
  uint32_t* orig = scratch + (size_t)blockIdx.x * 3 * (size_t)vpad;
  uint32_t* A = orig + vpad;
  uint32_t* B = A + vpad;
  float* Af = reinterpret_cast<float*>(A);
  const int nwork = *a.full_count;

  for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
    const int row = a.full_list[w];
    const nls_row_params p = a.params[row];
    int64_t K64;
    const int mode = row_mode(p, V, &K64);
    const bool greedy = (mode == kModeGreedy);
    if (!greedy && a.uniforms == nullptr) {
      if (tid == 0) { a.out_ids[row] = -1; record_status(a.status, NLS_ERR_INVALID_ARG); }
      continue;
    }
    // heap path iff k < V (sampler.nim:86)
    const bool heap = (K64 < V);
    const int ncand = heap ? (int)K64 : V;

    PatchTable T{S.hkey, S.hcnt, S.hbias, S.hflag, bitmap, FT_HASH_LOG2, 0, V, 0};
    const int npatch = build_patches(a, row, p, T, &S.counter, &S.patch_overflow, &S.dup);
    if (S.patch_overflow || S.dup) {
      if (tid == 0) {
        a.out_ids[row] = -1;
        record_status(a.status, S.dup ? NLS_ERR_INVALID_ARG : NLS_ERR_CAPACITY);
      }
      __syncthreads();
      continue;
    }
    if (tid == 0) S.nan = 0;
    __syncthreads();

    const float* rowp = a.logits + (int64_t)row * a.ld;
    if (greedy) {
      // argmax over the patched row (sampler.nim:45-49, 77-78)
      float gb = 0.0f;
      int gi = INT_MAX;
      for (int i = tid; i < V; i += FT_THREADS) {
        float x = rowp[i];
        if (npatch > 0 && patch_bit(T, i)) {
          const int slot = patch_find(T, i);
          if (slot >= 0) x = patch_apply(x, T, slot, p);
        }
        if (i == 0 && x != x) S.nan = 1;
        if (!(x != x) && (gi == INT_MAX || x > gb)) { gb = x; gi = i; }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        float ob = __shfl_down_sync(0xffffffffu, gb, off);
        int oi = __shfl_down_sync(0xffffffffu, gi, off);
        if (oi != INT_MAX && (gi == INT_MAX || ob > gb || (ob == gb && oi < gi))) { gb = ob; gi = oi; }
      }
      if ((tid & 31) == 0) { S.fred[tid >> 5] = gb; S.ired[tid >> 5] = gi; }
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

    // 1. transform
    const float invT = __double2float_rn(__ddiv_rn(1.0, p.temperature));
    int anynan = 0;
    for (int i = tid; i < V; i += FT_THREADS) {
      float x = rowp[i];
      if (npatch > 0 && patch_bit(T, i)) {
        const int slot = patch_find(T, i);
        if (slot >= 0) x = patch_apply(x, T, slot, p);
      }
      const float y = __fmul_rn(x, invT);
      anynan |= (y != y);
      orig[i] = desc_key(y);
    }
    if (block_sum_int(anynan, S) > 0) {
      if (tid == 0) {
        a.out_ids[row] = -1;
        if (a.out_probs) a.out_probs[row] = 0.0f;
        record_status(a.status, NLS_ERR_NAN_LOGITS);
      }
      continue;
    }
    __threadfence_block();
    __syncthreads();
    // 2. sort: orig -> A -> B -> A -> B
    lsd_count(orig, V, 0, S);
    lsd_scatter(orig, A, V, 0, S);
    lsd_count(A, V, 8, S);
    lsd_scatter(A, B, V, 8, S);
    lsd_count(B, V, 16, S);
    lsd_scatter(B, A, V, 16, S);
    lsd_count(A, V, 24, S);
    lsd_scatter(A, B, V, 24, S);
    __syncthreads();

    const float mx = desc_key_value(B[0]);
    const double u_draw = a.uniforms[row];
    int pos;
    float s, prob;
    if (!isfinite(mx)) {
      // Non-finite maximum: the reference's arithmetic produces NaNs that a
      // grid replay cannot represent; run its loops literally (one thread).
      if (tid == 0) {
        float m = -INFINITY;
        for (int j = 0; j < ncand; ++j) {
          float y = desc_key_value(B[j]);
          m = (m <= y) ? y : m;
        }
        float ss = 0.0f;
        for (int j = 0; j < ncand; ++j) {
          float tj = ref_expf(__fsub_rn(desc_key_value(B[j]), m));
          Af[j] = tj;
          ss = __fadd_rn(ss, tj);
        }
        for (int j = 0; j < ncand; ++j) Af[j] = __fdiv_rn(Af[j], ss);
        int n = ncand;
        if (p.top_p > 0.0 && p.top_p < 1.0) {
          float cum = 0.0f;
          for (int j = 0; j < n; ++j) {
            cum = __fadd_rn(cum, Af[j]);
            if ((double)cum >= p.top_p) { n = j + 1; break; }
          }
        }
        if (p.min_p > 0.0) {
          const float thr = __fmul_rn(Af[0], __double2float_rn(p.min_p));
          int m2 = 1;
          while (m2 < n && Af[m2] >= thr) ++m2;
          n = m2;
        }
        float total = 0.0f;
        for (int j = 0; j < n; ++j) total = __fadd_rn(total, Af[j]);
        float r = __fmul_rn(__double2float_rn(u_draw), total);
        int ps = n - 1;
        for (int j = 0; j < n; ++j) {
          r = __fsub_rn(r, Af[j]);
          if (r <= 0.0f) { ps = j; break; }
        }
        S.ibuf[1] = ps;
        S.fbuf[1] = Af[ps];
      }
      __syncthreads();
      pos = S.ibuf[1];
      prob = S.fbuf[1];
      __syncthreads();
    } else {
      // 3. t_j = expf(y_j - max) in candidate order
      for (int j = tid; j < ncand; j += FT_THREADS)
        Af[j] = ref_expf(__fsub_rn(desc_key_value(B[j]), mx));
      __threadfence_block();
      __syncthreads();
      auto tval = [&](int j) { return Af[j]; };
      auto nostop = [](float) { return false; };
      // softmax denominator (sampler.nim:54-56)
      s = exact_scan<FT_THREADS, FT_EPT, false>(0, ncand, 0.0f, tval, nostop, false, true, S.scan).v;
      auto pval = [&](int j) { return __fdiv_rn(Af[j], s); };
      // min-p first cut (sampler.nim:110-113): first j >= 1 with p_j < thr
      int nlim = ncand;
      if (p.min_p > 0.0) {
        const float thr = __fmul_rn(__fdiv_rn(Af[0], s), __double2float_rn(p.min_p));
        const int q = block_find_nth(ncand, 0, [&](int j) { return j >= 1 && pval(j) < thr; }, S);
        if (q >= 0) nlim = q;
      }
      // top-p (sampler.nim:103-108) and the draw total (:115-116)
      int n;
      float total;
      if (p.top_p > 0.0 && p.top_p < 1.0) {
        const double tp = p.top_p;
        ScanResult r = exact_scan<FT_THREADS, FT_EPT, false>(
            0, nlim, 0.0f, pval, [tp](float v) { return (double)v >= tp; }, true, false, S.scan);
        n = (r.stop_j >= 0) ? r.stop_j + 1 : nlim;
        total = r.v;
      } else {
        n = nlim;
        total = exact_scan<FT_THREADS, FT_EPT, false>(0, nlim, 0.0f, pval, nostop, false, true, S.scan).v;
      }
      // draw (sampler.nim:117-121)
      const float r0 = __fmul_rn(__double2float_rn(u_draw), total);
      ScanResult d = exact_scan<FT_THREADS, FT_EPT, true>(
          0, n, r0, pval, [](float v) { return v <= 0.0f; }, true, false, S.scan);
      pos = (d.stop_j >= 0) ? d.stop_j : n - 1;
      prob = pval(pos);
    }

    // 4. token id of the drawn position
    const uint32_t kpos = B[pos];
    const int lb = lower_bound_u32(B, V, kpos);
    const int o = pos - lb;
    int id;
    if (!heap) {
      id = block_find_nth(V, o, [&](int i) { return orig[i] == kpos; }, S);
    } else {
      const uint32_t tkey = B[ncand - 1];
      if (kpos != tkey) {
        const int g = upper_bound_u32(B, V, kpos) - lb;
        id = block_find_nth(V, g - 1 - o, [&](int i) { return orig[i] == kpos; }, S);
      } else {
        const int tau = block_find_nth(V, ncand - 1, [&](int i) { return orig[i] <= tkey; }, S);
        const int mt = block_count(tau + 1, [&](int i) { return orig[i] == tkey; }, S);
        id = block_find_nth(tau + 1, mt - 1 - o, [&](int i) { return orig[i] == tkey; }, S);
      }
    }
    if (tid == 0) {
      a.out_ids[row] = id;
      if (a.out_probs) a.out_probs[row] = prob;
    }
    __syncthreads();
  }
}

cudaError_t launch_full(const BatchArgs& a, uint32_t* scratch, int vpad, int slots,
                        cudaStream_t stream) {
  const size_t smem = full_smem_bytes(a.V);
  cudaError_t e = cudaFuncSetAttribute(full_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  full_kernel<<<slots, FT_THREADS, smem, stream>>>(a, scratch, vpad);
  return cudaGetLastError();
}

}  // namespace nls
