// nls_light.cu -- streaming kernel for greedy rows and top-k rows (k <= 256).
//
// One thread-block cluster per row (cluster size C = 1..16). CTA c streams the
// chunk [c*chunk, (c+1)*chunk) of the row from HBM exactly once with 16-byte
// loads, applying the row's penalties and bias (a bitmap marks the patched
// positions) and the temperature on the fly (src/nimllm/sampler.nim:63-81).
//  - greedy rows (temperature <= 0): argmax with the reference's strict `>`
//    (sampler.nim:45-49, 77-78);
//  - top-k rows: every element whose order key reaches a running threshold
//    is appended to a shared-memory candidate buffer; when the buffer fills,
//    a radix select over it raises the threshold to the current k-th largest
//    key, keeping all ties. At the end each CTA holds a superset of its
//    chunk's top-k, including every element equal to the row's k-th largest
//    value, which the reference's heap tie rule needs (sampler.nim:88-95).
// CTA 0 then gathers the candidates of the cluster through distributed
// shared memory, selects the reference's exact survivor set, sorts it in heap
// output order (value descending, ties by index descending), and one warp
// replays softmax, top-p, min-p and the draw with the reference's sequential
// fp32 loops (sampler.nim:98-121). Rows whose ties overflow the buffers are
// handed to the full-sort kernel.
#include <cooperative_groups.h>

#include "nls_common.cuh"
#include "nls_kernels.h"

namespace cg = cooperative_groups;

namespace nls {

constexpr int LT_THREADS = 512;
constexpr int LT_UNROLL = 2;                          // float4 loads in flight per thread
constexpr int LT_TILE = LT_THREADS * LT_UNROLL * 4;   // elements per tile
constexpr int LT_SLOT = 512;                          // candidates a CTA hands to the merge
constexpr int LT_CAP = LT_SLOT + LT_TILE;             // candidate buffer
constexpr int LT_HASH_LOG2 = 10;
constexpr int LT_PER_THREAD = (LT_CAP + LT_THREADS - 1) / LT_THREADS;

struct LightShared {
  uint32_t cand_key[LT_CAP];
  int cand_idx[LT_CAP];
  int hkey[1 << LT_HASH_LOG2];
  int hcnt[1 << LT_HASH_LOG2];
  float hbias[1 << LT_HASH_LOG2];
  int hflag[1 << LT_HASH_LOG2];
  unsigned long long sortbuf[kLightKMax];
  float tval[kLightKMax];
  float pval[kLightKMax];
  uint32_t hist[256];
  uint32_t sel[4];
  float gbest_w[LT_THREADS / 32];
  int gidx_w[LT_THREADS / 32];
  // published for the cluster merge
  int ncand;
  int nan;
  int overflow;
  int nan0;
  float gbest;
  int gidx;
  // scratch
  uint32_t thr;
  int counter, patch_overflow, dup;
  int cnt_gt, cnt_ge, nsurv;
  int mtotal;
};

static_assert(sizeof(LightShared) % 16 == 0 || true, "");

size_t light_smem_bytes(int C, int chunk) {
  size_t bm_words = ((size_t)chunk + 31) / 32;
  bm_words = (bm_words + 3) & ~(size_t)3;
  size_t base = (sizeof(LightShared) + 15) & ~(size_t)15;
  size_t merge = (C > 1) ? (size_t)C * LT_SLOT * (sizeof(uint32_t) + sizeof(int)) : 0;
  return base + bm_words * 4 + merge;
}

// Keep the candidates whose key is >= the K-th largest; raises S.thr.
// Returns the new candidate count (the same value in every thread).
__device__ int light_compact(LightShared& S, uint32_t K) {
  const int tid = threadIdx.x;
  const int n = S.ncand;
  uint32_t t = block_select_kth_largest(
      n, K, [&](int i, uint32_t* k) { *k = S.cand_key[i]; return true; }, S.hist, S.sel);
  uint32_t keys[LT_PER_THREAD];
  int ids[LT_PER_THREAD];
#pragma unroll
  for (int r = 0; r < LT_PER_THREAD; ++r) {
    int i = tid + r * LT_THREADS;
    keys[r] = (i < n) ? S.cand_key[i] : 0u;
    ids[r] = (i < n) ? S.cand_idx[i] : -1;
  }
  __syncthreads();
  if (tid == 0) { S.ncand = 0; S.thr = t; }
  __syncthreads();
  const int lane = tid & 31;
#pragma unroll
  for (int r = 0; r < LT_PER_THREAD; ++r) {
    bool keep = ids[r] >= 0 && keys[r] >= t;
    unsigned m = __ballot_sync(0xffffffffu, keep);
    if (m) {
      int leader = __ffs(m) - 1;
      int basepos = 0;
      if (lane == leader) basepos = atomicAdd(&S.ncand, __popc(m));
      basepos = __shfl_sync(0xffffffffu, basepos, leader);
      if (keep) {
        int pos = basepos + __popc(m & lanemask_lt());
        S.cand_key[pos] = keys[r];
        S.cand_idx[pos] = ids[r];
      }
    }
  }
  __syncthreads();
  const int nnew = S.ncand;
  __syncthreads();
  return nnew;
}

__global__ void __launch_bounds__(LT_THREADS)
light_kernel(BatchArgs a, int C, int chunk) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  LightShared& S = *reinterpret_cast<LightShared*>(smem_raw);
  const size_t base_bytes = (sizeof(LightShared) + 15) & ~(size_t)15;
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem_raw + base_bytes);
  int bm_words = (chunk + 31) / 32;
  bm_words = (bm_words + 3) & ~3;
  uint32_t* mkey = bitmap + bm_words;
  int* midx = reinterpret_cast<int*>(mkey + C * LT_SLOT);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int crank = (C > 1) ? (int)cg::this_cluster().block_rank() : 0;
  const int row = blockIdx.x / C;
  const int V = a.V;

  nls_row_params p{};
  int64_t K64 = V;
  int mode = kModeGreedy;
  if (!a.argmax_only) {
    p = a.params[row];
    mode = row_mode(p, V, &K64);
  }
  if (mode == kModeFull) {
    if (crank == 0 && tid == 0) {
      int w = atomicAdd(a.full_count, 1);
      a.full_list[w] = row;
    }
    return;
  }
  if (mode == kModeTopK && a.uniforms == nullptr) {
    if (crank == 0 && tid == 0) {
      a.out_ids[row] = -1;
      record_status(a.status, NLS_ERR_INVALID_ARG);
    }
    return;
  }
  const uint32_t K = (uint32_t)K64;
  const int lo = min(V, crank * chunk);
  const int hi = min(V, lo + chunk);
  const int len = hi - lo;

  PatchTable T{S.hkey, S.hcnt, S.hbias, S.hflag, bitmap, LT_HASH_LOG2, lo, hi};
  int npatch = 0;
  if (!a.argmax_only) npatch = build_patches(a, row, p, T, &S.counter, &S.patch_overflow, &S.dup);
  if (tid == 0) {
    S.ncand = 0;
    S.thr = 0u;
    S.nan = 0;
    S.overflow = 0;
    S.nan0 = 0;
  }
  __syncthreads();
  const bool bad_patch = (!a.argmax_only) && (S.patch_overflow || S.dup);

  const float* rowp = a.logits + (int64_t)row * a.ld + lo;
  const bool vec = ((reinterpret_cast<uintptr_t>(rowp) & 15u) == 0);
  const float invT = (mode == kModeTopK) ? __double2float_rn(__ddiv_rn(1.0, p.temperature)) : 1.0f;

  bool anynan = false;
  float gb = 0.0f;
  int gi = INT_MAX;  // greedy: best non-NaN value and its first index
  uint32_t thr = 0u;
  bool overflow = false;

  for (int t0 = 0; t0 < len; t0 += LT_TILE) {
    if (mode == kModeTopK) {
      // every thread reads the count before any thread appends again
      int nc = S.ncand;
      __syncthreads();
      if (nc > LT_CAP - LT_TILE) {
        nc = light_compact(S, K);
        if (nc > LT_CAP - LT_TILE) { overflow = true; break; }
      }
      thr = S.thr;
    }
    float vals[LT_UNROLL][4];
#pragma unroll
    for (int u = 0; u < LT_UNROLL; ++u) {
      const int off = t0 + (u * LT_THREADS + tid) * 4;
      if (vec && off + 4 <= len) {
        float4 v4 = __ldcs(reinterpret_cast<const float4*>(rowp + off));
        vals[u][0] = v4.x; vals[u][1] = v4.y; vals[u][2] = v4.z; vals[u][3] = v4.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) vals[u][e] = (off + e < len) ? __ldcs(rowp + off + e) : 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < LT_UNROLL; ++u) {
      const int off = t0 + (u * LT_THREADS + tid) * 4;
      uint32_t pbits = 0u;
      if (npatch > 0 && off < len) pbits = (T.bits[off >> 5] >> (off & 31)) & 0xFu;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const bool valid = (off + e < len);
        float x = vals[u][e];
        const int gidx = lo + off + e;
        if (valid && (pbits >> e) & 1u) {
          int slot = patch_find(T, gidx);
          if (slot >= 0) x = patch_apply(x, T, slot, p);
        }
        if (mode == kModeGreedy) {
          if (valid) {
            if (gidx == 0 && x != x) S.nan0 = 1;
            if (!(x != x) && (gi == INT_MAX || x > gb)) { gb = x; gi = gidx; }
          }
        } else {
          const float y = __fmul_rn(x, invT);
          anynan |= valid && (y != y);
          const uint32_t key = fkey(y);
          const bool pass = valid && key >= thr;
          unsigned m = __ballot_sync(0xffffffffu, pass);
          if (m) {
            int leader = __ffs(m) - 1;
            int basepos = 0;
            if (lane == leader) basepos = atomicAdd(&S.ncand, __popc(m));
            basepos = __shfl_sync(0xffffffffu, basepos, leader);
            if (pass) {
              int pos = basepos + __popc(m & lanemask_lt());
              S.cand_key[pos] = key;
              S.cand_idx[pos] = gidx;
            }
          }
        }
      }
    }
    __syncthreads();
  }

  // ---- per-CTA results -------------------------------------------------
  if (mode == kModeTopK) {
    if (anynan) atomicExch(&S.nan, 1);
    if (!overflow && S.ncand > (int)K) (void)light_compact(S, K);
    __syncthreads();
    if (tid == 0) {
      if (overflow || bad_patch || (C > 1 && S.ncand > LT_SLOT)) S.overflow = 1;
    }
  } else {
    // block argmax reduction: larger value wins, ties keep the lower index
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      float ob = __shfl_down_sync(0xffffffffu, gb, off);
      int oi = __shfl_down_sync(0xffffffffu, gi, off);
      if (oi != INT_MAX && (gi == INT_MAX || ob > gb || (ob == gb && oi < gi))) { gb = ob; gi = oi; }
    }
    if (lane == 0) { S.gbest_w[warp] = gb; S.gidx_w[warp] = gi; }
    __syncthreads();
    if (tid == 0) {
      float b = 0.0f;
      int bi = INT_MAX;
      for (int w = 0; w < LT_THREADS / 32; ++w) {
        float ob = S.gbest_w[w];
        int oi = S.gidx_w[w];
        if (oi != INT_MAX && (bi == INT_MAX || ob > b || (ob == b && oi < bi))) { b = ob; bi = oi; }
      }
      S.gbest = b;
      S.gidx = bi;
      if (bad_patch) S.overflow = 1;
    }
  }
  __syncthreads();

  // ---- cluster merge into CTA 0 ----------------------------------------
  uint32_t* keys = S.cand_key;
  int* ids = S.cand_idx;
  int nm = 0;
  int any_nan = 0, any_over = 0, nan0 = 0;
  float gbest = 0.0f;
  int gidx = INT_MAX;
  if (C > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (crank == 0) {
      int offs = 0;
      for (int r = 0; r < C; ++r) {
        LightShared* R = cluster.map_shared_rank(&S, r);
        const int nr = R->ncand;
        any_nan |= R->nan;
        any_over |= R->overflow;
        nan0 |= R->nan0;
        const float ob = R->gbest;
        const int oi = R->gidx;
        if (oi != INT_MAX && (gidx == INT_MAX || ob > gbest || (ob == gbest && oi < gidx))) {
          gbest = ob;
          gidx = oi;
        }
        if (mode == kModeTopK && !any_over) {
          const int ncopy = nr < LT_SLOT ? nr : LT_SLOT;
          for (int i = tid; i < ncopy; i += LT_THREADS) {
            mkey[offs + i] = R->cand_key[i];
            midx[offs + i] = R->cand_idx[i];
          }
          offs += ncopy;
        }
      }
      nm = offs;
    }
    cluster.sync();
    if (crank != 0) return;
    keys = mkey;
    ids = midx;
  } else {
    nm = S.ncand;
    any_nan = S.nan;
    any_over = S.overflow;
    nan0 = S.nan0;
    gbest = S.gbest;
    gidx = S.gidx;
  }
  (void)gbest;

  // ---- finish (CTA 0) ---------------------------------------------------
  if (any_over) {
    if (tid == 0) {
      if (a.argmax_only || mode == kModeGreedy) {
        // a greedy row only overflows through its patch table
        a.out_ids[row] = -1;
        record_status(a.status, NLS_ERR_CAPACITY);
      } else {
        int w = atomicAdd(a.full_count, 1);
        a.full_list[w] = row;
      }
    }
    return;
  }
  if (mode == kModeGreedy) {
    if (tid == 0) {
      a.out_ids[row] = nan0 ? 0 : (gidx == INT_MAX ? 0 : gidx);
      if (a.out_probs) a.out_probs[row] = 1.0f;
    }
    return;
  }
  if (any_nan) {
    if (tid == 0) {
      a.out_ids[row] = -1;
      if (a.out_probs) a.out_probs[row] = 0.0f;
      record_status(a.status, NLS_ERR_NAN_LOGITS);
    }
    return;
  }

  // exact survivor set of the reference heap (see block comment at top)
  const uint32_t t = block_select_kth_largest(
      nm, K, [&](int i, uint32_t* k) { *k = keys[i]; return true; }, S.hist, S.sel);
  if (tid == 0) { S.cnt_gt = 0; S.cnt_ge = 0; S.nsurv = 0; }
  __syncthreads();
  {
    int gt = 0, ge = 0;
    for (int i = tid; i < nm; i += LT_THREADS) {
      gt += keys[i] > t;
      ge += keys[i] >= t;
    }
    gt = __reduce_add_sync(0xffffffffu, gt);
    ge = __reduce_add_sync(0xffffffffu, ge);
    if (lane == 0) { atomicAdd(&S.cnt_gt, gt); atomicAdd(&S.cnt_ge, ge); }
  }
  __syncthreads();
  const int cgt = S.cnt_gt, cge = S.cnt_ge;
  uint32_t tau = 0xffffffffu, rho = 0u;
  if (cge != (int)K) {
    // tau: index of the K-th element (in index order) with value >= t;
    // survivors among the ties are the (K - cgt) highest indices <= tau.
    tau = ~block_select_kth_largest(
        nm, K,
        [&](int i, uint32_t* k) {
          if (keys[i] >= t) { *k = ~(uint32_t)ids[i]; return true; }
          return false;
        },
        S.hist, S.sel);
    rho = block_select_kth_largest(
        nm, K - (uint32_t)cgt,
        [&](int i, uint32_t* k) {
          if (keys[i] == t && (uint32_t)ids[i] <= tau) { *k = (uint32_t)ids[i]; return true; }
          return false;
        },
        S.hist, S.sel);
  }
  int n64 = 32;
  while (n64 < (int)K) n64 <<= 1;
  for (int i = tid; i < n64; i += LT_THREADS) S.sortbuf[i] = 0ull;
  __syncthreads();
  for (int i = tid; i < nm; i += LT_THREADS) {
    const uint32_t k = keys[i];
    const uint32_t id = (uint32_t)ids[i];
    const bool keep = (k > t) || (k == t && id >= rho && id <= tau);
    if (keep) {
      int pos = atomicAdd(&S.nsurv, 1);
      if (pos < kLightKMax) S.sortbuf[pos] = ((unsigned long long)k << 32) | id;
    }
  }
  __syncthreads();
  block_bitonic_desc(S.sortbuf, n64);

  // ---- replay of sampler.nim:98-121 by one warp ----------------------------
  if (warp == 0) {
    const int n = (int)K;
    for (int i = lane; i < n; i += 32) S.tval[i] = fkey_inv((uint32_t)(S.sortbuf[i] >> 32));
    __syncwarp();
    const float mx = S.tval[0];
    for (int i = lane; i < n; i += 32) S.tval[i] = ref_expf(__fsub_rn(S.tval[i], mx));
    __syncwarp();
    float s = 0.0f;
    if (lane == 0)
      for (int i = 0; i < n; ++i) s = __fadd_rn(s, S.tval[i]);
    s = __shfl_sync(0xffffffffu, s, 0);
    for (int i = lane; i < n; i += 32) S.pval[i] = __fdiv_rn(S.tval[i], s);
    __syncwarp();
    if (lane == 0) {
      int nn = n;
      if (p.top_p > 0.0 && p.top_p < 1.0) {
        float cum = 0.0f;
        for (int i = 0; i < nn; ++i) {
          cum = __fadd_rn(cum, S.pval[i]);
          if ((double)cum >= p.top_p) { nn = i + 1; break; }
        }
      }
      if (p.min_p > 0.0) {
        const float thrp = __fmul_rn(S.pval[0], __double2float_rn(p.min_p));
        int m = 1;
        while (m < nn && S.pval[m] >= thrp) ++m;
        nn = m;
      }
      float total = 0.0f;
      for (int i = 0; i < nn; ++i) total = __fadd_rn(total, S.pval[i]);
      float r = __fmul_rn(__double2float_rn(a.uniforms[row]), total);
      int pos = nn - 1;
      for (int i = 0; i < nn; ++i) {
        r = __fsub_rn(r, S.pval[i]);
        if (r <= 0.0f) { pos = i; break; }
      }
      a.out_ids[row] = (int64_t)(uint32_t)(S.sortbuf[pos] & 0xffffffffull);
      if (a.out_probs) a.out_probs[row] = S.pval[pos];
    }
  }
}

cudaError_t launch_light(const BatchArgs& a, int C, int chunk, cudaStream_t stream) {
  const size_t smem = light_smem_bytes(C, chunk);
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(light_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(light_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(a.rows * C), 1, 1);
  cfg.blockDim = dim3(LT_THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, light_kernel, a, C, chunk);
}

}  // namespace nls
