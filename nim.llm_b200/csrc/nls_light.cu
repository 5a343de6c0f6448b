// nls_light.cu -- streaming kernel for greedy rows and top-k rows (k <= 256).
//
// One thread-block cluster per row (cluster size C = 1..16). CTA c owns the
// chunk [c*chunk, (c+1)*chunk) of the row and reads it from HBM exactly once:
// one thread issues bulk copies (cp.async.bulk, 16 or 32 KB stages, a few in
// flight, mbarrier completion) into a shared-memory ring while the block
// consumes earlier stages. On the fly it applies the row's penalties and bias
// (a bitmap marks the patched float4 groups) and the temperature
// (src/nimllm/sampler.nim:63-81):
//  - greedy rows (temperature <= 0): argmax with the reference's strict `>`
//    (sampler.nim:45-49, 77-78);
//  - top-k rows: the first stage sets a threshold (a lower bound of its k-th
//    largest order key); every later element at or above the running
//    threshold is appended to a shared candidate buffer, and when the buffer
//    passes half full a radix select raises the threshold again. The
//    threshold never exceeds the chunk's true k-th largest value, so each CTA
//    ends with a superset of its chunk's top-k that contains every element
//    equal to the row's k-th largest value -- what the reference heap's tie
//    rule needs (sampler.nim:88-95).
// CTA 0 gathers the cluster's candidates through distributed shared memory,
// selects the reference's exact survivor set, sorts it in heap output order
// (value descending, ties by index descending), and one warp replays softmax,
// top-p, min-p and the draw with the reference's sequential fp32 loops
// (sampler.nim:98-121). Rows whose candidates overflow the buffers, or whose
// penalty window overflows the patch table, are handed to the full-sort
// kernel.
#include <cooperative_groups.h>

#include <atomic>
#include <type_traits>

#include "nls_common.cuh"
#include "nls_kernels.h"
#include "nls_tma.cuh"

namespace cg = cooperative_groups;

namespace nls {

constexpr int LT_THREADS = 256;
// Bulk-copy ring shapes (floats per stage, stages in flight); the kernel is
// instantiated for both. A CTA that streams a whole row (one CTA per row,
// batches of many rows) uses two 32 KB stages: per-stage costs (the mbarrier
// wait, the block barrier, the refill) are then paid per 8192 logits;
// measured on config 4 against 4 x 16 KB (2.62 TB/s), 6 x 12 KB (2.30),
// 3 x 24 KB (3.12) and 3 x 32 KB at one CTA per SM (2.12): 3.46 TB/s. A row
// split over a cluster (a few rows: each CTA holds a few thousand logits)
// uses four 16 KB stages, so its copies and its compute overlap.
constexpr int LT_STAGE_ROW = 8192, LT_NSTAGE_ROW = 2;
constexpr int LT_STAGE_SPLIT = 4096, LT_NSTAGE_SPLIT = 4;
// optimistic threshold: at least this many of stage 0's elements above it,
// and about this many of the whole chunk's expected above it
// (a threshold above the row's k-th value sends the row to the full-sort
// kernel, which costs about 1 ms at V = 151936: with an 8192-logit stage 0,
// floors of 8 and 64 let one config-4 row in 8192 through)
constexpr int LT_MFLOOR = 16;
constexpr int LT_CHUNK_FLOOR = 128;
constexpr int LT_CAP = 2048;                          // candidate buffer
constexpr int LT_LIMIT = LT_CAP / 2;                  // compact above this after a stage
constexpr int LT_SLOT = LT_LIMIT;                     // candidates a CTA hands to the merge
constexpr int LT_CMAX = 16;                           // CTAs per row at most (clusters above 8 are non-portable)
// a CTA's merge slot: halved above 8 CTAs so that CTA 0's merge buffer fits
__host__ __device__ constexpr int lt_slot(int C) { return C > 8 ? LT_SLOT / 2 : LT_SLOT; }
constexpr int LT_HASH_LOG2 = 10;
constexpr int LT_PER_THREAD = LT_CAP / LT_THREADS;
constexpr int LT_GSHIFT = 2;                          // one patch bit per float4 group
template <int LT_STAGE, int LT_NSTAGE>
struct LightShared {
  static_assert(LT_STAGE % (4 * LT_THREADS) == 0, "a stage splits into whole float4 groups");
  float ring[LT_NSTAGE][LT_STAGE];
  uint64_t full_bar[LT_NSTAGE];
  uint32_t cand_key[LT_CAP];
  int cand_idx[LT_CAP];
  int hkey[1 << LT_HASH_LOG2];
  int hcnt[1 << LT_HASH_LOG2];
  float hbias[1 << LT_HASH_LOG2];
  int hflag[1 << LT_HASH_LOG2];
  unsigned long long sortbuf[kLightKMax];
  float tval[kLightKMax];
  float pval[kLightKMax];
  float seq[kLightKMax];
  uint32_t hist[256];
  uint32_t sel[4];
  float gbest_w[LT_THREADS / 32];
  int gidx_w[LT_THREADS / 32];
  // published for the cluster merge
  uint32_t thr_pub;
  int ncand;
  int nan;
  int overflow;
  int nan0;
  int failed;
  float gbest;
  int gidx;
  // scratch
  uint32_t thr;
  int counter, patch_overflow, dup;
  int cnt_gt, cnt_ge, nsurv;
  // cluster merge: each CTA's summary, pushed into every CTA of the cluster
  struct MergeRec {
    int ncand;
    int flags;  // 1 nan, 2 overflow, 4 failed, 8 nan at index 0
    uint32_t thr;
    float gbest;
    int gidx;
  } rec[LT_CMAX];
};

static int bitmap_words_host(int chunk) {
  int groups = (chunk + (1 << LT_GSHIFT) - 1) >> LT_GSHIFT;
  int w = (groups + 31) >> 5;
  return (w + 3) & ~3;
}

template <int LT_STAGE, int LT_NSTAGE>
size_t light_smem_bytes_t(int C, int chunk) {
  size_t base = (sizeof(LightShared<LT_STAGE, LT_NSTAGE>) + 15) & ~(size_t)15;
  size_t merge = (C > 1) ? (size_t)C * lt_slot(C) * (sizeof(uint32_t) + sizeof(int)) : 0;
  return base + (size_t)bitmap_words_host(chunk) * 4 + merge;
}

// Keep the candidates whose key is at least a lower bound of the K-th largest
// (its top 16 bits, or all 32 when that leaves too many); raises S.thr.
// Returns the new candidate count (the same value in every thread).
template <class SharedT>
__device__ int light_compact(SharedT& S, uint32_t K) {
  const int tid = threadIdx.x;
  const int n = S.ncand;
  auto get = [&](int i, uint32_t* k) { *k = S.cand_key[i]; return S.cand_idx[i] >= 0; };
  uint32_t t = block_select_kth_largest(n, K, get, S.hist, S.sel, 2);
  if ((int)S.sel[2] > LT_LIMIT / 2) t = block_select_kth_largest(n, K, get, S.hist, S.sel, 4);
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

template <int LT_STAGE, int LT_NSTAGE>
__global__ void __launch_bounds__(LT_THREADS, 2)
light_kernel(BatchArgs a, int C, int chunk) {
  using LightShared = nls::LightShared<LT_STAGE, LT_NSTAGE>;
  constexpr int LT_GROUPS = LT_STAGE / 4 / LT_THREADS;  // float4 groups per thread per stage
  // a full-sort launch that depends on this grid may be scheduled now; it
  // waits (griddepcontrol.wait) for this grid's completion before reading
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  LightShared& S = *reinterpret_cast<LightShared*>(smem_raw);
  const size_t base_bytes = (sizeof(LightShared) + 15) & ~(size_t)15;
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(smem_raw + base_bytes);
  const int bm_words = [&] {
    int groups = (chunk + (1 << LT_GSHIFT) - 1) >> LT_GSHIFT;
    int w = (groups + 31) >> 5;
    return (w + 3) & ~3;
  }();
  uint32_t* mkey = bitmap + bm_words;
  const int slot = lt_slot(C);
  int* midx = reinterpret_cast<int*>(mkey + C * slot);

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
    if (!a.skip_full && crank == 0 && tid == 0) {
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
  const float* rowp = a.logits + (int64_t)row * a.ld + lo;
  const bool tma = ((reinterpret_cast<uintptr_t>(rowp) & 15u) == 0);
  const int nvec = tma ? (len & ~3) : 0;                   // elements fetched by bulk copies
  const int nst = (len + LT_STAGE - 1) / LT_STAGE;         // stages over the whole chunk
  auto stage_bytes = [&](int si) -> uint32_t {
    int b = nvec - si * LT_STAGE;
    b = b < LT_STAGE ? b : LT_STAGE;
    return b > 0 ? (uint32_t)b * 4u : 0u;
  };

  if (tid == 0) {
    for (int s = 0; s < LT_NSTAGE; ++s) mbar_init(&S.full_bar[s], 1);
    fence_mbar_init();
    S.ncand = 0;
    S.thr = 0u;
    S.nan = 0;
    S.overflow = 0;
    S.nan0 = 0;
    S.failed = 0;
  }
  __syncthreads();
  if (tid == 0 && tma) {
    for (int s = 0; s < LT_NSTAGE && s < nst; ++s) {
      const uint32_t b = stage_bytes(s);
      if (b) {
        mbar_arrive_expect_tx(&S.full_bar[s], b);
        bulk_copy_g2s_hint(S.ring[s], rowp + s * LT_STAGE, b, &S.full_bar[s], l2_policy_evict_first());
      }
    }
  }

  PatchTable T{S.hkey, S.hcnt, S.hbias, S.hflag, bitmap, LT_HASH_LOG2, lo, hi, LT_GSHIFT};
  int npatch = 0;
  if (!a.argmax_only)
    npatch = build_patches(a, row, p, T, rowp, &S.counter, &S.patch_overflow, &S.dup, false);
  const bool bad_patch = (!a.argmax_only) && (S.patch_overflow || S.dup);
  // Patched positions (penalty window, bias) get their final value once,
  // after the stream: their logits come by 4-byte asynchronous copies into
  // their slots that land while the row streams (the table's build waits
  // for no logit); the streaming loops leave those positions out and they
  // rejoin the candidates after.
  if (npatch > 0 && !bad_patch) {
    constexpr int HS = 1 << LT_HASH_LOG2;
    for (int i = tid; i < HS; i += LT_THREADS) {
      const int k = T.key[i];
      if (k >= 0) cp_async4(&T.bias[i], rowp + (k - lo));
    }
    cp_async_commit();
  }
  const float invT = (mode == kModeTopK) ? __double2float_rn(__ddiv_rn(1.0, p.temperature)) : 1.0f;

  float gb = 0.0f;
  int gi = INT_MAX;        // greedy: best non-NaN value and its first index
  uint32_t thr = 0u;
  float thrf = -INFINITY;  // fkey_inv(thr); -inf accepts everything but NaN
  bool overflow = false;
  int my_max = 0;          // largest candidate count this thread's appends produced

  // the four elements of float4 group g (chunk offset `off`) of the stage in `buf`
  auto load_group = [&](int buf, int g, int off, bool whole, float (&x)[4], bool (&valid)[4]) {
    if (whole) {
      const float4 q = *reinterpret_cast<const float4*>(&S.ring[buf][4 * g]);
      x[0] = q.x; x[1] = q.y; x[2] = q.z; x[3] = q.w;
#pragma unroll
      for (int e = 0; e < 4; ++e) valid[e] = true;
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        valid[e] = off + e < len;
        x[e] = !valid[e] ? 0.0f : (off + e < nvec ? S.ring[buf][4 * g + e] : __ldcs(rowp + off + e));
      }
    }
  };
  // Append the passing elements of one float4 group (warp-aggregated). A
  // store past the buffer is dropped; the overflow is detected afterwards.
  auto append4 = [&](const float (&y)[4], const bool (&pass)[4], int gidx0) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const unsigned m = __ballot_sync(0xffffffffu, pass[e]);
      if (m) {
        const int leader = __ffs(m) - 1;
        int basepos = 0;
        if (lane == leader) basepos = atomicAdd(&S.ncand, __popc(m));
        basepos = __shfl_sync(0xffffffffu, basepos, leader);
        const int end = basepos + __popc(m);
        my_max = end > my_max ? end : my_max;
        if (pass[e]) {
          const int pos = basepos + __popc(m & lanemask_lt());
          if (pos < LT_CAP) {
            S.cand_key[pos] = fkey(y[e]);
            S.cand_idx[pos] = gidx0 + e;
          }
        }
      }
    }
  };

  int si = 0;
  for (; si < nst; ++si) {
    const int sbase = si * LT_STAGE;
    const int buf = si % LT_NSTAGE;
    bool failed_local = false;
    if (stage_bytes(si) > 0 &&
        !mbar_wait_bounded(&S.full_bar[buf], (uint32_t)(si / LT_NSTAGE) & 1u, a.wait_ns)) {
      failed_local = true;
      S.failed = 1;
    }
    const bool whole = (sbase + LT_STAGE <= nvec);  // every element of the stage is in the ring

    if (mode == kModeTopK && si == 0) {
      // initial threshold: a lower bound of the K-th largest key of stage 0
      const int n0 = min(len, LT_STAGE);
      if (n0 > (int)K) {
        auto key0 = [&](int i, uint32_t* k) {
          const float x = (i < nvec) ? S.ring[0][i] : __ldcs(rowp + i);
          const float y = __fmul_rn(x, invT);
          if (y != y) return false;  // a NaN is never a candidate (see above)
          *k = fkey(y);
          return true;
        };
        // Optimistic threshold: (a lower bound of) the m-th largest key of
        // stage 0, with m chosen so that about max(128, 2K) elements of the
        // whole chunk are expected above it. It is verified at the merge: the
        // candidates are complete iff every chunk's threshold is at most the
        // row's K-th largest candidate; otherwise the row goes to the
        // full-sort kernel.
        int m = (int)(((long long)2 * K * n0 + len - 1) / len);
        const int m_floor = (int)(((long long)LT_CHUNK_FLOOR * n0 + len - 1) / len);
        m = max(m, max(m_floor, LT_MFLOOR));
        m = min(m, n0);
        constexpr int NW = LT_THREADS / 32;
        const int r = (2 * m + NW - 1) / NW;  // per-warp rank; j = ceil(m / r) <= NW / 2 + 1
        if (r <= 32) {
          // Each warp sorts its 32 thread maxima (register bitonic network)
          // and publishes its r-th largest; the j-th largest of those, with
          // j = ceil(m / r), has at least j * r >= m elements of the stage at
          // or above it, so it is a lower bound of the stage's m-th largest
          // key.
          const int jsel = (m + r - 1) / r;
          uint32_t v = 0u;  // 0 sorts last: a thread without keys bounds nothing
          if (n0 == LT_STAGE && nvec >= LT_STAGE) {
            // a whole first stage in the ring: float4 reads
#pragma unroll
            for (int j = 0; j < LT_GROUPS; ++j) {
              const float4 q = reinterpret_cast<const float4*>(S.ring[0])[tid + j * LT_THREADS];
              const float xs[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float y = __fmul_rn(xs[e], invT);
                const uint32_t k = fkey(y);
                v = (y == y && k > v) ? k : v;
              }
            }
          } else {
            for (int i = tid; i < n0; i += LT_THREADS) {
              uint32_t k;
              if (key0(i, &k)) v = k > v ? k : v;
            }
          }
#pragma unroll
          for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
            for (int j = kk >> 1; j > 0; j >>= 1) {
              const uint32_t o = __shfl_xor_sync(0xffffffffu, v, j);
              const bool desc_block = (lane & kk) == 0 || kk == 32;
              const bool lower = (lane & j) == 0;
              v = (desc_block == lower) ? (v > o ? v : o) : (v < o ? v : o);
            }
          }
          const uint32_t wr = __shfl_sync(0xffffffffu, v, r - 1);
          if (lane == 0) S.cand_key[warp] = wr;
          __syncthreads();
          // the jsel-th largest of the NW published values (ties counted)
          uint32_t tm = 0u;
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            const uint32_t x = S.cand_key[w];
            int above = 0, ge = 0;
#pragma unroll
            for (int w2 = 0; w2 < NW; ++w2) {
              above += S.cand_key[w2] > x;
              ge += S.cand_key[w2] >= x;
            }
            if (above < jsel && ge >= jsel) tm = x;
          }
          thr = tm;
          __syncthreads();
        } else {
          thr = block_select_kth_largest(n0, (uint32_t)m, key0, S.hist, S.sel, 2);
          if ((int)S.sel[2] < m) thr = 0u;
        }
        thrf = key_threshold_float(thr);
      }
    }

    (void)whole;
    // Hot paths: the stage's whole float4 groups in the ring (all of them
    // except in the last stage). All loads first.
    if (mode == kModeGreedy && sbase < nvec) {
      const int ngv = min(nvec - sbase, LT_STAGE) >> 2;  // same in every thread
      float4 q[LT_GROUPS];
#pragma unroll
      for (int j = 0; j < LT_GROUPS; ++j) {
        const int g = tid + j * LT_THREADS;
        q[j] = (g < ngv) ? reinterpret_cast<const float4*>(S.ring[buf])[g]
                         : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
      {
        // argmax: strict > in index order per thread; patched positions are
        // left out here and compared later with their patched values
#pragma unroll
        for (int j = 0; j < LT_GROUPS; ++j) {
          const int g = tid + j * LT_THREADS;
          const int off = sbase + 4 * g;
          const bool gpatch = npatch > 0 && g < ngv && patch_bit(T, off);
          const float x[4] = {q[j].x, q[j].y, q[j].z, q[j].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int gi2 = lo + off + e;
            const bool ok = g < ngv && !(gpatch && patch_find(T, gi2) >= 0);
            if (ok && gi2 == 0 && x[e] != x[e]) S.nan0 = 1;
            if (ok && !(x[e] != x[e]) && (gi == INT_MAX || x[e] > gb)) { gb = x[e]; gi = gi2; }
          }
        }
      }
    }
    if (mode == kModeTopK && sbase < nvec) {
      // top-k: per element one multiply, one compare and one NaN-propagating
      // max; the passing elements of the stage are appended with one warp
      // scan and one atomic. In the last stage, groups past the ring hold
      // -inf and are masked out (with an accept-all threshold, -inf, they
      // would otherwise pass); whole stages are compiled without the masks.
      const int ngv = min(nvec - sbase, LT_STAGE) >> 2;
      auto topk_stage = [&](auto partial_c) {
        constexpr bool PARTIAL = decltype(partial_c)::value;
        float4 q[LT_GROUPS];
#pragma unroll
        for (int j = 0; j < LT_GROUPS; ++j) {
          const int g = tid + j * LT_THREADS;
          if (PARTIAL)
            q[j] = (g < ngv) ? reinterpret_cast<const float4*>(S.ring[buf])[g]
                             : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
          else
            q[j] = reinterpret_cast<const float4*>(S.ring[buf])[g];
        }
        // pass bit 4j+e: element e of group j is at or above the threshold
        static_assert(4 * LT_GROUPS <= 32, "pass bits fit one word");
        uint32_t pm = 0u;
#pragma unroll
        for (int j = 0; j < LT_GROUPS; ++j) {
          const float x[4] = {q[j].x, q[j].y, q[j].z, q[j].w};
          const bool gv = !PARTIAL || (tid + j * LT_THREADS) < ngv;
          float y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            y[e] = __fmul_rn(x[e], invT);
            pm |= (gv && y[e] >= thrf) ? (1u << (4 * j + e)) : 0u;
          }
        }
        if (__any_sync(0xffffffffu, pm != 0u)) {
          const int cnt = __popc(pm);
          int incl = cnt;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
          }
          int base = 0;
          if (lane == 31) base = atomicAdd(&S.ncand, incl);
          base = __shfl_sync(0xffffffffu, base, 31);
          const int end = base + __shfl_sync(0xffffffffu, incl, 31);
          my_max = end > my_max ? end : my_max;
          int pos = base + incl - cnt;
          // only the passing elements, in (group, element) order; the value
          // is read again from the ring (still held until the stage barrier)
          while (pm) {
            const int bit = __ffs(pm) - 1;
            pm &= pm - 1u;
            const int rel = 4 * (tid + (bit >> 2) * LT_THREADS) + (bit & 3);  // offset in the stage
            const int off = sbase + rel;
            const float y = __fmul_rn(S.ring[buf][rel], invT);
            // a patched position rejoins later with its patched value
            const bool patched = npatch > 0 && patch_bit(T, off) && patch_find(T, lo + off) >= 0;
            if (pos < LT_CAP) {
              S.cand_key[pos] = patched ? 0u : fkey(y);
              S.cand_idx[pos] = patched ? -1 : lo + off;
            }
            ++pos;
          }
        }
      };
      if (ngv == LT_STAGE / 4) topk_stage(std::false_type{});
      else topk_stage(std::true_type{});
    }
    if (sbase < nvec && nvec < len && nvec < sbase + LT_STAGE) {
      // the chunk's last 1-3 elements (past the whole float4 groups) are not
      // in the ring: one thread each
      const int i = nvec + tid;
      if (i < len && i < sbase + LT_STAGE) {
        const float x = __ldcs(rowp + i);
        const bool excl = npatch > 0 && patch_bit(T, i) && patch_find(T, lo + i) >= 0;
        if (mode == kModeGreedy) {
          if (!excl && lo + i == 0 && x != x) S.nan0 = 1;
          if (!excl && !(x != x) && (gi == INT_MAX || x > gb)) { gb = x; gi = lo + i; }
        } else if (mode == kModeTopK) {
          const float y = __fmul_rn(x, invT);
          if (!excl && y >= thrf) {
            const int pos = atomicAdd(&S.ncand, 1);
            my_max = pos + 1 > my_max ? pos + 1 : my_max;
            if (pos < LT_CAP) {
              S.cand_key[pos] = fkey(y);
              S.cand_idx[pos] = lo + i;
            }
          }
        }
      }
    }
    if (sbase >= nvec) {
#pragma unroll 1
      for (int j = 0; j < LT_GROUPS; ++j) {
        const int g = tid + j * LT_THREADS;           // float4 group within the stage
        const int off = sbase + 4 * g;                // chunk-relative element offset
        float x[4];
        bool valid[4];
        load_group(buf, g, off, whole, x, valid);
        bool excl[4] = {false, false, false, false};
        if (npatch > 0 && off < len && patch_bit(T, off)) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int slot = valid[e] ? patch_find(T, lo + off + e) : -1;
            if (slot >= 0) excl[e] = true;  // (a greedy row's too: it competes after the stream)
          }
        }
        if (mode == kModeGreedy) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (valid[e] && !excl[e]) {
              if (lo + off + e == 0 && x[e] != x[e]) S.nan0 = 1;
              if (!(x[e] != x[e]) && (gi == INT_MAX || x[e] > gb)) { gb = x[e]; gi = lo + off + e; }
            }
          }
        } else {
          float y[4];
          bool pass[4];
          bool any = false;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            y[e] = __fmul_rn(x[e], invT);
            pass[e] = valid[e] && !excl[e] && y[e] >= thrf;
            any |= pass[e];
          }
          if (__any_sync(0xffffffffu, any)) append4(y, pass, lo + off);
        }
      }
    }
    // One barrier per stage: the ring slot is free, appends are complete, and
    // the block learns whether the candidate buffer needs a compaction
    // (S.ncand only grows within a stage, so "some append pushed it past the
    // limit" is "its final value is past the limit").
    bool need = false;
    int ncand_now = 0;
    if (__syncthreads_or(failed_local || my_max > LT_LIMIT)) {
      const int fail = S.failed;
      ncand_now = S.ncand;
      need = ncand_now > LT_LIMIT;
      __syncthreads();
      if (fail) break;
    }
    if (tid == 0 && si + LT_NSTAGE < nst) {
      const uint32_t b = stage_bytes(si + LT_NSTAGE);
      if (b) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&S.full_bar[buf], b);
        bulk_copy_g2s_hint(S.ring[buf], rowp + (si + LT_NSTAGE) * LT_STAGE, b, &S.full_bar[buf],
                           l2_policy_evict_first());
      }
    }
    if (mode == kModeTopK && need) {
      if (ncand_now > LT_CAP) { overflow = true; ++si; break; }  // some appends were dropped
      const int nn = light_compact(S, K);
      my_max = 0;
      if (nn > LT_LIMIT) { overflow = true; ++si; break; }
      thr = S.thr;
      thrf = key_threshold_float(thr);
    }
  }
  // Leave no bulk copy in flight into this CTA's shared memory (bounded by
  // the normal limit, whatever the call's: these copies are real and land).
  if (tid == 0 && tma) {
    for (int s2 = si; s2 < nst && s2 < si + LT_NSTAGE; ++s2) {
      if (stage_bytes(s2) && !mbar_wait_bounded(&S.full_bar[s2 % LT_NSTAGE], (uint32_t)(s2 / LT_NSTAGE) & 1u))
        S.failed = 1;
    }
  }
  __syncthreads();

  // The patched positions' logits have landed: their final values.
  if (npatch > 0 && !bad_patch) {
    cp_async_wait<0>();
    __syncthreads();
    precompute_patches(T, p);
  }

  // A NaN among the row's first K positions enters the reference's heap in
  // its first K pushes and never leaves it (sampler.nim:88-91); such a row
  // goes to the full-sort kernel, which runs the heap as written. A NaN
  // further on is never pushed (`x > h[0][0]` is false for it), and it never
  // passes the threshold tests either: it is simply left out.
  if (mode == kModeTopK && lo < (int)K) {
    const int e = min(hi, (int)K) - lo;
    bool nan_here = false;
    for (int i = tid; i < e; i += LT_THREADS) {
      float x = rowp[i];
      if (npatch > 0 && !bad_patch && patch_bit(T, i)) {
        const int slot = patch_find(T, lo + i);
        if (slot >= 0) x = patched_value(T, slot);
      }
      const float y = __fmul_rn(x, invT);
      nan_here |= (y != y);
    }
    if (__syncthreads_or(nan_here) && tid == 0) S.nan = 1;
  }

  // Patched positions rejoin the top-k candidates with their patched values.
  if (mode == kModeTopK && npatch > 0 && !bad_patch && !overflow && !S.failed) {
    constexpr int HS = 1 << LT_HASH_LOG2;
    for (int i0 = 0; i0 < HS; i0 += LT_THREADS) {
      const int i = i0 + tid;
      const int k = T.key[i];
      float y = 0.0f;
      bool pass = false;
      if (k >= 0) {
        y = __fmul_rn(patched_value(T, i), invT);
        pass = y >= thrf;
      }
      const unsigned m = __ballot_sync(0xffffffffu, pass);
      if (m) {
        const int leader = __ffs(m) - 1;
        int basepos = 0;
        if (lane == leader) basepos = atomicAdd(&S.ncand, __popc(m));
        basepos = __shfl_sync(0xffffffffu, basepos, leader);
        if (pass) {
          const int pos = basepos + __popc(m & lanemask_lt());
          if (pos < LT_CAP) {
            S.cand_key[pos] = fkey(y);
            S.cand_idx[pos] = k;
          }
        }
      }
    }
    __syncthreads();
    if (S.ncand > LT_CAP) overflow = true;
    __syncthreads();
  }

  // Patched positions of a greedy row compete with their patched values
  // (lowest index among equal values, as the reference's strict `>`).
  if (mode == kModeGreedy && npatch > 0 && !bad_patch) {
    constexpr int HS = 1 << LT_HASH_LOG2;
    for (int i0 = 0; i0 < HS; i0 += LT_THREADS) {
      const int i = i0 + tid;
      const int k = T.key[i];
      if (k >= 0) {
        const float x = patched_value(T, i);
        if (k == 0 && x != x) S.nan0 = 1;
        if (!(x != x) && (gi == INT_MAX || x > gb || (x == gb && k < gi))) { gb = x; gi = k; }
      }
    }
  }

  // ---- per-CTA results -------------------------------------------------
  if (mode == kModeTopK) {
    // Before the merge, keep only this chunk's top K (with all its ties at
    // the K-th key): the row's K-th largest key is at least every chunk's, so
    // nothing at or above it is dropped, and CTA 0 gets ~C*K candidates.
    if (!overflow && !S.failed && C > 1 && S.ncand > min(4 * (int)K, slot / 2)) (void)light_compact(S, K);
    __syncthreads();
    if (tid == 0) {
      if (overflow || bad_patch || (C > 1 && S.ncand > slot)) S.overflow = 1;
      S.thr_pub = thr;
    }
  } else {
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
  int any_nan = 0, any_over = 0, nan0 = 0, any_fail = 0;
  uint32_t thr_max = 0u;  // largest chunk threshold of the row
  float gbest = 0.0f;
  int gidx = INT_MAX;
  if (C > 1) {
    cg::cluster_group cluster = cg::this_cluster();
    // Push: thread j stores this CTA's summary into CTA j (remote stores do
    // not wait); after the barrier every CTA knows all counts locally.
    if (tid < C) {
      LightShared* R = cluster.map_shared_rank(&S, tid);
      typename LightShared::MergeRec m;
      m.ncand = S.ncand;
      m.flags = (S.nan ? 1 : 0) | (S.overflow ? 2 : 0) | (S.failed ? 4 : 0) | (S.nan0 ? 8 : 0);
      m.thr = S.thr_pub;
      m.gbest = S.gbest;
      m.gidx = S.gidx;
      R->rec[crank] = m;
    }
    cluster.sync();
    int offs = 0, myoff = 0;
    for (int r = 0; r < C; ++r) {
      const typename LightShared::MergeRec m = S.rec[r];
      any_nan |= m.flags & 1;
      any_over |= (m.flags >> 1) & 1;
      any_fail |= (m.flags >> 2) & 1;
      nan0 |= (m.flags >> 3) & 1;
      thr_max = max(thr_max, m.thr);
      if (m.gidx != INT_MAX && (gidx == INT_MAX || m.gbest > gbest || (m.gbest == gbest && m.gidx < gidx))) {
        gbest = m.gbest;
        gidx = m.gidx;
      }
      if (r == crank) myoff = offs;
      offs += m.ncand < slot ? m.ncand : slot;
    }
    if (mode == kModeTopK && !any_over) {
      // this CTA's candidates go to CTA 0's merge buffer at its offset
      uint32_t* mk0 = cluster.map_shared_rank(mkey, 0);
      int* mi0 = cluster.map_shared_rank(midx, 0);
      const int ncopy = S.ncand < slot ? S.ncand : slot;
      for (int i = tid; i < ncopy; i += LT_THREADS) {
        mk0[myoff + i] = S.cand_key[i];
        mi0[myoff + i] = S.cand_idx[i];
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
    any_fail = S.failed;
    nan0 = S.nan0;
    thr_max = S.thr_pub;
    gbest = S.gbest;
    gidx = S.gidx;
  }
  (void)gbest;

  // ---- finish (CTA 0) ---------------------------------------------------
  if (any_fail) {
    if (tid == 0) {
      a.out_ids[row] = -1;
      record_status(a.status, NLS_ERR_TIMEOUT);
    }
    return;
  }
  if (any_over) {
    if (tid == 0) {
      int w = atomicAdd(a.full_count, 1);
      a.full_list[w] = row;
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
  if (any_nan) {  // a NaN among the first K positions: the heap as written
    if (tid == 0) {
      int w = atomicAdd(a.full_count, 1);
      a.full_list[w] = row;
    }
    return;
  }

  // exact survivor set of the reference heap (see block comment at top)
  uint32_t t, tau = 0xffffffffu, rho = 0u;
  int n64 = 32;
  while (n64 < (int)K) n64 <<= 1;
  if (nm <= 384) {
    // few candidates: one warp selects and sorts, no block barriers (with
    // more, the block's radix passes are faster)
    if (warp != 0) return;
    int nge, ngt;
    t = warp_select_kth_largest(
        nm, K, [&](int i, uint32_t* k) { *k = keys[i]; return ids[i] >= 0; }, S.hist, &nge, &ngt);
    // The candidates hold every element >= t only if no chunk threshold was
    // above t (and there are K of them); otherwise redo the row exactly.
    if (nge < (int)K || t < thr_max) {
      if (lane == 0) {
        int w = atomicAdd(a.full_count, 1);
        a.full_list[w] = row;
      }
      return;
    }
    if (nge != (int)K) {
      // tau: index of the K-th element (in index order) with value >= t;
      // survivors among the ties are the (K - ngt) highest indices <= tau.
      int u1, u2;
      tau = ~warp_select_kth_largest(
          nm, K,
          [&](int i, uint32_t* k) {
            if (ids[i] >= 0 && keys[i] >= t) { *k = ~(uint32_t)ids[i]; return true; }
            return false;
          },
          S.hist, &u1, &u2);
      rho = warp_select_kth_largest(
          nm, K - (uint32_t)ngt,
          [&](int i, uint32_t* k) {
            if (ids[i] >= 0 && keys[i] == t && (uint32_t)ids[i] <= tau) { *k = (uint32_t)ids[i]; return true; }
            return false;
          },
          S.hist, &u1, &u2);
    }
    for (int i = lane; i < n64; i += 32) S.sortbuf[i] = 0ull;
    __syncwarp();
    int base = 0;
    for (int i0 = 0; i0 < nm; i0 += 32) {
      const int i = i0 + lane;
      bool keep = false;
      unsigned long long v = 0ull;
      if (i < nm) {
        const uint32_t k = keys[i];
        const uint32_t id = (uint32_t)ids[i];
        keep = ids[i] >= 0 && ((k > t) || (k == t && id >= rho && id <= tau));
        v = ((unsigned long long)k << 32) | id;
      }
      const unsigned m = __ballot_sync(0xffffffffu, keep);
      if (keep) {
        const int pos = base + __popc(m & lanemask_lt());
        if (pos < kLightKMax) S.sortbuf[pos] = v;
      }
      base += __popc(m);
    }
    __syncwarp();
    warp_bitonic_desc(S.sortbuf, n64);
  } else {
    t = block_select_kth_largest(
        nm, K, [&](int i, uint32_t* k) { *k = keys[i]; return ids[i] >= 0; }, S.hist, S.sel);
    if ((int)S.sel[2] < (int)K || t < thr_max) {
      if (tid == 0) {
        int w = atomicAdd(a.full_count, 1);
        a.full_list[w] = row;
      }
      return;
    }
    if (tid == 0) { S.cnt_gt = 0; S.cnt_ge = 0; S.nsurv = 0; }
    __syncthreads();
    {
      int gt = 0, ge = 0;
      for (int i = tid; i < nm; i += LT_THREADS) {
        gt += ids[i] >= 0 && keys[i] > t;
        ge += ids[i] >= 0 && keys[i] >= t;
      }
      gt = __reduce_add_sync(0xffffffffu, gt);
      ge = __reduce_add_sync(0xffffffffu, ge);
      if (lane == 0) { atomicAdd(&S.cnt_gt, gt); atomicAdd(&S.cnt_ge, ge); }
    }
    __syncthreads();
    const int cgt = S.cnt_gt, cge = S.cnt_ge;
    if (cge != (int)K) {
      tau = ~block_select_kth_largest(
          nm, K,
          [&](int i, uint32_t* k) {
            if (ids[i] >= 0 && keys[i] >= t) { *k = ~(uint32_t)ids[i]; return true; }
            return false;
          },
          S.hist, S.sel);
      rho = block_select_kth_largest(
          nm, K - (uint32_t)cgt,
          [&](int i, uint32_t* k) {
            if (ids[i] >= 0 && keys[i] == t && (uint32_t)ids[i] <= tau) { *k = (uint32_t)ids[i]; return true; }
            return false;
          },
          S.hist, S.sel);
    }
    for (int i = tid; i < n64; i += LT_THREADS) S.sortbuf[i] = 0ull;
    __syncthreads();
    for (int i = tid; i < nm; i += LT_THREADS) {
      const uint32_t k = keys[i];
      const uint32_t id = (uint32_t)ids[i];
      const bool keep = ids[i] >= 0 && ((k > t) || (k == t && id >= rho && id <= tau));
      if (keep) {
        int pos = atomicAdd(&S.nsurv, 1);
        if (pos < kLightKMax) S.sortbuf[pos] = ((unsigned long long)k << 32) | id;
      }
    }
    __syncthreads();
    block_bitonic_desc(S.sortbuf, n64);
  }

  // ---- replay of sampler.nim:98-121 by one warp ----------------------------
  // The fp32 chains (sum, running sum, draw) run in one lane in the
  // reference's order; the break conditions are evaluated afterwards on the
  // stored running values, so the chains carry no data-dependent branches.
  if (warp == 0) {
    const int n = (int)K;
    for (int i = lane; i < n; i += 32) S.tval[i] = fkey_inv((uint32_t)(S.sortbuf[i] >> 32));
    __syncwarp();
    const float mx = S.tval[0];
    for (int i = lane; i < n; i += 32) S.tval[i] = ref_expf(__fsub_rn(S.tval[i], mx));
    __syncwarp();
    float s = 0.0f;
    if (lane == 0) {
#pragma unroll 8
      for (int i = 0; i < n; ++i) s = __fadd_rn(s, S.tval[i]);
    }
    s = __shfl_sync(0xffffffffu, s, 0);
    for (int i = lane; i < n; i += 32) S.pval[i] = __fdiv_rn(S.tval[i], s);
    __syncwarp();
    int nn = n;
    if (p.top_p > 0.0 && p.top_p < 1.0) {
      if (lane == 0) {
        float cum = 0.0f;
#pragma unroll 8
        for (int i = 0; i < n; ++i) { cum = __fadd_rn(cum, S.pval[i]); S.seq[i] = cum; }
      }
      __syncwarp();
      int first = n;
      for (int c0 = 0; c0 < n; c0 += 32) {
        const int i = c0 + lane;
        const unsigned b = __ballot_sync(0xffffffffu, i < n && (double)S.seq[i] >= p.top_p);
        if (b) { first = c0 + __ffs(b) - 1; break; }
      }
      if (first < n) nn = first + 1;
    }
    if (p.min_p > 0.0) {
      const float thrp = __fmul_rn(S.pval[0], __double2float_rn(p.min_p));
      int m = nn;
      for (int c0 = 0; c0 < nn; c0 += 32) {
        const int i = c0 + lane;
        const unsigned b = __ballot_sync(0xffffffffu, i >= 1 && i < nn && !(S.pval[i] >= thrp));
        if (b) { m = c0 + __ffs(b) - 1; break; }
      }
      nn = m < 1 ? 1 : m;
    }
    __syncwarp();
    if (lane == 0) {
      float total = 0.0f;
#pragma unroll 8
      for (int i = 0; i < nn; ++i) total = __fadd_rn(total, S.pval[i]);
      float r = __fmul_rn(__double2float_rn(a.uniforms[row]), total);
#pragma unroll 8
      for (int i = 0; i < nn; ++i) { r = __fsub_rn(r, S.pval[i]); S.seq[i] = r; }
    }
    __syncwarp();
    int pos = nn - 1;
    for (int c0 = 0; c0 < nn; c0 += 32) {
      const int i = c0 + lane;
      const unsigned b = __ballot_sync(0xffffffffu, i < nn && S.seq[i] <= 0.0f);
      if (b) { pos = c0 + __ffs(b) - 1; break; }
    }
    if (lane == 0) {
      a.out_ids[row] = (int64_t)(uint32_t)(S.sortbuf[pos] & 0xffffffffull);
      if (a.out_probs) a.out_probs[row] = S.pval[pos];
    }
  }
}

static std::atomic<int> g_light_smem_set_row[kMaxDevicesAttr];
static std::atomic<int> g_light_smem_set_split[kMaxDevicesAttr];

// one CTA per row: the whole-row ring shape; a row split over a cluster: the
// split shape
size_t light_smem_bytes(int C, int chunk) {
  return C == 1 ? light_smem_bytes_t<LT_STAGE_ROW, LT_NSTAGE_ROW>(C, chunk)
                : light_smem_bytes_t<LT_STAGE_SPLIT, LT_NSTAGE_SPLIT>(C, chunk);
}

static std::atomic<int> g_light_big_cluster[kMaxDevicesAttr];  // 0 unknown, 1 no, 2 yes

// Clusters of more than 8 CTAs need the non-portable size allowed, and room
// on one GPC for 16 CTAs of this size; answered once per device.
int light_max_cluster(int V) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevicesAttr) return 8;
  const int known = g_light_big_cluster[dev].load(std::memory_order_relaxed);
  if (known) return known == 2 ? LT_CMAX : 8;
  int ok = 1;
  const int chunk = ((V + LT_CMAX - 1) / LT_CMAX + 3) & ~3;
  const size_t smem = light_smem_bytes(LT_CMAX, chunk);
  const void* fn = reinterpret_cast<const void*>(light_kernel<LT_STAGE_SPLIT, LT_NSTAGE_SPLIT>);
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
      ensure_smem_attr(fn, (int)smem, g_light_smem_set_split) == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(LT_CMAX, 1, 1);
    cfg.blockDim = dim3(LT_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = LT_CMAX;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) == cudaSuccess &&
        n >= 1)
      ok = 2;
  }
  (void)cudaGetLastError();
  g_light_big_cluster[dev].store(ok, std::memory_order_relaxed);
  return ok == 2 ? LT_CMAX : 8;
}

cudaError_t launch_light(const BatchArgs& a, int C, int chunk, cudaStream_t stream) {
  const size_t smem = light_smem_bytes(C, chunk);
  const void* fn = C == 1 ? reinterpret_cast<const void*>(light_kernel<LT_STAGE_ROW, LT_NSTAGE_ROW>)
                          : reinterpret_cast<const void*>(light_kernel<LT_STAGE_SPLIT, LT_NSTAGE_SPLIT>);
  cudaError_t e = ensure_smem_attr(fn, (int)smem, C == 1 ? g_light_smem_set_row : g_light_smem_set_split);
  if (e != cudaSuccess) return e;
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
  if (C == 1) return cudaLaunchKernelEx(&cfg, light_kernel<LT_STAGE_ROW, LT_NSTAGE_ROW>, a, C, chunk);
  return cudaLaunchKernelEx(&cfg, light_kernel<LT_STAGE_SPLIT, LT_NSTAGE_SPLIT>, a, C, chunk);
}

}  // namespace nls
