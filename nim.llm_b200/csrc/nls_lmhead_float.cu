// nls_lmhead_float.cu -- the output projection's float path (dequantRow then
// dotF32, quant.nim:336-374; taken by model.nim:185 for F16 weights, for
// Q8_0 above 4 batch rows and under exactMatmul) for F16, Q8_0 and Q4_0
// weights, any batch size, tiled for instruction-level parallelism.
//
// dotF32 keeps eight fp32 accumulators: s_j += x[i] * y[i] for i = j, j + 8,
// ... in order (a multiply, then an add: no fused multiply-add), and returns
// (((s0 + s1) + (s2 + s3)) + (s4 + s5)) + (s6 + s7). Only each chain's own
// order is fixed, so a thread can advance many chains at once: thread
// (chain j, row group, batch group) holds the chains j of 4 weight rows x up
// to 8 batch rows (up to 32 independent dependency chains) and walks them together,
// one dequantised weight serving all its batch rows. A CTA of 256 threads
// takes a tile of R weight rows (R = 128 / batch groups) for every batch row
// of the launch; the tile's weights and the activations stream through
// shared memory in chunks of 256 values (16-byte cp.async, double-buffered).
// The 8 chains of a (row, batch row) sit in 8 consecutive lanes and combine
// through shuffles in dotF32's order.
#include <cuda_fp16.h>

#include <algorithm>

#include "nls_kernels.h"
#include "nls_tma.cuh"

namespace nls {

namespace {

constexpr int kFThreads = 256;
constexpr int kFChunk = 256;     // values per chunk
constexpr int kFSteps = kFChunk / 8;

struct FloatArgs {
  const uint8_t* w;  // rows x row_bytes, 16-byte aligned, row_bytes % 16 == 0
  int64_t row_bytes;
  int rows, cols, nb;
  int G;             // batch groups (1, 2, 4): batch rows per thread = BB, G * BB >= nb
  int R;             // weight rows per tile = 4 * (32 / G)
  int ntiles;
  int chunk_bytes;   // bytes of 256 values of one row (multiple of 16)
  const float* x;    // [nb x cols], 16-byte aligned
  float* y;          // y[b * ldy + r]
  int64_t ldy;
};

__device__ __forceinline__ float half_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// weights e .. e + 24 (step 8) of one row's chunk, dequantised as dequantRow
// does (quant.nim:336-352): F16 converted; Q8_0 d * q; Q4_0 (q - 8) * d, all
// exact in fp32
template <int WT>
__device__ __forceinline__ void load_w4(const uint8_t* row, int e, float (&w)[4]) {
  if constexpr (WT == 1) {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(row);
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = half_to_float(h[e + 8 * u]);
  } else if constexpr (WT == 8) {
    const uint8_t* b = row + (e >> 5) * 34;  // e .. e + 24 share a block
    const float d = half_to_float((uint16_t)(b[0] | (b[1] << 8)));
#pragma unroll
    for (int u = 0; u < 4; ++u) w[u] = (float)(int)(int8_t)b[2 + ((e + 8 * u) & 31)] * d;
  } else {  // Q4_0
    const uint8_t* b = row + (e >> 5) * 18;
    const float d = half_to_float((uint16_t)(b[0] | (b[1] << 8)));
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int j = (e + 8 * u) & 31;
      const uint8_t q = b[2 + (j & 15)];
      w[u] = (float)((j < 16 ? (q & 0xF) : (q >> 4)) - 8) * d;
    }
  }
}

template <int WT, int BB>
__global__ void __launch_bounds__(kFThreads) lmh_float_kernel(const FloatArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int tid = threadIdx.x, kk = tid & 7, rest = tid >> 3;
  const int bg = rest % a.G, rg = rest / a.G;  // batch group, row group
  const int nbp = a.G * BB;                    // batch rows staged (padded)
  uint8_t* wbuf = smem;                                          // [2][R][chunk_bytes]
  float* xbuf = reinterpret_cast<float*>(smem + 2 * (size_t)a.R * a.chunk_bytes);  // [2][nbp][256]
  const int nchunks = a.cols / kFChunk;
  const int wunits = a.R * (a.chunk_bytes / 16), xunits = nbp * (kFChunk / 4);

  for (int t = blockIdx.x; t < a.ntiles; t += gridDim.x) {
    const int r0 = t * a.R;
    auto stage = [&](int c) {
      const int buf = c & 1;
      for (int i = tid; i < wunits; i += kFThreads) {
        const int rr = i / (a.chunk_bytes / 16), u = i % (a.chunk_bytes / 16);
        const int r = r0 + rr;
        if (r < a.rows)
          cp_async16(wbuf + ((size_t)buf * a.R + rr) * a.chunk_bytes + 16 * u,
                     a.w + (size_t)r * a.row_bytes + (size_t)c * a.chunk_bytes + 16 * u);
      }
      for (int i = tid; i < xunits; i += kFThreads) {
        const int b = i / (kFChunk / 4), u = i % (kFChunk / 4);
        float* dst = xbuf + ((size_t)buf * nbp + b) * kFChunk + 4 * u;
        if (b < a.nb)
          cp_async16(dst, a.x + (size_t)b * a.cols + (size_t)c * kFChunk + 4 * u);
        else
          *reinterpret_cast<float4*>(dst) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
      cp_async_commit();
    };
    float acc[4][BB];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < BB; ++j) acc[i][j] = 0.0f;
    stage(0);
    for (int c = 0; c < nchunks; ++c) {
      if (c + 1 < nchunks) stage(c + 1);
      else cp_async_commit();
      cp_async_wait<1>();
      __syncthreads();
      const int buf = c & 1;
      const uint8_t* wr = wbuf + ((size_t)buf * a.R + 4 * rg) * a.chunk_bytes;
      const float* xr = xbuf + ((size_t)buf * nbp + bg * BB) * kFChunk;
      // steps k of the chunk, four at a time (one Q8_0 / Q4_0 block)
#pragma unroll 1
      for (int k = 0; k < kFSteps; k += 4) {
        const int e = kk + 8 * k;
        float w[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) load_w4<WT>(wr + (size_t)i * a.chunk_bytes, e, w[i]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float xv[BB];
#pragma unroll
          for (int j = 0; j < BB; ++j) xv[j] = xr[j * kFChunk + e + 8 * u];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < BB; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(w[i][u], xv[j]));
        }
      }
      __syncthreads();  // the buffer is staged again two chunks on
    }
    // dotF32's combination (quant.nim:374): the 8 chains of a (row, batch
    // row) are lanes 8q .. 8q + 7
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < BB; ++j) {
        const float s = acc[i][j];
        const float s1 = __shfl_down_sync(0xffffffffu, s, 1, 8);
        const float s2 = __shfl_down_sync(0xffffffffu, s, 2, 8);
        const float s3 = __shfl_down_sync(0xffffffffu, s, 3, 8);
        const float s4 = __shfl_down_sync(0xffffffffu, s, 4, 8);
        const float s5 = __shfl_down_sync(0xffffffffu, s, 5, 8);
        const float s6 = __shfl_down_sync(0xffffffffu, s, 6, 8);
        const float s7 = __shfl_down_sync(0xffffffffu, s, 7, 8);
        const int r = r0 + 4 * rg + i, b = bg * BB + j;
        if (kk == 0 && r < a.rows && b < a.nb) {
          float v = __fadd_rn(s, s1);
          v = __fadd_rn(v, __fadd_rn(s2, s3));
          v = __fadd_rn(v, __fadd_rn(s4, s5));
          v = __fadd_rn(v, __fadd_rn(s6, s7));
          a.y[(size_t)b * a.ldy + r] = v;
        }
      }
    }
  }
  cp_async_wait<0>();
}

template <int WT>
cudaError_t launch_bb(const FloatArgs& a, int BB, size_t smem, int grid, cudaStream_t st) {
  cudaError_t e;
  switch (BB) {
    case 1:
      e = cudaFuncSetAttribute(lmh_float_kernel<WT, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) lmh_float_kernel<WT, 1><<<grid, kFThreads, smem, st>>>(a);
      break;
    case 2:
      e = cudaFuncSetAttribute(lmh_float_kernel<WT, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) lmh_float_kernel<WT, 2><<<grid, kFThreads, smem, st>>>(a);
      break;
    case 4:
      e = cudaFuncSetAttribute(lmh_float_kernel<WT, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) lmh_float_kernel<WT, 4><<<grid, kFThreads, smem, st>>>(a);
      break;
    default:
      e = cudaFuncSetAttribute(lmh_float_kernel<WT, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e == cudaSuccess) lmh_float_kernel<WT, 8><<<grid, kFThreads, smem, st>>>(a);
      break;
  }
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

int chunk_bytes_of(int wtype) {
  switch (wtype) {
    case 1: return kFChunk * 2;
    case 8: return kFChunk / 32 * 34;
    case 2: return kFChunk / 32 * 18;
    default: return 0;
  }
}

}  // namespace

bool lm_head_float_tiled(int wtype, int cols, int64_t row_bytes) {
  return chunk_bytes_of(wtype) > 0 && cols % kFChunk == 0 && row_bytes % 16 == 0;
}

// batch rows per launch: 16 (four groups of 4)
cudaError_t launch_lm_head_float(const uint8_t* w, int wtype, int64_t row_bytes, int rows, int cols,
                                 const float* x, int nb, float* y, int64_t ldy, int sm_count,
                                 cudaStream_t st) {
  for (int b0 = 0; b0 < nb; b0 += 16) {
    const int n = std::min(16, nb - b0);
    const int BB = n >= 8 ? 8 : (n >= 4 ? 4 : (n >= 2 ? 2 : 1));
    FloatArgs a{};
    a.w = w;
    a.row_bytes = row_bytes;
    a.rows = rows;
    a.cols = cols;
    a.nb = n;
    const int g = (n + BB - 1) / BB;
    a.G = g <= 1 ? 1 : (g <= 2 ? 2 : 4);  // a power of two (row groups 32 / G)
    a.R = 4 * (32 / a.G);
    a.ntiles = (rows + a.R - 1) / a.R;
    a.chunk_bytes = chunk_bytes_of(wtype);
    a.x = x + (size_t)b0 * cols;
    a.y = y + (size_t)b0 * ldy;
    a.ldy = ldy;
    const size_t smem = 2 * (size_t)a.R * a.chunk_bytes + 2 * (size_t)a.G * BB * kFChunk * 4;
    const int per_sm = std::max(1, std::min(8, (int)((size_t)(227 * 1024) / (smem + 1024))));
    const int grid = std::min(a.ntiles, sm_count * per_sm);
    cudaError_t e;
    switch (wtype) {
      case 1: e = launch_bb<1>(a, BB, smem, grid, st); break;
      case 8: e = launch_bb<8>(a, BB, smem, grid, st); break;
      default: e = launch_bb<2>(a, BB, smem, grid, st); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace nls
