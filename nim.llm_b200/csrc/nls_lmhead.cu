// nls_lmhead.cu -- the output projection that produces the sampler's logits:
// matmul(m.output, xb, logits, nb) (model.nim:466-470 -> :179-189, row task
// :144-169), bit for bit.
//
// The reference computes, per output row r and batch row b, one dot product
// whose fp32 rounding order is fixed by the code:
//  * int8 activation path (the default; quantizeAct quant.nim:646-662 with
//    dotQ8_0i / dotQ4_0i / dotQ6K quant.nim:731-786): per weight block an
//    exact integer dot product, then acc += (d_w * d_a) * float(sumi) block
//    after block (Q6_K: (d_a * d_w) * float(sumi));
//  * float path (exactMatmul, Q8_0 with more than 4 batch rows, F32/F16):
//    dequantRow then dotF32 (quant.nim:362-374): eight strided fp32
//    accumulators combined as (((s0+s1) + (s2+s3)) + (s4+s5)) + (s6+s7).
//    (F16 / Q8_0 / Q4_0 rows of whole 256-value chunks at more than one batch
//    row, or Q8_0 / Q4_0 at any, take the tiled kernel of nls_lmhead_float.cu.)
// Both are HBM-bound on the weights (one pass over rows x rowBytes per call at
// small batch). The kernel streams row tiles of the weights through a ring of
// shared-memory slots with cp.async.bulk (no multicast) and:
//  * int8 path: warps 1.. compute every block term of a tile in parallel
//    (dp4a on the packed int8 values) into a shared-memory table; warp 0 then
//    replays each (row, batch) sum in block order, one lane per sum, while the
//    other warps already work on the next tile;
//  * float path: one lane per (row, batch, accumulator) walks its strided
//    elements in order, dequantising on the fly.
// Everything is exact fp32 arithmetic in the reference's order: the library
// is built with -fmad=false, so no multiply-add is fused.
#include <cuda_fp16.h>

#include <algorithm>

#include "nls_kernels.h"
#include "nls_tma.cuh"

namespace nls {

namespace {

constexpr int kLmhThreads = 256;      // float path
constexpr int kLmhTermThreads = 256;  // int8 path: warps 1..8 compute block terms,
constexpr int kLmhInt8Threads = kLmhTermThreads + 32;  // warp 0 replays the sums
constexpr int kLmhMaxChains = 32;     // int8 path: one warp replays the sums
constexpr int kLmhInt8MaxNb = 4;      // batch rows per int8 launch
// int8 path: two CTAs per SM (about 110 KB of shared memory each) for twice
// the warps to hide shared-memory and dp4a latency, except Q6_K with more
// than 2 batch rows (its activations in registers need more than the 96
// registers a thread gets then): one CTA per SM with the whole shared memory
constexpr int kLmhSmemMax2 = 110 * 1024;
constexpr int kLmhSmemMax = 226 * 1024;  // the kernel also has static shared variables
constexpr int kLmhSlotTarget1 = 48 * 1024, kLmhSlotTarget2 = 32 * 1024;
constexpr int kLmhGroupChains1 = 64, kLmhGroupChains2 = 32;  // sums replayed per group

struct LmhArgs {
  const uint8_t* w;  // rows x row_bytes, 16-byte aligned
  int64_t row_bytes;
  int rows, cols;
  int nblk;          // weight blocks per row (int8 path)
  int nb;            // batch rows of this launch
  const float* x;    // [nb x cols] activations of this launch
  float* y;          // y[b * ldy + r]
  int64_t ldy;
  int R;             // rows per tile
  int ntiles;
  int slot_bytes;    // one ring slot (multiple of 16)
  int nst;           // ring slots
  int padded;        // 1: row i of a tile at slot + i*pitch; 0: one contiguous copy
  int pitch;
  int act_bytes;     // shared bytes of the activation region (multiple of 16)
  int tpitch;        // int8 path: floats per sum in the term table (odd)
  int gtiles;        // int8 path: tiles per group (their sums are replayed together)
  int gchains;       //            gtiles * R * nb, at most 64 (two per replay lane)
  int par;           // Q6_K at one batch row, Q8_0: slots arranged so that every warp
                     // holds blocks of one parity (so one 4-byte alignment of the block start)
  int fixed;         // int8 path: 1 when each term thread keeps one block's
                     // activations in registers (lanes per block x blocks per
                     // row <= term threads), else 0 (generic loop)
  int* status;
};

__device__ __forceinline__ void set_status(int* st, int code) { atomicCAS(st, 0, code); }

// Bytes [p, p + 4n) of shared memory as n 32-bit words, p 2-byte aligned.
// Reads one aligned word past the end (the caller keeps that inside the
// CTA's shared memory).
template <int N>
__device__ __forceinline__ void ld_words(const uint8_t* p, uint32_t (&out)[N]) {
  const uint32_t* a = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
  const uint32_t sel = (reinterpret_cast<uintptr_t>(p) & 2) ? 0x5432u : 0x3210u;
  uint32_t prev = a[0];
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const uint32_t next = a[k + 1];
    out[k] = __byte_perm(prev, next, sel);
    prev = next;
  }
}

// dot product of four unsigned bytes of a with four signed bytes of b, plus c
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// sum of the four signed bytes of w
__device__ __forceinline__ int bytesum(int w) { return __dp4a(w, 0x01010101, 0); }

// ld_words for a p known to be 4-byte aligned (A4) or only 2-byte aligned
template <bool A4, int N>
__device__ __forceinline__ void ld_words_al(const uint8_t* p, uint32_t (&out)[N]) {
  if constexpr (A4) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(p);
#pragma unroll
    for (int k = 0; k < N; ++k) out[k] = w[k];
  } else {
    ld_words<N>(p, out);
  }
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// ---- int8 path: one block term per (row, block) for every batch row ---------

// dotQ8_0i (quant.nim:762-772): s = sum of 32 int8 products, term = (dw * da) * float(s)
template <int NB>
__device__ __forceinline__ void terms_q8_0(const uint8_t* blk, int ib, const LmhArgs& a,
                                           const int32_t* aqw, const float* ad, float* T, int tp) {
  uint32_t W[9];
  ld_words<9>(blk, W);
  const float dw = half_bits_to_float(W[0]);
  int q[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) q[k] = (int)__byte_perm(W[k], W[k + 1], 0x5432);
  const int wpb = a.cols >> 2;  // activation words per batch row
  const int apb = a.cols >> 5;  // activation blocks per batch row
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b >= a.nb) break;
    const int32_t* av = aqw + b * wpb + ib * 8;
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) s = __dp4a(q[k], av[k], s);
    T[b * tp] = (dw * ad[b * apb + ib]) * __int2float_rn(s);
  }
}

// dotQ4_0i (quant.nim:774-786): nibbles minus 8 against a[l] and a[l + 16]
template <int NB>
__device__ __forceinline__ void terms_q4_0(const uint8_t* blk, int ib, const LmhArgs& a,
                                           const int32_t* aqw, const float* ad, float* T, int tp) {
  uint32_t W[5];
  ld_words<5>(blk, W);
  const float dw = half_bits_to_float(W[0]);
  int lo[4], hi[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t q = __byte_perm(W[k], W[k + 1], 0x5432);
    lo[k] = (int)__vsub4(q & 0x0F0F0F0Fu, 0x08080808u);
    hi[k] = (int)__vsub4((q >> 4) & 0x0F0F0F0Fu, 0x08080808u);
  }
  const int wpb = a.cols >> 2;
  const int apb = a.cols >> 5;
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b >= a.nb) break;
    const int32_t* av = aqw + b * wpb + ib * 8;
    int s = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s = __dp4a(lo[k], av[k], s);
      s = __dp4a(hi[k], av[4 + k], s);
    }
    T[b * tp] = (dw * ad[b * apb + ib]) * __int2float_rn(s);
  }
}

// dotQ6K (quant.nim:731-760): ql[128] qh[64] int8 scales[16] d at 208
template <int NB>
__device__ __forceinline__ void terms_q6_k(const uint8_t* blk, int ib, const LmhArgs& a,
                                           const int32_t* aqw, const float* ad, float* T, int tp) {
  uint32_t SC[4], DW[1];
  ld_words<4>(blk + 192, SC);
  ld_words<1>(blk + 208, DW);
  const float dw = half_bits_to_float(DW[0]);
  const int wpb = a.cols >> 2;
  const int apb = a.cols >> 8;
  int sumi[NB];
#pragma unroll
  for (int b = 0; b < NB; ++b) sumi[b] = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t QA[4], QB[4], QH[4];
      ld_words<4>(blk + 64 * h + 16 * half, QA);
      ld_words<4>(blk + 64 * h + 32 + 16 * half, QB);
      ld_words<4>(blk + 128 + 32 * h + 16 * half, QH);
      int q1[4], q2[4], q3[4], q4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t hq = QH[k];
        q1[k] = (int)__vsub4((QA[k] & 0x0F0F0F0Fu) | ((hq & 0x03030303u) << 4), 0x20202020u);
        q2[k] = (int)__vsub4((QB[k] & 0x0F0F0F0Fu) | (((hq >> 2) & 0x03030303u) << 4), 0x20202020u);
        q3[k] = (int)__vsub4(((QA[k] >> 4) & 0x0F0F0F0Fu) | (((hq >> 4) & 0x03030303u) << 4), 0x20202020u);
        q4[k] = (int)__vsub4(((QB[k] >> 4) & 0x0F0F0F0Fu) | (((hq >> 6) & 0x03030303u) << 4), 0x20202020u);
      }
      const int so = 8 * h + half;
      const int sc0 = (int)(int8_t)(SC[so >> 2] >> (8 * (so & 3)));
      const int sc1 = (int)(int8_t)(SC[(so + 2) >> 2] >> (8 * ((so + 2) & 3)));
      const int sc2 = (int)(int8_t)(SC[(so + 4) >> 2] >> (8 * ((so + 4) & 3)));
      const int sc3 = (int)(int8_t)(SC[(so + 6) >> 2] >> (8 * ((so + 6) & 3)));
      const int w0 = (128 * h + 16 * half) >> 2;  // activation word of l = 16*half
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        if (b >= a.nb) break;
        const int32_t* av = aqw + b * wpb + ib * 64 + w0;
        int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          s0 = __dp4a(q1[k], av[k], s0);
          s1 = __dp4a(q2[k], av[8 + k], s1);
          s2 = __dp4a(q3[k], av[16 + k], s2);
          s3 = __dp4a(q4[k], av[24 + k], s3);
        }
        sumi[b] += sc0 * s0 + sc1 * s1 + sc2 * s2 + sc3 * s3;
      }
    }
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b >= a.nb) break;
    T[b * tp] = (ad[b * apb + ib] * dw) * __int2float_rn(sumi[b]);
  }
}

// ---- int8 path, fixed mapping: the thread's block index is fixed, so its
// activation words (and scale) stay in registers for the whole kernel ------

// AL: the block start modulo 4 when known for the whole warp (0 or 2: plain
// word loads), else -1 (2-byte aligned, byte permutes)
template <int NB, int AL = -1>
__device__ __forceinline__ void term_q8_0_reg(const uint8_t* blk, const int (&av)[NB][16],
                                              const float (&da)[NB], int nb, float* T, int tp) {
  int q[8];
  float dw;
  if constexpr (AL == 2) {
    // the 32 values start on a word boundary; the scale is the high half of
    // the word before them
    const uint32_t* w = reinterpret_cast<const uint32_t*>(blk + 2);
#pragma unroll
    for (int k = 0; k < 8; ++k) q[k] = (int)w[k];
    dw = half_bits_to_float(w[-1] >> 16);
  } else {
    uint32_t W[9];
    ld_words_al<AL == 0, 9>(blk, W);
    dw = half_bits_to_float(W[0]);
#pragma unroll
    for (int k = 0; k < 8; ++k) q[k] = (int)__byte_perm(W[k], W[k + 1], 0x5432);
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b >= nb) break;
    int s = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) s = __dp4a(q[k], av[b][k], s);
    T[b * tp] = (dw * da[b]) * __int2float_rn(s);
  }
}

// (q - 8) . a = q . a - 8 * sum(a): asum[b] is the sum of the block's 32
// activation values of batch row b (integers, exact)
template <int NB>
__device__ __forceinline__ void term_q4_0_reg(const uint8_t* blk, const int (&av)[NB][16],
                                              const float (&da)[NB], const int (&asum)[NB][4],
                                              int nb, float* T, int tp) {
  uint32_t W[5];
  ld_words<5>(blk, W);
  const float dw = half_bits_to_float(W[0]);
  uint32_t lo[4], hi[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t q = __byte_perm(W[k], W[k + 1], 0x5432);
    lo[k] = q & 0x0F0F0F0Fu;
    hi[k] = (q >> 4) & 0x0F0F0F0Fu;
  }
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b >= nb) break;
    int s = -8 * asum[b][0];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s = dp4a_us(lo[k], av[b][k], s);
      s = dp4a_us(hi[k], av[b][4 + k], s);
    }
    T[b * tp] = (dw * da[b]) * __int2float_rn(s);
  }
}

// Q6_K: four lanes per block, lane qi taking (h, half) = (qi >> 1, qi & 1);
// their integer partial sums add up exactly (shuffles within the 4-lane
// group `gmask`), and lane qi == 0 forms the term.
template <int NB>
__device__ __forceinline__ void term_q6_k_reg(const uint8_t* blk, int qi, const int (&av)[NB][16],
                                              const float (&da)[NB], const int (&asum)[NB][4],
                                              int nb, float* T, int tp, unsigned gmask) {
  const int h = qi >> 1, half = qi & 1;
  uint32_t QA[4], QB[4], QH[4], SC[2], DW[1];
  ld_words<4>(blk + 64 * h + 16 * half, QA);
  ld_words<4>(blk + 64 * h + 32 + 16 * half, QB);
  ld_words<4>(blk + 128 + 32 * h + 16 * half, QH);
  ld_words<2>(blk + 192 + 8 * h, SC);
  ld_words<1>(blk + 208, DW);
  // the 6-bit values before the - 32 (quant.nim:744-747): low nibble from
  // ql, bits 4-5 from the qh byte's bit pair
  uint32_t q1[4], q2[4], q3[4], q4[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t hq = QH[k];
    q1[k] = (QA[k] & 0x0F0F0F0Fu) | ((hq << 4) & 0x30303030u);
    q2[k] = (QB[k] & 0x0F0F0F0Fu) | ((hq << 2) & 0x30303030u);
    q3[k] = ((QA[k] >> 4) & 0x0F0F0F0Fu) | (hq & 0x30303030u);
    q4[k] = ((QB[k] >> 4) & 0x0F0F0F0Fu) | ((hq >> 2) & 0x30303030u);
  }
  // scales so, so+2, so+4, so+6 with so = 8h + half (bytes of SC[0], SC[1])
  const int sc0 = (int)(int8_t)(SC[0] >> (8 * half));
  const int sc1 = (int)(int8_t)(SC[0] >> (8 * (half + 2)));
  const int sc2 = (int)(int8_t)(SC[1] >> (8 * half));
  const int sc3 = (int)(int8_t)(SC[1] >> (8 * (half + 2)));
  const float dw = half_bits_to_float(DW[0]);
#pragma unroll
  for (int b = 0; b < NB; ++b) {
    if (b >= nb) break;
    // (q - 32) . a = q . a - 32 * sum(a), sums of the 16 activation values
    int s0 = -32 * asum[b][0], s1 = -32 * asum[b][1], s2 = -32 * asum[b][2], s3 = -32 * asum[b][3];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      s0 = dp4a_us(q1[k], av[b][k], s0);
      s1 = dp4a_us(q2[k], av[b][4 + k], s1);
      s2 = dp4a_us(q3[k], av[b][8 + k], s2);
      s3 = dp4a_us(q4[k], av[b][12 + k], s3);
    }
    int part = sc0 * s0 + sc1 * s1 + sc2 * s2 + sc3 * s3;
    part += __shfl_xor_sync(gmask, part, 1);
    part += __shfl_xor_sync(gmask, part, 2);
    if (qi == 0) T[b * tp] = (da[b] * dw) * __int2float_rn(part);
  }
}

// Q6_K with one batch row: two lanes per block, lane h taking both 16-value
// groups of half h (the 32 activation words stay in registers); the two
// integer partial sums add up exactly through one shuffle.
// A4: the block starts on a 4-byte boundary (plain word loads, no byte
// permutes); else on a 2-byte boundary
template <bool A4>
__device__ __forceinline__ void term_q6_k_pair(const uint8_t* blk, int h, const int (&av)[32],
                                               float da, const int (&asum)[8], float* T,
                                               unsigned gmask) {
  uint32_t SC[2];
  ld_words_al<A4>(blk + 192 + 8 * h, SC);
  int part = 0;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t QA[4], QB[4], QH[4];
    ld_words_al<A4>(blk + 64 * h + 16 * half, QA);
    ld_words_al<A4>(blk + 64 * h + 32 + 16 * half, QB);
    ld_words_al<A4>(blk + 128 + 32 * h + 16 * half, QH);
    // scales so, so+2, so+4, so+6 with so = 8h + half
    const int sc0 = (int)(int8_t)(SC[0] >> (8 * half));
    const int sc1 = (int)(int8_t)(SC[0] >> (8 * (half + 2)));
    const int sc2 = (int)(int8_t)(SC[1] >> (8 * half));
    const int sc3 = (int)(int8_t)(SC[1] >> (8 * (half + 2)));
    int s0 = -32 * asum[4 * half], s1 = -32 * asum[4 * half + 1];
    int s2 = -32 * asum[4 * half + 2], s3 = -32 * asum[4 * half + 3];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t qa = QA[k], qb = QB[k], hq = QH[k];
      s0 = dp4a_us((qa & 0x0F0F0F0Fu) | ((hq << 4) & 0x30303030u), av[16 * half + k], s0);
      s1 = dp4a_us((qb & 0x0F0F0F0Fu) | ((hq << 2) & 0x30303030u), av[16 * half + 4 + k], s1);
      s2 = dp4a_us(((qa >> 4) & 0x0F0F0F0Fu) | (hq & 0x30303030u), av[16 * half + 8 + k], s2);
      s3 = dp4a_us(((qb >> 4) & 0x0F0F0F0Fu) | ((hq >> 2) & 0x30303030u), av[16 * half + 12 + k], s3);
    }
    part += sc0 * s0 + sc1 * s1 + sc2 * s2 + sc3 * s3;
  }
  uint32_t DW[1];
  ld_words_al<A4>(blk + 208, DW);
  part += __shfl_xor_sync(gmask, part, 1);
  if (h == 0) T[0] = (da * half_bits_to_float(DW[0])) * __int2float_rn(part);
}

// ---- float path: dequantised element e of a row (dequantRow, quant.nim:336-352)
template <int WT>
__device__ __forceinline__ float wval(const uint8_t* row, int e) {
  if constexpr (WT == 0) {
    return reinterpret_cast<const float*>(row)[e];
  } else if constexpr (WT == 1) {
    return half_bits_to_float(reinterpret_cast<const uint16_t*>(row)[e]);
  } else if constexpr (WT == 8) {
    const uint8_t* b = row + (e >> 5) * 34;
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(b));
    return (float)(int)(int8_t)b[2 + (e & 31)] * d;
  } else if constexpr (WT == 2) {
    const uint8_t* b = row + (e >> 5) * 18;
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(b));
    const int j = e & 31;
    const uint8_t q = b[2 + (j & 15)];
    const int v = (j < 16 ? (q & 0xF) : (q >> 4)) - 8;
    return (float)v * d;
  } else {  // Q6_K
    const uint8_t* b = row + (e >> 8) * 210;
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t*>(b + 208));
    const int j = e & 255;
    const int n = j >> 7, jj = j & 127, qd = jj >> 5, l = jj & 31;
    const uint8_t lb = b[64 * n + l + 32 * (qd & 1)];
    const uint8_t hb = b[128 + 32 * n + l];
    const int q = (int)(((qd >= 2) ? (lb >> 4) : (lb & 0xF)) | (((hb >> (2 * qd)) & 3) << 4)) - 32;
    const float sc = (float)(int)(int8_t)b[192 + 8 * n + (l >> 4) + 2 * qd];
    return (d * sc) * (float)q;
  }
}

// ---- the kernel ------------------------------------------------------------

struct RingPos {
  int slot;
  uint32_t parity;
};

__device__ __forceinline__ RingPos ring_pos(int k, int nst) {
  return RingPos{k % nst, (uint32_t)((k / nst) & 1)};
}

// Thread 0: start the copy of tile t into ring slot `slot`.
__device__ __forceinline__ void issue_tile(const LmhArgs& a, int t, uint8_t* slot, uint64_t* bar) {
  const int r0 = t * a.R;
  const int nr = min(a.R, a.rows - r0);
  if (a.padded) {
    const uint32_t rb = (uint32_t)a.row_bytes;
    mbar_arrive_expect_tx(bar, rb * (uint32_t)nr);
    for (int i = 0; i < nr; ++i)
      bulk_copy_g2s(slot + (size_t)i * a.pitch, a.w + (size_t)(r0 + i) * a.row_bytes, rb, bar);
    return;
  }
  // one copy of [start & ~15, end rounded up), never past the last whole
  // 16 bytes of the weights; the few bytes after those go by plain loads
  const int64_t start = (int64_t)r0 * a.row_bytes;
  const int64_t end = start + (int64_t)nr * a.row_bytes;
  const int64_t lo = start & ~int64_t(15);
  const int64_t last16 = ((int64_t)a.rows * a.row_bytes) & ~int64_t(15);
  int64_t hi = (end + 15) & ~int64_t(15);
  if (hi > last16) hi = last16;
  if (hi < lo) hi = lo;
  for (int64_t g = max(hi, start); g < end; ++g) slot[g - lo] = a.w[g];
  mbar_arrive_expect_tx(bar, (uint32_t)(hi - lo));
  if (hi > lo) bulk_copy_g2s(slot, a.w + lo, (uint32_t)(hi - lo), bar);
}

__device__ __forceinline__ const uint8_t* tile_row(const LmhArgs& a, const uint8_t* slot, int t, int i) {
  if (a.padded) return slot + (size_t)i * a.pitch;
  const int64_t start = (int64_t)t * a.R * a.row_bytes;
  return slot + (start & 15) + (size_t)i * a.row_bytes;
}

// WT: ggml type; EXACT: float path; NB: batch rows compiled for (a.nb <= NB)
template <int WT, bool EXACT, int NB>
__global__ void __launch_bounds__(EXACT ? kLmhThreads : kLmhInt8Threads,
                                  (!EXACT && (NB <= 2 || WT != 14)) ? 2 : 1)
    lmh_kernel(const LmhArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* ring = smem;
  uint8_t* act = ring + (size_t)a.nst * a.slot_bytes;
  float* terms = reinterpret_cast<float*>(act + a.act_bytes);
  const int tchains = EXACT ? 0 : a.gchains;
  uint64_t* full = reinterpret_cast<uint64_t*>(
      reinterpret_cast<uint8_t*>(terms) + (size_t)2 * tchains * a.tpitch * sizeof(float) + 16);
  full = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(full) + 7) & ~uintptr_t(7));
  __shared__ int s_timeout;
  __shared__ int s_issued;  // tiles whose copies were started

  const int tid = threadIdx.x;
  const int my_tiles = (a.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  if (tid == 0) {
    s_timeout = 0;
    for (int s = 0; s < a.nst; ++s) mbar_init(&full[s], 1);
    if constexpr (!EXACT) {
      // term table handoff: full[4 + buf] (term threads -> replay warp),
      // full[6 + buf] (replay warp -> term threads)
      mbar_init(&full[4], kLmhTermThreads);
      mbar_init(&full[5], kLmhTermThreads);
      mbar_init(&full[6], 32);
      mbar_init(&full[7], 32);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) {
    int k = 0;
    for (; k < a.nst && k < my_tiles; ++k)
      issue_tile(a, (int)blockIdx.x + k * (int)gridDim.x, ring + (size_t)k * a.slot_bytes, &full[k]);
    s_issued = k;
  }
  // activations into shared memory (read by every tile)
  if constexpr (EXACT) {
    float* xs = reinterpret_cast<float*>(act);
    for (int i = tid; i < a.nb * a.cols; i += (int)blockDim.x) xs[i] = a.x[i];
  } else {
    // quantizeAct (quant.nim:646-662) of this launch's batch rows, straight
    // into shared memory: one warp per activation block of bl values
    const int bl = (WT == 14) ? 256 : 32;
    const int nblocks = a.nb * (a.cols / bl);
    int8_t* qs = reinterpret_cast<int8_t*>(act);
    float* ds = reinterpret_cast<float*>(act + (size_t)a.nb * a.cols);
    const int nwarps = (int)blockDim.x >> 5, wl = tid & 31;
    // loads for several blocks go out together (L2 latency once per chunk)
    constexpr int kPer = 8;                 // values per lane in flight
    constexpr int kBlk = (WT == 14) ? 1 : kPer;  // blocks per chunk
    constexpr int kVals = (WT == 14) ? 8 : 1;    // values per lane per block
    for (int base = (tid >> 5) * kBlk; base < nblocks; base += nwarps * kBlk) {
      float v[kPer];
#pragma unroll
      for (int u = 0; u < kPer; ++u) {
        const int blk = base + u / kVals;
        v[u] = blk < nblocks ? a.x[(size_t)blk * bl + (u % kVals) * 32 + wl] : 0.0f;
      }
#pragma unroll
      for (int ub = 0; ub < kBlk; ++ub) {
        const int blk = base + ub;
        if (blk >= nblocks) break;  // warp-uniform
        float amax = 0.0f;
        bool bad = false;
#pragma unroll
        for (int u = 0; u < kVals; ++u) {
          bad |= !isfinite(v[ub * kVals + u]);
          amax = fmaxf(amax, fabsf(v[ub * kVals + u]));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (__any_sync(0xffffffffu, bad) && wl == 0 && blockIdx.x == 0)
          set_status(a.status, NLS_ERR_NAN_LOGITS);
        const float d = amax / 127.0f;
        const float id = d > 0.0f ? 1.0f / d : 0.0f;
        if (wl == 0) ds[blk] = d;
#pragma unroll
        for (int u = 0; u < kVals; ++u) {
          const float q0 = v[ub * kVals + u] * id;
          const int q = q0 >= 0.0f ? (int)(q0 + 0.5f) : -(int)(-q0 + 0.5f);
          qs[(size_t)blk * bl + u * 32 + wl] = (int8_t)q;
        }
      }
    }
  }
  __syncthreads();

  // fixed mapping (int8 path): term thread j = tid - 32 keeps block fb's
  // activations of every batch row in registers and visits rows
  // fr, fr + fg, fr + 2 fg, ... of each tile (Q6_K: four lanes per block)
  constexpr bool kPair = (WT == 14 && NB == 1);  // Q6_K, one batch row: two lanes per block
  int av[NB][16];
  float dav[NB];
  int asum[NB][4];  // Q4_0: [b][0] = sum of the block's 32 values; Q6_K: per 16
  int avp[kPair ? 32 : 1];
  int asp[kPair ? 8 : 1];
  int fb = 0, fr = 0, fg = 1, fq = 0;
  if constexpr (!EXACT) {
    if (a.fixed && tid >= 32) {
      const int j = tid - 32;
      // lanes per block lpb; block slots units = term threads / lpb; slot q
      // takes block q % nblk of rows q / nblk, q / nblk + fg, ...; slots past
      // the last whole row group stay idle
      constexpr int lpb = kPair ? 2 : (WT == 14 ? 4 : 1);
      constexpr int units = kLmhTermThreads / lpb;
      const int q = j / lpb;
      const int fb0 = q % a.nblk;
      fg = units / a.nblk;
      const int fr0 = q / a.nblk;
      const int32_t* aw = reinterpret_cast<const int32_t*>(act);
      const float* ds = reinterpret_cast<const float*>(act + (size_t)a.nb * a.cols);
      const int wpb = a.cols >> 2;
      if constexpr (kPair) {
        fq = j & 1;
        fb = fb0;
        fr = fr0;
        if (a.par) {
          // warp w holds the blocks of parity w & 1 of rgw row groups: slot u
          // (0..15) takes block 2 (u % hb) + (w & 1) of row group
          // (w >> 1) rgw + u / hb, hb = nblk / 2, rgw = 16 / hb
          const int w = j >> 5, u = (j & 31) >> 1, hb = a.nblk >> 1;
          fr = (w >> 1) * (16 / hb) + u / hb;
          fb = 2 * (u % hb) + (w & 1);
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int w0 = (128 * fq + 16 * half) >> 2;
#pragma unroll
          for (int m = 0; m < 4; ++m) {
#pragma unroll
            for (int k = 0; k < 4; ++k) avp[16 * half + 4 * m + k] = aw[fb * 64 + w0 + 8 * m + k];
            asp[4 * half + m] = bytesum(avp[16 * half + 4 * m]) + bytesum(avp[16 * half + 4 * m + 1]) +
                                bytesum(avp[16 * half + 4 * m + 2]) + bytesum(avp[16 * half + 4 * m + 3]);
          }
        }
        dav[0] = ds[fb];
      } else if constexpr (WT == 14) {
        fq = j & 3;
        fb = fb0;
        fr = fr0;
        const int w0 = (128 * (fq >> 1) + 16 * (fq & 1)) >> 2;
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
          for (int m = 0; m < 4; ++m)
#pragma unroll
            for (int k = 0; k < 4; ++k)
              av[b][4 * m + k] = b < a.nb ? aw[b * wpb + fb * 64 + w0 + 8 * m + k] : 0;
          dav[b] = b < a.nb ? ds[b * (a.cols >> 8) + fb] : 0.0f;
#pragma unroll
          for (int m = 0; m < 4; ++m)
            asum[b][m] = bytesum(av[b][4 * m]) + bytesum(av[b][4 * m + 1]) +
                         bytesum(av[b][4 * m + 2]) + bytesum(av[b][4 * m + 3]);
        }
      } else {
        fb = fb0;
        fr = fr0;
        if (a.par) {
          // nblk / 32 warps per row group: warp w takes the blocks of parity
          // p of one 64-block segment: block 2 (32 seg + lane) + p
          const int w = j >> 5, wpr = a.nblk >> 5, within = w % wpr;
          fr = w / wpr;
          fb = 2 * (32 * (within >> 1) + (j & 31)) + (within & 1);
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
#pragma unroll
          for (int k = 0; k < 16; ++k) av[b][k] = (b < a.nb && k < 8) ? aw[b * wpb + fb * 8 + k] : 0;
          dav[b] = b < a.nb ? ds[b * (a.cols >> 5) + fb] : 0.0f;
          int t8 = 0;
#pragma unroll
          for (int k = 0; k < 8; ++k) t8 += bytesum(av[b][k]);
          asum[b][0] = t8;
          asum[b][1] = asum[b][2] = asum[b][3] = 0;
        }
      }
    }
  }

  if (fr >= fg) fr = 1 << 30;  // an idle block slot (past the last whole row group)

  const float* xs = reinterpret_cast<const float*>(act);
  const int32_t* aqw = reinterpret_cast<const int32_t*>(act);
  const float* ads = reinterpret_cast<const float*>(act + (size_t)a.nb * a.cols);
  const int warp = tid >> 5, lane = tid & 31;

  if constexpr (EXACT) {
    for (int k = 0; k < my_tiles; ++k) {
      const int t = (int)blockIdx.x + k * (int)gridDim.x;
      const RingPos rp = ring_pos(k, a.nst);
      uint8_t* slot = ring + (size_t)rp.slot * a.slot_bytes;
      const int r0 = t * a.R;
      const int nr = min(a.R, a.rows - r0);
      // one lane per (row, batch row, accumulator): dotF32 (quant.nim:362-374)
      bool ok = !s_timeout;
      if (ok && !mbar_wait_bounded(&full[rp.slot], rp.parity)) {
        ok = false;
        s_timeout = 1;
        set_status(a.status, NLS_ERR_TIMEOUT);
      }
      const int c = tid >> 3, kk = tid & 7;
      const bool active = ok && c < nr * a.nb;
      const int row = active ? c / a.nb : 0, b = active ? c - row * a.nb : 0;
      float s = 0.0f;
      if (active) {
        const uint8_t* rowp = tile_row(a, slot, t, row);
        const float* xb = xs + (size_t)b * a.cols;
        const int n8 = a.cols & ~7;
        int e = kk;
#pragma unroll 4
        for (; e < n8; e += 8) s = s + wval<WT>(rowp, e) * xb[e];
        if (kk == 0)
          for (e = n8; e < a.cols; ++e) s = s + wval<WT>(rowp, e) * xb[e];
      }
      // every lane takes part in the 8-lane shuffles
      const float s1 = __shfl_down_sync(0xffffffffu, s, 1, 8);
      const float s2 = __shfl_down_sync(0xffffffffu, s, 2, 8);
      const float s3 = __shfl_down_sync(0xffffffffu, s, 3, 8);
      const float s4 = __shfl_down_sync(0xffffffffu, s, 4, 8);
      const float s5 = __shfl_down_sync(0xffffffffu, s, 5, 8);
      const float s6 = __shfl_down_sync(0xffffffffu, s, 6, 8);
      const float s7 = __shfl_down_sync(0xffffffffu, s, 7, 8);
      if (active && kk == 0) {
        float r = s + s1;
        r = r + (s2 + s3);
        r = r + (s4 + s5);
        r = r + (s6 + s7);
        a.y[(size_t)b * a.ldy + r0 + row] = r;
      }
      __syncthreads();
      if (tid == 0 && k + a.nst < my_tiles && !s_timeout) {
        fence_proxy_async_smem();
        issue_tile(a, t + a.nst * (int)gridDim.x, slot, &full[rp.slot]);
        s_issued = k + a.nst + 1;
      }
    }
  } else {
    // Warp-specialised pipeline. Warps 1..8 compute the block terms of each
    // tile into the term table of its group (gtiles tiles, gchains sums) and
    // recycle ring slots among themselves; warp 0 replays each group's sums
    // in block order (two per lane) while they go on with the next group.
    uint64_t* tfull = full + 4;
    uint64_t* tempty = full + 6;
    const int cpt = a.R * a.nb;  // sums per full tile
    const int ngroups = (my_tiles + a.gtiles - 1) / a.gtiles;
    if (warp == 0) {
      for (int g = 0; g < ngroups; ++g) {
        const int buf = g & 1;
        bool ok = !s_timeout;
        if (ok && !mbar_wait_bounded(&tfull[buf], (uint32_t)((g >> 1) & 1))) {
          ok = false;
          s_timeout = 1;
          set_status(a.status, NLS_ERR_TIMEOUT);
        }
        if (ok) {
          const float* Tg = terms + (size_t)buf * a.gchains * a.tpitch;
          const int k0 = g * a.gtiles;
          const int nsum = min(a.gtiles, my_tiles - k0) * cpt;
          const int c0 = lane, c1 = lane + 32;
          const float* T0 = Tg + (size_t)min(c0, a.gchains - 1) * a.tpitch;
          const float* T1 = Tg + (size_t)min(c1, a.gchains - 1) * a.tpitch;
          // the reference's block-order fp32 sums (quant.nim:762-786, :731-760)
          float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll 8
          for (int ib = 0; ib < a.nblk; ++ib) {
            acc0 = acc0 + T0[ib];
            acc1 = acc1 + T1[ib];
          }
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const int c = m ? c1 : c0;
            if (c >= nsum) break;
            const int pos = c / cpt, w = c - pos * cpt;
            const int row = w / a.nb, b = w - row * a.nb;
            const int r = ((int)blockIdx.x + (k0 + pos) * (int)gridDim.x) * a.R + row;
            if (r < a.rows) a.y[(size_t)b * a.ldy + r] = m ? acc1 : acc0;
          }
        }
        __syncwarp();
        mbar_arrive(&tempty[buf]);
      }
    } else {
      for (int k = 0; k < my_tiles; ++k) {
        const int t = (int)blockIdx.x + k * (int)gridDim.x;
        const RingPos rp = ring_pos(k, a.nst);
        uint8_t* slot = ring + (size_t)rp.slot * a.slot_bytes;
        const int r0 = t * a.R;
        const int nr = min(a.R, a.rows - r0);
        const int g = k / a.gtiles, pos = k - g * a.gtiles, buf = g & 1;
        float* T = terms + (size_t)buf * a.gchains * a.tpitch + (size_t)pos * cpt * a.tpitch;
        bool ok = !s_timeout;
        // the replay of group g - 2 has released this term buffer
        if (ok && pos == 0 && g >= 2 &&
            !mbar_wait_bounded(&tempty[buf], (uint32_t)(((g >> 1) - 1) & 1))) {
          ok = false;
          s_timeout = 1;
          set_status(a.status, NLS_ERR_TIMEOUT);
        }
        if (ok && !mbar_wait_bounded(&full[rp.slot], rp.parity)) {
          ok = false;
          s_timeout = 1;
          set_status(a.status, NLS_ERR_TIMEOUT);
        }
        if (ok && a.fixed) {
          // two rows per pass for independent work in flight
          const unsigned gmask = kPair ? (0x3u << (lane & ~1)) : (0xFu << (lane & ~3));
          for (int row = fr; row < nr; row += 2 * fg) {
            const int row2 = row + fg;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int rr = u ? row2 : row;
              if (rr >= nr) break;
              const uint8_t* rowp = tile_row(a, slot, t, rr);
              float* Tp = T + (size_t)rr * a.nb * a.tpitch + fb;
              if constexpr (WT == 8) {
                // (warp-uniform when a.par: the block start is 4-aligned for even fb)
                if (a.par) {
                  if (fb & 1) term_q8_0_reg<NB, 2>(rowp + fb * 34, av, dav, a.nb, Tp, a.tpitch);
                  else term_q8_0_reg<NB, 0>(rowp + fb * 34, av, dav, a.nb, Tp, a.tpitch);
                } else {
                  term_q8_0_reg<NB>(rowp + fb * 34, av, dav, a.nb, Tp, a.tpitch);
                }
              }
              else if constexpr (WT == 2) term_q4_0_reg<NB>(rowp + fb * 18, av, dav, asum, a.nb, Tp, a.tpitch);
              else if constexpr (kPair) {
                // (a warp-uniform branch when a.par: all its blocks share a parity)
                if (a.par && !(fb & 1)) term_q6_k_pair<true>(rowp + fb * 210, fq, avp, dav[0], asp, Tp, gmask);
                else term_q6_k_pair<false>(rowp + fb * 210, fq, avp, dav[0], asp, Tp, gmask);
              }
              else term_q6_k_reg<NB>(rowp + fb * 210, fq, av, dav, asum, a.nb, Tp, a.tpitch, gmask);
            }
          }
        } else if (ok) {
          const int items = nr * a.nblk;
          for (int it = tid - 32; it < items; it += (int)blockDim.x - 32) {
            const int row = it / a.nblk, ib = it - row * a.nblk;
            const uint8_t* rowp = tile_row(a, slot, t, row);
            float* Tp = T + (size_t)row * a.nb * a.tpitch + ib;
            if constexpr (WT == 8) terms_q8_0<NB>(rowp + ib * 34, ib, a, aqw, ads, Tp, a.tpitch);
            else if constexpr (WT == 2) terms_q4_0<NB>(rowp + ib * 18, ib, a, aqw, ads, Tp, a.tpitch);
            else terms_q6_k<NB>(rowp + ib * 210, ib, a, aqw, ads, Tp, a.tpitch);
          }
        }
        // all term threads are done with the slot: refill it
        asm volatile("bar.sync 1, %0;" ::"r"(kLmhTermThreads) : "memory");
        if (tid == 32 && k + a.nst < my_tiles && !s_timeout) {
          fence_proxy_async_smem();
          issue_tile(a, t + a.nst * (int)gridDim.x, slot, &full[rp.slot]);
          s_issued = k + a.nst + 1;
        }
        if (pos == a.gtiles - 1 || k == my_tiles - 1) mbar_arrive(&tfull[buf]);
      }
    }
  }
  // a wait that ran out may leave a copy in flight: drain it (bounded)
  __syncthreads();
  if (tid == 0 && s_timeout) {
    for (int k = max(0, s_issued - a.nst); k < s_issued; ++k) {
      const RingPos rp = ring_pos(k, a.nst);
      (void)mbar_wait_bounded(&full[rp.slot], rp.parity);
    }
  }
}

int block_values(int wt) {
  switch (wt) {
    case 0: case 1: return 1;
    case 2: case 8: return 32;
    case 14: return 256;
    default: return 0;
  }
}

int block_bytes(int wt) {
  switch (wt) {
    case 0: return 4;
    case 1: return 2;
    case 2: return 18;
    case 8: return 34;
    case 14: return 210;
    default: return 0;
  }
}

template <int WT, bool EXACT, int NB>
cudaError_t launch_one(const LmhArgs& a, int grid, size_t smem, cudaStream_t st) {
  auto fn = lmh_kernel<WT, EXACT, NB>;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  fn<<<grid, EXACT ? kLmhThreads : kLmhInt8Threads, smem, st>>>(a);
  return cudaGetLastError();
}

template <int WT>
cudaError_t dispatch(const LmhArgs& a, bool exact, int grid, size_t smem, cudaStream_t st) {
  if (exact || WT == 0 || WT == 1) {
    if constexpr (WT == 0 || WT == 1 || WT == 2 || WT == 8 || WT == 14)
      return launch_one<WT, true, 1>(a, grid, smem, st);
  }
  if constexpr (WT == 2 || WT == 8 || WT == 14) {
    if (a.nb <= 1) return launch_one<WT, false, 1>(a, grid, smem, st);
    if (a.nb <= 2) return launch_one<WT, false, 2>(a, grid, smem, st);
    return launch_one<WT, false, 4>(a, grid, smem, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

int lm_head_row_bytes(int wtype, int64_t cols, int64_t* out) {
  const int bv = block_values(wtype);
  if (bv == 0 || cols < 1 || cols % bv != 0) return 0;
  *out = cols / bv * block_bytes(wtype);
  return 1;
}

bool lm_head_int8_path(int wtype, int cols, int nb, bool exact) {
  const int bl = (wtype == 14) ? 256 : (wtype == 8 || wtype == 2) ? 32 : 0;
  return !exact && bl > 0 && cols % bl == 0 && (nb <= 4 || wtype != 8);
}

cudaError_t launch_lm_head(const uint8_t* w, int wtype, int rows, int cols, const float* x, int nb,
                           int path_nb, float* y, bool exact, int* status, int sm_count,
                           unsigned long long wait_ns, uint8_t* act_scratch, cudaStream_t st) {
  int64_t rb = 0;
  if (!lm_head_row_bytes(wtype, cols, &rb) || rows < 1 || nb < 1) return cudaErrorInvalidValue;
  const bool int8 = lm_head_int8_path(wtype, cols, path_nb, exact);
  // the float path, tiled across batch rows (nls_lmhead_float.cu)
  if (!int8 && lm_head_float_tiled(wtype, cols, rb) && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      (nb > 1 || wtype != 1))
    return launch_lm_head_float(w, wtype, rb, rows, cols, x, nb, y, rows, sm_count, st);
  // Q6_K / Q8_0 / Q4_0 on the int8 path at 8 or more batch rows: the same exact
  // arithmetic on the tensor cores, the weights read once per 16 batch rows
  // (nls_lmhead_mma.cu); a tail of fewer than 8 rows takes the path below
  int b_first = 0;
  if (int8 && act_scratch && lm_head_mma_path(wtype, cols, nb)) {
    const int lo = lm_head_mma_min_rows(wtype);
    const int tail = (nb % 16 < lo) ? nb % 16 : 0;
    const int nm = nb - tail;
    cudaError_t e = launch_lm_head_mma(w, wtype, rb, rows, cols, x, nm, y, rows, status, sm_count, wait_ns, act_scratch, st);
    if (e != cudaSuccess || tail == 0) return e;
    b_first = nm;
  }
  const int bl = (wtype == 14) ? 256 : 32;
  // the int8 path's warps read consecutive blocks of one row, so its tiles
  // need no padding (one copy per tile); the float path pads rows so that
  // its 8-lane groups of different rows fall in different banks
  const bool padded = (rb % 16) == 0 && !int8;
  const int pitch = padded ? (int)(((rb + 127) & ~int64_t(127)) + 32) : (int)rb;
  const int unit = padded ? pitch : (int)rb;
  // batch rows per launch: the int8 path keeps a block's activations of every
  // batch row in registers; the float path keeps x in shared memory
  const int nbt_max = int8 ? kLmhInt8MaxNb : std::max(1, std::min(32, (64 * 1024) / (cols * 4)));
  for (int b0 = b_first; b0 < nb; b0 += nbt_max) {
    const int nbt = std::min(nbt_max, nb - b0);
    const bool two = int8 && (nbt <= 2 || wtype != 14);
    const size_t smem_max = two ? kLmhSmemMax2 : kLmhSmemMax;
    const int slot_target = two ? kLmhSlotTarget2 : kLmhSlotTarget1;
    const int gmax = two ? kLmhGroupChains2 : kLmhGroupChains1;
    LmhArgs a{};
    a.w = w;
    a.row_bytes = rb;
    a.rows = rows;
    a.cols = cols;
    a.nblk = int8 ? cols / bl : cols;
    a.nb = nbt;
    a.x = x + (size_t)b0 * cols;
    a.y = y + (size_t)b0 * rows;
    a.ldy = rows;
    a.padded = padded ? 1 : 0;
    a.pitch = pitch;
    a.status = status;
    a.act_bytes = int8 ? (int)(((size_t)nbt * cols + (size_t)nbt * (cols / bl) * 4 + 15) & ~size_t(15))
                       : (int)(((size_t)nbt * cols * 4 + 15) & ~size_t(15));
    a.tpitch = int8 ? ((cols / bl) | 1) : 0;
    const int lpb = (wtype == 14) ? (nbt == 1 ? 2 : 4) : 1;  // lanes per block
    a.fixed = (int8 && lpb * (cols / bl) <= kLmhTermThreads) ? 1 : 0;
    {
      // parity-uniform warps: every row base is 4-byte aligned (rb % 4 == 0)
      // and a warp's 16 slots are whole groups of same-parity blocks
      const int nblk = cols / bl, hb = nblk / 2;
      a.par = (a.fixed && wtype == 14 && nbt == 1 && rb % 4 == 0 && nblk % 2 == 0 && hb >= 1 &&
               16 % hb == 0) ? 1 : 0;
      // Q8_0: nblk / 32 warps per row group, an even number (whole 64-block
      // segments, one parity per warp)
      if (a.fixed && wtype == 8 && rb % 4 == 0 && nblk % 64 == 0) a.par = 1;
    }
    auto slot_for = [&](int r) {
      return (int)((padded ? (int64_t)r * pitch : (int64_t)r * rb + 32 + 4) + 15) & ~15;
    };
    // tiles per replay group: up to gmax sums, and a term table (two
    // buffers) that leaves room for two ring slots
    auto gtiles_for = [&](int r) {
      int g = std::max(1, gmax / (r * nbt));
      const size_t per = (size_t)2 * r * nbt * a.tpitch * sizeof(float);
      const size_t other = (size_t)a.act_bytes + 2 * (size_t)slot_for(r) + 128;
      while (g > 1 && other + g * per > smem_max) --g;
      return g;
    };
    auto fixed_for = [&](int r) {
      const size_t terms = int8 ? (size_t)2 * gtiles_for(r) * r * nbt * a.tpitch * sizeof(float) : 0;
      return (size_t)a.act_bytes + terms + 16 + 8 + 8 * 8 + 16;
    };
    // int8 path: slots of about slot_target bytes, R x nbt sums per tile;
    // float path: as many rows as 256 lanes take (8 per sum) that fit twice
    int R = int8 ? std::max(1, slot_target / unit) : kLmhThreads / 8;
    const int rmax = std::max(1, (int8 ? kLmhMaxChains : kLmhThreads / 8) / nbt);
    R = std::min(R, rmax);
    if (a.fixed) {
      // term thread fr takes rows fr, fr + fg, fr + 2 fg, ... of a tile, so a
      // tile costs ceil(R / fg) rows of work per thread: make R a multiple of
      // fg, rounded up where that is close and fits, else down where that
      // halves the work per thread (a tile also has a fixed cost, so a
      // smaller tile only pays off then)
      const int fg = kLmhTermThreads / lpb / (cols / bl);
      const int Ru = (R + fg - 1) / fg * fg;
      if (Ru - R <= fg / 2 && Ru <= rmax && fixed_for(Ru) + 2 * (size_t)slot_for(Ru) <= smem_max)
        R = Ru;
      else if (R > fg && R < 2 * fg)
        R = fg;
    }
    R = std::min(R, rows);
    while (R > 1 && fixed_for(R) + 2 * (size_t)slot_for(R) > smem_max) --R;
    a.R = R;
    a.ntiles = (rows + R - 1) / R;
    a.gtiles = int8 ? gtiles_for(R) : 1;
    a.gchains = int8 ? a.gtiles * R * nbt : 0;
    a.slot_bytes = slot_for(R);
    const size_t fixed = fixed_for(R);
    int nst = 4;
    while (nst > 2 && fixed + (size_t)nst * a.slot_bytes > smem_max) --nst;
    if (fixed + (size_t)nst * a.slot_bytes > smem_max) return cudaErrorInvalidValue;
    a.nst = nst;
    const size_t smem = fixed + (size_t)nst * a.slot_bytes;
    const int grid = std::min(a.ntiles, sm_count * (two ? 2 : 1));
    cudaError_t e;
    switch (wtype) {
      case 0: e = dispatch<0>(a, true, grid, smem, st); break;
      case 1: e = dispatch<1>(a, true, grid, smem, st); break;
      case 2: e = dispatch<2>(a, !int8, grid, smem, st); break;
      case 8: e = dispatch<8>(a, !int8, grid, smem, st); break;
      case 14: e = dispatch<14>(a, !int8, grid, smem, st); break;
      default: e = cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace nls
