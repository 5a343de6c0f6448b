// nls_lmhead_mma.cu -- the output projection for Q6_K, Q8_0 and Q4_0 weights at 8
// to 16 batch rows per launch on the int8 path, on the 5th-generation
// tensor cores.
//
// The reference's integer path (quantizeAct quant.nim:646-662, dotQ6K
// quant.nim:731-760, dotQ8_0i quant.nim:762-772, matmulTask model.nim:144-155)
// computes per weight row r, batch row b and weight block exact integer
// sums of int8 x int8 products, then fp32 terms block after block:
//  * Q6_K (256-value blocks): sumi = sum_j sc_j * s_j over 16 sub-blocks of
//    16 values, s_j = sum (q_l - 32) * a_l, int8 scales sc_j; then
//    acc += (d_a * d_w) * float(sumi);
//  * Q8_0 and Q4_0 (32-value blocks, activations quantized in blocks of
//    32): s = sum q_l * a_l (Q4_0: q_l a nibble minus 8); then
//    acc += (d_w * d_a) * float(s).
// The s_j and s are int8 x int8 -> int32 contractions (|s| <= 32 * 128 * 127),
// which tcgen05.mma kind::i8 computes exactly; the scale products, the
// float conversion and the fp32 operations are the reference's, in its
// order, on the CUDA cores. (Q8_0 takes the int8 path at more than 4 batch
// rows only when the rows are separate sequences, model.nim:185.)
//
// One CTA per SM, persistent over tiles of 128 weight rows, warp-specialised
// (warp 0; kUnpackWarps unpackers; kSumWarps summers). A step covers 256
// values of every row of the tile (one Q6_K block, eight Q8_0 or Q4_0
// blocks). Per (tile, step):
//  * warp 0 stages the tile's bytes of the step two steps ahead into shared
//    memory: one tensor-map copy of a 128-row box (the weights seen as rows
//    of 8-byte elements), or, where a row is not a multiple of 16 bytes, one
//    bulk copy per row;
//  * the unpackers lay the step's weights out as the A operand of its parity
//    (one of two buffers; no-swizzle K-major layout, 8-row x 16-byte core
//    matrices) and record the scales. Q6_K: a thread unpacks (row, quarter)
//    units of the block -- four sub-blocks of 16 values, q - 32 as int8 --
//    even sub-blocks as the first 16 values of a 32-value K step, odd ones
//    as the second, and the other half of both is one shared block of zeros
//    that the descriptors point at. Q8_0 / Q4_0: a thread lays out two
//    blocks of a row, 16 int8 values per half (Q4_0: nibbles minus 8), one
//    K step per block;
//  * warp 0 issues the step's MMAs (M = 128 rows, N = 16 batch rows, K = 32;
//    16 for Q6_K, sub-block j into TMEM columns 16j .. 16j+15, 8 for the
//    others, block i into columns 16i ..) into one of two regions and
//    commits them to an mbarrier;
//  * the summers read, for the 32 weight rows of their TMEM lane quarter
//    (warp % 4) and a share of the 16 batch rows, the step's sums and form
//    the fp32 terms in block order, while the unpackers work on later steps.
// All hand-offs are mbarriers (staging -> unpackers -> warp 0 -> summers ->
// warp 0), every wait bounded. The activations are quantized once per launch
// by a small kernel before it (lmh_mma_quant_kernel, into device scratch in
// the operand layout; batch rows past nb are zeros) whose programmatic
// dependent this kernel is: its set-up and first weight copies run while
// that kernel does, then one bulk copy brings the operand and the scales.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>

#include "nls_kernels.h"
#include "nls_tma.cuh"

namespace nls {

namespace {

constexpr int kMmaRows = 128;    // weight rows per tile (MMA M)
constexpr int kMmaN = 16;        // batch rows per launch (MMA N)
constexpr int kQ6Bytes = 210;    // a Q6_K block
// Q6_K's A buffer: even sub-blocks [0, 16 KB), a 2 KB block of zeros, odd
// ones [18 KB, 34 KB); K step i of a parity at + 2 KB * i, row r at + 16 r
constexpr int kAEven = 0, kAZero = 16384, kAOdd = 18432;
// per-step scales: written by a step's unpack, read by its sums; the
// unpackers run up to three steps ahead of the summers (step s is unpacked
// once the MMAs of step s - 2 have completed, which were issued once the
// sums of step s - 4 had read their TMEM region)
constexpr int kSlots = 4;

// offset of the 16 values of row r, sub-block j inside a Q6_K A buffer
__device__ __forceinline__ int a_off(int r, int j) { return ((j & 1) ? kAOdd : kAEven) + (j >> 1) * 2048 + r * 16; }
// offset of byte k of batch row b inside the activation operand (K steps of
// 32 values, 512 bytes each for 16 rows)
__device__ __forceinline__ int b_off(int b, int k) {
  return (k >> 5) * (kMmaN * 32) + (b >> 3) * 256 + ((k >> 4) & 1) * 128 + (b & 7) * 16 + (k & 15);
}

// shared-memory matrix descriptor: no swizzle, K-major; lbo: from a row's
// first 16 bytes of K to its second, sbo: from 8 rows to the next 8
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version of sm_100
  return d;
}

// instruction descriptor: s32 accumulator, s8 x s8, both K-major, N = 16, M = 128
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kMmaN >> 3) << 17) |
                            ((uint32_t)(kMmaRows >> 4) << 24);

// D = A . B^T (no accumulation into the previous contents)
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t da, uint64_t db) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(kIdesc)
      : "memory");
}

// N (4 or 8) consecutive TMEM columns of this warp's 32 lanes
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]) {
  if constexpr (N == 4) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  } else {
    static_assert(N == 8, "4 or 8 columns");
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
  }
}

// 16 bytes at a 2-byte aligned shared address, as four words (reads the
// aligned words inside [p - 2, p + 18))
__device__ __forceinline__ void ld16s(const uint8_t* p, uint32_t (&w)[4]) {
  const uint32_t* a = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(p) & ~uintptr_t(3));
  const uint32_t sel = (reinterpret_cast<uintptr_t>(p) & 2) ? 0x5432u : 0x3210u;
  uint32_t x[5];
#pragma unroll
  for (int k = 0; k < 5; ++k) x[k] = a[k];
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] = __byte_perm(x[k], x[k + 1], sel);
}

struct MmaArgs {
  const uint8_t* w;  // rows x row_bytes, 16-byte aligned
  int64_t row_bytes;
  int64_t total;     // rows * row_bytes
  int rows, cols, nblk;
  int nb;            // batch rows of this launch, <= 16
  const uint8_t* q;  // the quantized activations in the B operand layout (16 x cols bytes)
  const float* dq;   // their block scales d_a [16][cols / block]
  float* y;          // y[b * ldy + r]
  int64_t ldy;
  int ntiles;
  int tiled;         // the weights have a tensor map (row_bytes % 16 == 0)
  unsigned long long wait_ns;
  int* status;
};

// 2-D tensor copy (no multicast): box {x .. , y ..} of the map into shared
// memory, completing on the mbarrier
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <int WT>
struct MmaType;
// A step covers 256 values of a weight row (one K step of 32 per MMA).
template <>
struct MmaType<14> {                 // Q6_K: one 210-byte block per step
  static constexpr int kBL = 256;    // activation block (quantizeAct)
  static constexpr int kStepBytes = kQ6Bytes;
  static constexpr int kRawRow = 240;  // the block and its 16-byte alignment
  static constexpr int kDw = 1;      // d per row and step
  static constexpr int kScWords = 4; // sub-block scales per row and step
  static constexpr int kRegion = 256;  // TMEM columns per step: 16 sub-blocks x 16
  static constexpr int kAStage = 34816;
  static constexpr int kUnpackWarps = 8, kSumWarps = 8;  // (measured: above 4 + 8, 4 + 16, 8 + 16)
};
template <>
struct MmaType<8> {                  // Q8_0: eight 34-byte blocks per step
  static constexpr int kBL = 32;
  static constexpr int kStepBytes = 8 * 34;
  static constexpr int kRawRow = 8 * 34;  // 16-byte aligned (rows of whole steps)
  static constexpr int kDw = 8;
  static constexpr int kScWords = 0;
  static constexpr int kRegion = 128;  // 8 blocks x 16
  static constexpr int kAStage = 32768;  // block i: [its first 16 values of every row][its second 16]
  static constexpr int kUnpackWarps = 4, kSumWarps = 8;  // (measured: 4 + 8 above 8 + 8, 4 + 16, 8 + 16)
};
template <>
struct MmaType<2> {                  // Q4_0: eight 18-byte blocks per step
  static constexpr int kBL = 32;
  static constexpr int kStepBytes = 8 * 18;
  static constexpr int kRawRow = 8 * 18;
  static constexpr int kDw = 8;
  static constexpr int kScWords = 0;
  static constexpr int kRegion = 128;
  static constexpr int kAStage = 32768;
  static constexpr int kUnpackWarps = 4, kSumWarps = 8;
};

template <int WT>
__host__ __device__ constexpr size_t mma_smem(int cols) {
  using T = MmaType<WT>;
  return (size_t)(cols / 32) * (kMmaN * 32) + 2 * (size_t)T::kAStage + 2 * (size_t)kMmaRows * T::kRawRow +
         (size_t)kMmaN * (cols / T::kBL) * 4 + (size_t)kSlots * kMmaRows * T::kDw * 4 +
         (size_t)kSlots * kMmaRows * T::kScWords * 4 + 8 + 11 * 8 + 16 + 16;
}

// Q8_0: one thread lays out blocks 2Q and 2Q + 1 of a row from the 80 bytes
// at 64Q of its staged step (five 16-byte words W; block j's d at byte 34j,
// its values at 34j + 2). Q is uniform across the warp.
template <int Q>
__device__ __forceinline__ void q8_units(const uint32_t (&W)[20], uint8_t* ab, float* dslot, int rr, bool in) {
  uint32_t v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = __byte_perm(W[Q + k], W[Q + k + 1], 0x5432);  // block 2Q at 4Q + 2
  *reinterpret_cast<uint4*>(ab + 4096 * (2 * Q) + 16 * rr) = make_uint4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<uint4*>(ab + 4096 * (2 * Q) + 2048 + 16 * rr) = make_uint4(v[4], v[5], v[6], v[7]);
  // block 2Q + 1 at 4Q + 36 (word aligned)
  *reinterpret_cast<uint4*>(ab + 4096 * (2 * Q + 1) + 16 * rr) = make_uint4(W[Q + 9], W[Q + 10], W[Q + 11], W[Q + 12]);
  *reinterpret_cast<uint4*>(ab + 4096 * (2 * Q + 1) + 2048 + 16 * rr) =
      make_uint4(W[Q + 13], W[Q + 14], W[Q + 15], W[Q + 16]);
  const float d0 = __half2float(__ushort_as_half((unsigned short)(W[Q] & 0xFFFFu)));
  const float d1 = __half2float(__ushort_as_half((unsigned short)(W[Q + 8] >> 16)));
  dslot[(2 * Q) * kMmaRows + rr] = in ? d0 : 0.0f;
  dslot[(2 * Q + 1) * kMmaRows + rr] = in ? d1 : 0.0f;
}

// q - 8 as int8 for four packed nibbles q (q + 120 stays below 256 in every
// byte; its bit 7 flipped is q - 8 in two's complement)
__device__ __forceinline__ uint32_t nib_minus8(uint32_t v) { return (v + 0x78787878u) ^ 0x80808080u; }

// Q4_0 (dotQ4_0i quant.nim:774-786: values 0-15 of a block are the low
// nibbles of its 16 bytes, values 16-31 the high ones): blocks 2Q and 2Q + 1
// from the 48 bytes at 32Q of the staged step (block j's d at 18j, its
// bytes at 18j + 2).
template <int Q>
__device__ __forceinline__ void q4_units(const uint32_t (&W)[12], uint8_t* ab, float* dslot, int rr, bool in) {
  uint32_t b0[4], b1[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    b0[k] = __byte_perm(W[Q + k], W[Q + k + 1], 0x5432);  // block 2Q at 4Q + 2
    b1[k] = W[Q + 5 + k];                                   // block 2Q + 1 at 4Q + 20
  }
  uint32_t lo[4], hi[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    lo[k] = nib_minus8(b0[k] & 0x0F0F0F0Fu);
    hi[k] = nib_minus8((b0[k] >> 4) & 0x0F0F0F0Fu);
  }
  *reinterpret_cast<uint4*>(ab + 4096 * (2 * Q) + 16 * rr) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  *reinterpret_cast<uint4*>(ab + 4096 * (2 * Q) + 2048 + 16 * rr) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    lo[k] = nib_minus8(b1[k] & 0x0F0F0F0Fu);
    hi[k] = nib_minus8((b1[k] >> 4) & 0x0F0F0F0Fu);
  }
  *reinterpret_cast<uint4*>(ab + 4096 * (2 * Q + 1) + 16 * rr) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  *reinterpret_cast<uint4*>(ab + 4096 * (2 * Q + 1) + 2048 + 16 * rr) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  const float d0 = __half2float(__ushort_as_half((unsigned short)(W[Q] & 0xFFFFu)));
  const float d1 = __half2float(__ushort_as_half((unsigned short)(W[Q + 4] >> 16)));
  dslot[(2 * Q) * kMmaRows + rr] = in ? d0 : 0.0f;
  dslot[(2 * Q + 1) * kMmaRows + rr] = in ? d1 : 0.0f;
}

// quantizeAct (quant.nim:646-662) once per launch of 16 batch rows, with the
// type's blocks (256 values for Q6_K, 32 for the others), into the B operand
// layout in global memory (rows nb .. 15 zeros) and the block scales d_a:
// each thread takes 32 consecutive values, the G threads of a block
// (consecutive lanes) combine their maxima by shuffles. The projection
// kernel is its programmatic dependent: it is released at once and sets
// itself up while this grid runs.
template <int WT>
__global__ void __launch_bounds__(256) lmh_mma_quant_kernel(const float* x, int nb, int cols, uint8_t* q,
                                                            float* dq, int* status) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  using T = MmaType<WT>;
  constexpr int G = T::kBL / 32;
  const int lane = threadIdx.x & 31;
  const int per_row = cols / 32, nab = cols / T::kBL;
  const int units = kMmaN * per_row;  // a multiple of 8: whole blocks per warp
  const int nthreads = (int)(gridDim.x * blockDim.x);
  for (int base = (int)(blockIdx.x * blockDim.x + threadIdx.x) - lane; base < units; base += nthreads) {
    const int u = base + lane;
    const bool act = u < units;
    const int b = act ? u / per_row : 0, c = act ? u % per_row : 0;
    const bool real = act && b < nb;
    const float* xs = x + (size_t)b * cols + (size_t)c * 32;
    float v[32];
    if (real && (reinterpret_cast<uintptr_t>(xs) & 15) == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 f = reinterpret_cast<const float4*>(xs)[k];
        v[4 * k] = f.x;
        v[4 * k + 1] = f.y;
        v[4 * k + 2] = f.z;
        v[4 * k + 3] = f.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = real ? xs[k] : 0.0f;
    }
    float amax = 0.0f;
    bool bad = false;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      bad |= !isfinite(v[k]);
      amax = fmaxf(amax, fabsf(v[k]));
    }
#pragma unroll
    for (int o = 1; o < G; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicCAS(status, 0, NLS_ERR_NAN_LOGITS);
    if (act) {
      const float d = amax / 127.0f;
      const float id = d > 0.0f ? 1.0f / d : 0.0f;
      if (c % G == 0) dq[b * nab + c / G] = d;
      uint32_t qw[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint32_t wv = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float q0 = v[4 * k + e] * id;
          const int qi = q0 >= 0.0f ? (int)(q0 + 0.5f) : -(int)(-q0 + 0.5f);
          wv |= ((uint32_t)qi & 0xFFu) << (8 * e);
        }
        qw[k] = wv;
      }
      *reinterpret_cast<uint4*>(q + b_off(b, c * 32)) = make_uint4(qw[0], qw[1], qw[2], qw[3]);
      *reinterpret_cast<uint4*>(q + b_off(b, c * 32 + 16)) = make_uint4(qw[4], qw[5], qw[6], qw[7]);
    }
  }
}

template <int WT>
__global__ void __launch_bounds__(32 * (1 + MmaType<WT>::kUnpackWarps + MmaType<WT>::kSumWarps), 1)
    lmh_mma_kernel(const MmaArgs a,
                                                                const __grid_constant__ CUtensorMap wmap) {
  using T = MmaType<WT>;
  constexpr int kRawRow = T::kRawRow, kRawStage = kMmaRows * kRawRow, kAStage = T::kAStage;
  // warp 0: staging and the MMAs; warps 1 .. kUnpackWarps: the A operands
  // and scales of a step; the rest: the fp32 sums from TMEM
  constexpr int kUnpackWarps = T::kUnpackWarps, kSumWarps = T::kSumWarps;
  constexpr int kMmaThreads = 32 * (1 + kUnpackWarps + kSumWarps);
  constexpr int kUnpackParts = 16 / kUnpackWarps;  // (row, quarter) units per unpacker thread
  constexpr int EB = 16 / (kSumWarps / 4);          // batch rows per summer thread
  static_assert(kUnpackWarps % 4 == 0 && 16 % kUnpackWarps == 0 && kSumWarps % 4 == 0 && 16 % (kSumWarps / 4) == 0,
                "role split");
  constexpr int kTmemCols = 2 * T::kRegion;  // two regions: steps s and s + 1
  extern __shared__ __align__(1024) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kb_steps = a.cols / 32;
  const int nab = a.cols / T::kBL;                              // activation blocks per row
  uint8_t* bop = smem;                                          // activations: kb_steps x 512 B
  uint8_t* aop = bop + (size_t)kb_steps * (kMmaN * 32);         // 2 A buffers
  uint8_t* raw = aop + 2 * kAStage;                             // 2 x 128 rows x kRawRow B
  float* dsa = reinterpret_cast<float*>(raw + 2 * kRawStage);   // d_a [16][nab]
  float* dws = dsa + kMmaN * nab;                               // d_w [kSlots][kDw][128]
  uint32_t* scs = reinterpret_cast<uint32_t*>(dws + kSlots * kMmaRows * T::kDw);  // Q6_K sc [kSlots][128][4 words]
  uint64_t* bar = reinterpret_cast<uint64_t*>(
      (reinterpret_cast<uintptr_t>(scs + kSlots * kMmaRows * T::kScWords) + 7) & ~uintptr_t(7));
  uint64_t* full = bar;       // [2] raw buffer s & 1 holds step s (bulk copies)
  uint64_t* ready = bar + 2;  // [4] every unpacker has laid out step s (slot s % 4)
  uint64_t* done = bar + 6;   // [2] MMAs of step s completed (tcgen05.commit)
  uint64_t* tfree = bar + 8;  // [2] every summer has read TMEM region s & 1 for step s
  uint64_t* actbar = bar + 10;  // the activation operand and scales (bulk copies)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 11);
  int* s_fail = reinterpret_cast<int*>(tmem_holder + 1);
  int* s_last = s_fail + 1;    // the last step whose MMAs were issued
  int* s_staged = s_fail + 2;  // the last step whose copies were issued

  const int my_tiles = (a.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  // (tile, step in the row) of this CTA's step s, advanced step by step
  // (no division per step)
  struct Pos {
    int t, kb;
  };
  auto next = [&](Pos& q) {
    if (++q.kb == a.nblk) {
      q.kb = 0;
      q.t += (int)gridDim.x;
    }
  };
  const Pos first{(int)blockIdx.x, 0};
  const int nsteps = my_tiles * a.nblk;
  const int64_t last16 = a.total & ~int64_t(15);

  // warp 0 stages step s into raw buffer s & 1: row rr of the tile at
  // rr * kRawRow, the step's bytes from their 16-byte boundary on. With a
  // tensor map (the weights as rows of 8-byte elements, row_bytes apart) one
  // copy moves the 128 x kRawRow box (rows past the matrix and bytes past a
  // row read as zeros); otherwise one bulk copy per row, and a row whose copy
  // would pass the weights' last whole 16 bytes goes by plain loads before
  // the arrival.
  auto stage = [&](int s, Pos q) {
    if (s >= nsteps) return;
    const int t = q.t, kb = q.kb;
    uint8_t* dst = raw + (size_t)(s & 1) * kRawStage;
    if (a.tiled) {
      if (lane == 0) {
        const int x = ((kb * T::kStepBytes) >> 4) * 2;
        mbar_arrive_expect_tx(&full[s & 1], kRawStage);
        tma_load_2d(dst, &wmap, x, t * kMmaRows, &full[s & 1]);
        *s_staged = s;
      }
      return;
    }
    int64_t g[4];
    uint32_t bytes = 0;
    unsigned bulk = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int rr = lane + 32 * k;
      const int r = t * kMmaRows + rr;
      g[k] = ((int64_t)r * a.row_bytes + (int64_t)kb * T::kStepBytes) & ~int64_t(15);
      if (r >= a.rows) continue;
      if (g[k] + kRawRow <= last16) {
        bulk |= 1u << k;
        bytes += kRawRow;
      } else {
        uint8_t* d = dst + rr * kRawRow;
        for (int e = 0; e < kRawRow; ++e) d[e] = (g[k] + e < a.total) ? a.w[g[k] + e] : 0;
      }
    }
    bytes = __reduce_add_sync(0xffffffffu, bytes);
    __threadfence_block();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive_expect_tx(&full[s & 1], bytes);
      *s_staged = s;
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (bulk & (1u << k)) bulk_copy_g2s(dst + (lane + 32 * k) * kRawRow, a.w + g[k], kRawRow, &full[s & 1]);
  };

  if (tid == 0) {
    for (int k = 0; k < 11; ++k)
      mbar_init(&bar[k], (k >= 2 && k < 6) ? kUnpackWarps : (k >= 8 && k < 10) ? kSumWarps : 1);
    *s_fail = 0;
    *s_last = -1;
    *s_staged = -1;
    fence_mbar_init();
  }
  // zeros: both A buffers (Q6_K's zero blocks stay zero)
  for (int i = tid; i < 2 * kAStage / 16; i += kMmaThreads) reinterpret_cast<uint4*>(aop)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  if (warp == 0) {
    Pos q = first;
    stage(0, q);
    next(q);
    stage(1, q);
    // the activations, quantized by the launch this kernel depends on: wait
    // for that grid (everything above ran while it did), then one bulk copy
    // of the operand and one of the scales
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      const uint32_t qbytes = (uint32_t)kb_steps * (kMmaN * 32), dbytes = (uint32_t)(kMmaN * nab * 4);
      mbar_arrive_expect_tx(actbar, qbytes + dbytes);
      bulk_copy_g2s(bop, a.q, qbytes, actbar);
      bulk_copy_g2s(dsa, a.dq, dbytes, actbar);
    }
    __syncwarp();
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tbase = *tmem_holder;
  // the activations have landed (the default limit: the copies are real)
  bool fail = !mbar_wait_bounded(actbar, 0u, kWaitLimitNs);
  auto wait_bar = [&](uint64_t* b2, int s) -> bool {  // barrier b2[s & 1] completed for step s
    return mbar_wait_bounded(&b2[s & 1], (uint32_t)((s >> 1) & 1), a.wait_ns);
  };
  auto wait4 = [&](uint64_t* b4, int s) -> bool {  // barrier b4[s % 4] completed for step s
    return mbar_wait_bounded(&b4[s & 3], (uint32_t)((s >> 2) & 1), a.wait_ns);
  };

  if (fail) {
    // (the activations never landed: no role runs; the cleanup below drains
    // the staged copies)
  } else if (warp == 0) {
    // staging two steps ahead, and the MMAs of step s once every unpacker
    // has laid it out (which also frees raw buffer s & 1 for step s + 2) and
    // the sums of step s - 2 have read TMEM region s & 1
    Pos cur = first, st2 = first;
    next(st2);
    next(st2);
    for (int s = 0; s < nsteps; ++s, next(cur), next(st2)) {
      bool ok = true;
      if (lane == 0) ok = wait4(ready, s) && (s < 2 || wait_bar(tfree, s - 2)) && !*s_fail;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        fail = true;
        break;
      }
      stage(s + 2, st2);
      if (lane == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int kb = cur.kb;
        const uint32_t ab = smem_u32(aop) + (uint32_t)((s & 1) * kAStage);
        const uint32_t bb = smem_u32(bop) + (uint32_t)(kb * 8) * (kMmaN * 32);
        const uint32_t dreg = tbase + (uint32_t)((s & 1) * T::kRegion);
        // descriptors of K step i: the first's with the start address (bits
        // 0-13, in 16-byte units) and leading-byte offset (bits 16-29)
        // advanced; no field overflows (shared addresses are below 256 KB)
        const uint64_t db0 = smem_desc(bb, 128, 256);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint64_t db = db0 + (uint64_t)(i * (kMmaN * 32) / 16);
          if constexpr (WT == 14) {
            // even sub-block 2i: its values, then the zeros; odd 2i + 1: the
            // zeros, then its values
            const uint64_t de0 = smem_desc(ab + kAEven, kAZero - kAEven, 128);
            const uint64_t do0 = smem_desc(ab + kAZero, kAOdd - kAZero, 128);
            mma_i8(dreg + 32 * i, de0 + (uint64_t)(2048 * i / 16) - ((uint64_t)(2048 * i / 16) << 16), db);
            mma_i8(dreg + 32 * i + 16, do0 + ((uint64_t)(2048 * i / 16) << 16), db);
          } else {
            // block i: its first 16 values of every row, then its second 16
            const uint64_t da0 = smem_desc(ab, 2048, 128);
            mma_i8(dreg + 16 * i, da0 + (uint64_t)(4096 * i / 16), db);
          }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         smem_u32(&done[s & 1]))
                     : "memory");
        *s_last = s;
      }
      __syncwarp();
    }
  } else if (warp <= kUnpackWarps) {
    // unpackers: step s's weights into A buffer s & 1 once they have landed
    // and the MMAs of step s - 2 (the buffer's last readers) have completed
    const int uw = warp - 1;
    Pos cur = first;
    for (int s = 0; s < nsteps; ++s, next(cur)) {
      bool ok = wait_bar(full, s);
      if (ok && s >= 2) ok = wait_bar(done, s - 2);
      if (__any_sync(0xffffffffu, !ok)) {
        fail = true;
        break;
      }
      const int t = cur.t, kb = cur.kb;
      const uint8_t* rs = raw + (size_t)(s & 1) * kRawStage;
      uint8_t* ab = aop + (size_t)(s & 1) * kAStage;
      if constexpr (WT == 14) {
#pragma unroll 1
        for (int part = 0; part < kUnpackParts; ++part) {
          const int wi = (tid - 32) + 32 * kUnpackWarps * part;
          const int ur = wi >> 2, uh = (wi >> 1) & 1, uhalf = wi & 1;  // (row, quarter)
          const int r = t * kMmaRows + ur;
          const int64_t g = (int64_t)r * a.row_bytes + (int64_t)kb * kQ6Bytes;
          const uint8_t* blk = rs + ur * kRawRow + (int)(g & 15);
          uint32_t QA[4], QB[4], QH[4];
          ld16s(blk + 64 * uh + 16 * uhalf, QA);
          ld16s(blk + 64 * uh + 32 + 16 * uhalf, QB);
          ld16s(blk + 128 + 32 * uh + 16 * uhalf, QH);
          if (uh == 0 && uhalf == 0) {
            // this row's sub-block scales and d for the sums (rows past the
            // matrix: zeros)
            uint32_t sc4[4];
            ld16s(blk + 192, sc4);
            const bool in = r < a.rows;
            uint32_t* sd = scs + ((size_t)(s % kSlots) * kMmaRows + ur) * 4;
#pragma unroll
            for (int k = 0; k < 4; ++k) sd[k] = in ? sc4[k] : 0u;
            const uint32_t dwb = (uint32_t)blk[208] | ((uint32_t)blk[209] << 8);
            dws[(s % kSlots) * kMmaRows + ur] = in ? __half2float(__ushort_as_half((unsigned short)dwb)) : 0.0f;
          }
          // the four sub-blocks j = 8h + 2c + half of this quarter (dotQ6K's
          // q1..q4, quant.nim:744-747): the 6-bit value q, then q - 32 as int8
          // (q + 96 stays below 256 in every byte; its bit 7 flipped is
          // q - 32 in two's complement)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t lo4 = ((c & 1) ? QB[k] : QA[k]) >> ((c & 2) ? 4 : 0);
              const uint32_t q6 = (lo4 & 0x0F0F0F0Fu) | (((QH[k] >> (2 * c)) << 4) & 0x30303030u);
              v[k] = (q6 + 0x60606060u) ^ 0x80808080u;
            }
            *reinterpret_cast<uint4*>(ab + a_off(ur, 8 * uh + 2 * c + uhalf)) = make_uint4(v[0], v[1], v[2], v[3]);
          }
        }
      } else {
        // Q8_0 / Q4_0: a thread takes blocks 2q, 2q + 1 of kUnpackParts rows
        // (q uniform across the warp, 32 consecutive rows per warp and part,
        // so its 16-byte loads and stores are free of bank conflicts); block
        // j goes to K step j, values 0-15 then 16-31, as int8
        const int q = uw & 3, g = uw >> 2;
        float* dslot = dws + (size_t)(s % kSlots) * 8 * kMmaRows;
#pragma unroll 1
        for (int part = 0; part < kUnpackParts; ++part) {
          const int rr = 32 * (g + (kUnpackWarps / 4) * part) + lane;
          const bool in = t * kMmaRows + rr < a.rows;
          if constexpr (WT == 8) {
            const uint4* src = reinterpret_cast<const uint4*>(rs + rr * kRawRow + 64 * q);
            uint32_t W[20];
#pragma unroll
            for (int k = 0; k < 5; ++k) {
              const uint4 c4 = src[k];
              W[4 * k] = c4.x;
              W[4 * k + 1] = c4.y;
              W[4 * k + 2] = c4.z;
              W[4 * k + 3] = c4.w;
            }
            switch (q) {
              case 0: q8_units<0>(W, ab, dslot, rr, in); break;
              case 1: q8_units<1>(W, ab, dslot, rr, in); break;
              case 2: q8_units<2>(W, ab, dslot, rr, in); break;
              default: q8_units<3>(W, ab, dslot, rr, in); break;
            }
          } else {
            const uint4* src = reinterpret_cast<const uint4*>(rs + rr * kRawRow + 32 * q);
            uint32_t W[12];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
              const uint4 c4 = src[k];
              W[4 * k] = c4.x;
              W[4 * k + 1] = c4.y;
              W[4 * k + 2] = c4.z;
              W[4 * k + 3] = c4.w;
            }
            switch (q) {
              case 0: q4_units<0>(W, ab, dslot, rr, in); break;
              case 1: q4_units<1>(W, ab, dslot, rr, in); break;
              case 2: q4_units<2>(W, ab, dslot, rr, in); break;
              default: q4_units<3>(W, ab, dslot, rr, in); break;
            }
          }
        }
      }
      // the operands (async proxy: the MMAs) and the step's scales (the
      // summers, which also wait on this barrier) before the arrival
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[s % 4]);
    }
  } else {
    // summers: the sums of step p once its MMAs have completed; weight row em
    // of the tile (TMEM lane quarter warp % 4), batch rows eb0 .. eb0+EB-1
    const int sw = warp - 1 - kUnpackWarps;
    const int em = 32 * (warp & 3) + lane, eb0 = EB * (sw >> 2);
    float acc[EB];
#pragma unroll
    for (int e = 0; e < EB; ++e) acc[e] = 0.0f;
    Pos cur = first;
    for (int p = 0; p < nsteps; ++p, next(cur)) {
      bool ok = wait_bar(done, p);
      if (ok) ok = wait4(ready, p);  // (complete since the MMAs were issued: orders the scales)
      if (__any_sync(0xffffffffu, !ok)) {  // (tcgen05.ld is warp-wide)
        fail = true;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int kb = cur.kb;
      const uint32_t ta = tbase + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)((p & 1) * T::kRegion + eb0);
      if constexpr (WT == 14) {
        const uint32_t* sd = scs + ((size_t)(p % kSlots) * kMmaRows + em) * 4;
        uint32_t scw[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) scw[k] = sd[k];
        int sumi[EB];
#pragma unroll
        for (int e = 0; e < EB; ++e) sumi[e] = 0;
#pragma unroll
        for (int j0 = 0; j0 < 16; j0 += 4) {
          uint32_t d[4][EB];
#pragma unroll
          for (int u = 0; u < 4; ++u) tmem_ld<EB>(ta + 16 * (j0 + u), d[u]);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = j0 + u;
            const int sc = (int)(int8_t)(scw[j >> 2] >> (8 * (j & 3)));
#pragma unroll
            for (int e = 0; e < EB; ++e) sumi[e] += sc * (int)d[u][e];
          }
        }
        const float dw = dws[(p % kSlots) * kMmaRows + em];
#pragma unroll
        for (int e = 0; e < EB; ++e) {
          const int b = eb0 + e;
          if (b < a.nb)
            acc[e] = __fadd_rn(acc[e], __fmul_rn(__fmul_rn(dsa[b * nab + kb], dw), __int2float_rn(sumi[e])));
        }
      } else {
        // dotQ8_0i / dotQ4_0i (quant.nim:762-786): block after block,
        // acc += (d_w * d_a) * float(s); blocks 0-3, then 4-7
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t d[4][EB];
#pragma unroll
          for (int i = 0; i < 4; ++i) tmem_ld<EB>(ta + 16 * (4 * h + i), d[i]);
          float dw[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) dw[i] = dws[((p % kSlots) * 8 + 4 * h + i) * kMmaRows + em];
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int e = 0; e < EB; ++e) {
            const int b = eb0 + e;
            if (b >= a.nb) break;
            const float4 da = *reinterpret_cast<const float4*>(dsa + b * nab + kb * 8 + 4 * h);
            acc[e] = __fadd_rn(acc[e], __fmul_rn(__fmul_rn(dw[0], da.x), __int2float_rn((int)d[0][e])));
            acc[e] = __fadd_rn(acc[e], __fmul_rn(__fmul_rn(dw[1], da.y), __int2float_rn((int)d[1][e])));
            acc[e] = __fadd_rn(acc[e], __fmul_rn(__fmul_rn(dw[2], da.z), __int2float_rn((int)d[2][e])));
            acc[e] = __fadd_rn(acc[e], __fmul_rn(__fmul_rn(dw[3], da.w), __int2float_rn((int)d[3][e])));
          }
        }
      }
      // TMEM region p & 1 read: the MMAs of step p + 2 may overwrite it
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[p & 1]);
      if (kb == a.nblk - 1) {
        const int r = cur.t * kMmaRows + em;
#pragma unroll
        for (int e = 0; e < EB; ++e) {
          const int b = eb0 + e;
          if (b < a.nb && r < a.rows) a.y[(size_t)b * a.ldy + r] = acc[e];
          acc[e] = 0.0f;
        }
      }
    }
  }
  if (fail) *s_fail = 1;
  __syncthreads();
  if (*s_fail) {  // (uniform after the barrier)
    if (tid == 0) {
      atomicCAS(a.status, 0, NLS_ERR_TIMEOUT);
      // let the copies and MMAs in flight finish before the shared memory and
      // the columns are released, under the default limit whatever the
      // call's (they are real and land); only the last two of each can be
      // in flight (a step is staged, or its MMAs issued, once the one two
      // steps before it has been waited for)
      auto drain = [&](uint64_t* b2, int s) {
        (void)mbar_wait_bounded(&b2[s & 1], (uint32_t)((s >> 1) & 1), kWaitLimitNs);
      };
      const int st = *s_staged, last = *s_last;
      if (st >= 0) drain(full, st);
      if (st >= 1) drain(full, st - 1);
      if (last >= 0) drain(done, last);
      if (last >= 1) drain(done, last - 1);
    }
    __syncthreads();
  }
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kTmemCols) : "memory");
}

}  // namespace

size_t lm_head_mma_smem(int wtype, int cols) {
  return wtype == 14 ? mma_smem<14>(cols) : wtype == 8 ? mma_smem<8>(cols) : wtype == 2 ? mma_smem<2>(cols) : 0;
}

int lm_head_mma_min_rows(int wtype) { return wtype == 14 ? 8 : 8; }

bool lm_head_mma_path(int wtype, int cols, int nb) {
  return (wtype == 14 || wtype == 8 || wtype == 2) && nb >= lm_head_mma_min_rows(wtype) && cols % 256 == 0 &&
         cols >= 256 && lm_head_mma_smem(wtype, cols) <= (size_t)(227 * 1024);
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// the driver's tensor-map encoder (through the runtime, so the library needs
// no link to the driver library); null if the driver has none
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (EncodeTiledFn) nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

}  // namespace

size_t lm_head_act_scratch_bytes(int cols) {
  // the operand of 16 batch rows, then the scales (blocks of 32 at most)
  return (size_t)kMmaN * cols + (size_t)kMmaN * (cols / 32) * 4;
}

cudaError_t launch_lm_head_mma(const uint8_t* w, int wtype, int64_t row_bytes, int rows, int cols, const float* x,
                               int nb, float* y, int64_t ldy, int* status, int sm_count,
                               unsigned long long wait_ns, uint8_t* act_scratch, cudaStream_t st) {
  if ((reinterpret_cast<uintptr_t>(act_scratch) & 15) != 0) return cudaErrorInvalidValue;
  if (wtype != 14 && wtype != 8 && wtype != 2) return cudaErrorInvalidValue;
  const int raw_row = (wtype == 14) ? MmaType<14>::kRawRow : (wtype == 8) ? MmaType<8>::kRawRow : MmaType<2>::kRawRow;
  // the weights as a 2-D tensor of 8-byte elements: row_bytes / 8 per row,
  // rows rows, row_bytes apart; a box of 128 rows x one staged step
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  int tiled = 0;
  if (row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0) {
    if (EncodeTiledFn enc = encode_tiled()) {
      const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)rows};
      const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
      const cuuint32_t box[2] = {(cuuint32_t)(raw_row / 8), (cuuint32_t)kMmaRows};
      const cuuint32_t estr[2] = {1, 1};
      tiled = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t*>(w), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
  }
  MmaArgs a{};
  a.w = w;
  a.row_bytes = row_bytes;
  a.total = (int64_t)rows * row_bytes;
  a.rows = rows;
  a.cols = cols;
  a.nblk = cols / 256;
  a.ldy = ldy;
  a.ntiles = (rows + kMmaRows - 1) / kMmaRows;
  a.wait_ns = wait_ns;
  a.status = status;
  a.tiled = tiled;
  const size_t smem = lm_head_mma_smem(wtype, cols);
  auto kern = (wtype == 14) ? lmh_mma_kernel<14> : (wtype == 8) ? lmh_mma_kernel<8> : lmh_mma_kernel<2>;
  auto roles = [](auto t) { return 32 * (1 + decltype(t)::kUnpackWarps + decltype(t)::kSumWarps); };
  const int threads = (wtype == 14) ? roles(MmaType<14>{}) : (wtype == 8) ? roles(MmaType<8>{}) : roles(MmaType<2>{});
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int grid = std::min(a.ntiles, sm_count);
  auto quant = (wtype == 14) ? lmh_mma_quant_kernel<14> : (wtype == 8) ? lmh_mma_quant_kernel<8>
                                                                        : lmh_mma_quant_kernel<2>;
  uint8_t* qs = act_scratch;
  float* ds = reinterpret_cast<float*>(act_scratch + (size_t)kMmaN * cols);
  a.q = qs;
  a.dq = ds;
  const int qgrid = (kMmaN * (cols / 32) + 255) / 256;
  for (int b0 = 0; b0 < nb; b0 += kMmaN) {
    a.nb = std::min(kMmaN, nb - b0);
    a.y = y + (size_t)b0 * ldy;
    // (the next chunk's quantization starts after this chunk's projection
    // has finished reading the scratch: plain stream order)
    quant<<<qgrid, 256, 0, st>>>(x + (size_t)b0 * cols, a.nb, cols, qs, ds, status);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid, 1, 1);
    cfg.blockDim = dim3((unsigned)threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a, map);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace nls
