/*
 * oracle/ref_lmhead.c -- CPU restatement of nimllm's output projection, the
 * matmul that produces the sampler's logits (model.nim:466-470).
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU legs may load this library; the product path (nim.llm_b200/)
 * never links or calls it.
 *
 * Parity status: UNPINNED against the reference itself (no Nim toolchain
 * here, and the reference's tests hold no golden vectors for matmul).
 * Cross-checked against oracle/translit.py (a separate line-by-line Python
 * transliteration with numpy float32 scalars).
 *
 * Follows, with the reference's operation order and rounding points:
 *   matmul        model.nim:179-189  path choice: int8 activations when
 *                                    !exactMatmul, the type has an activation
 *                                    block (actBlockLen, quant.nim:639-644),
 *                                    cols is a whole number of blocks and
 *                                    (nb <= 4 or the type is not Q8_0);
 *   matmulTask    model.nim:144-169  y[b*rows + r], one dot product per (b, r);
 *   quantizeAct   quant.nim:646-662
 *   dotQ8_0i / dotQ4_0i / dotQ6K     quant.nim:762-786, :731-760
 *   dequantRow / dequantBlock        quant.nim:336-352, :160-202, :303-321
 *   dotF32        quant.nim:362-374  eight strided fp32 accumulators
 *   halfToFloat   quant.nim:83-110   (exact half -> float)
 * Two literal-typing and contraction assumptions, both as a plain x86-64 build
 * of the reference (-d:release, no -march=native) compiles them: `v + 0.5` in
 * quantizeAct is a float32 addition (Nim types the literal as the float32
 * operand), and no multiply-add is fused (-ffp-contract=off here).
 * Weight types restated: F32, F16, Q4_0, Q8_0, Q6_K.
 */
#include "ref_lmhead.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* halfToFloatSlow (quant.nim:83-96); the reference reads it from a table. */
static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t ex = (h >> 10) & 0x1Fu;
  const uint32_t mant = h & 0x3FFu;
  uint32_t bits;
  if (ex == 0) {
    const float v = (float)((double)mant * ldexp(1.0, -24));
    return sign ? -v : v;
  } else if (ex == 31) {
    bits = sign | 0x7F800000u | (mant << 13);
  } else {
    bits = sign | ((ex + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* rdHalf (quant.nim:144-147): little-endian 16 bits at byte o. */
static float rd_half(const uint8_t* p, int64_t o) {
  return half_to_float((uint16_t)(p[o] | (p[o + 1] << 8)));
}

static int64_t block_size(int32_t t) {
  switch (t) {
    case NLO_F32: case NLO_F16: return 1;
    case NLO_Q4_0: case NLO_Q8_0: return 32;
    case NLO_Q6_K: return 256;
    default: return 0;
  }
}

static int64_t type_size(int32_t t) {
  switch (t) {
    case NLO_F32: return 4;
    case NLO_F16: return 2;
    case NLO_Q4_0: return 18;
    case NLO_Q8_0: return 34;
    case NLO_Q6_K: return 210;
    default: return 0;
  }
}

int64_t nlo_row_bytes(int32_t t, int64_t cols) {
  const int64_t bs = block_size(t);
  if (bs == 0 || cols < 0 || cols % bs != 0) return -1;
  return cols / bs * type_size(t);
}

/* actBlockLen (quant.nim:639-644) over the restated types. */
static int64_t act_block_len(int32_t t) {
  switch (t) {
    case NLO_Q6_K: return 256;
    case NLO_Q8_0: case NLO_Q4_0: return 32;
    default: return 0;
  }
}

void nlo_quantize_act(const float* x, int64_t n, int64_t bl, float* d_out, int8_t* qs) {
  const int64_t nb = n / bl;
  for (int64_t b = 0; b < nb; ++b) {
    float amax = 0.0f;
    for (int64_t i = 0; i < bl; ++i) {
      const float a = fabsf(x[b * bl + i]);
      amax = (amax <= a) ? a : amax; /* max(amax, abs(x)) */
    }
    const float d = amax / 127.0f;
    const float id = d > 0.0f ? 1.0f / d : 0.0f;
    d_out[b] = d;
    for (int64_t i = 0; i < bl; ++i) {
      const float v = x[b * bl + i] * id;
      const int q = v >= 0.0f ? (int)(v + 0.5f) : -(int)(-v + 0.5f);
      qs[b * bl + i] = (int8_t)q;
    }
  }
}

/* dotF32 (quant.nim:362-374). */
static float dot_f32(const float* a, const float* b, int64_t n) {
  float s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0, s5 = 0, s6 = 0, s7 = 0;
  int64_t i = 0;
  while (i + 8 <= n) {
    s0 += a[i] * b[i];
    s1 += a[i + 1] * b[i + 1];
    s2 += a[i + 2] * b[i + 2];
    s3 += a[i + 3] * b[i + 3];
    s4 += a[i + 4] * b[i + 4];
    s5 += a[i + 5] * b[i + 5];
    s6 += a[i + 6] * b[i + 6];
    s7 += a[i + 7] * b[i + 7];
    i += 8;
  }
  while (i < n) {
    s0 += a[i] * b[i];
    ++i;
  }
  float t = s0 + s1;
  t = t + (s2 + s3);
  t = t + (s4 + s5);
  t = t + (s6 + s7);
  return t;
}

/* dequantRow (quant.nim:336-352) for one row of n values. */
static void dequant_row(int32_t t, const uint8_t* s, float* y, int64_t n) {
  switch (t) {
    case NLO_F32:
      memcpy(y, s, (size_t)n * 4);
      return;
    case NLO_F16:
      for (int64_t i = 0; i < n; ++i) y[i] = rd_half(s, 2 * i);
      return;
    case NLO_Q8_0:
      for (int64_t ib = 0; ib < n / 32; ++ib) {
        const uint8_t* b = s + ib * 34;
        const float d = rd_half(b, 0);
        for (int j = 0; j < 32; ++j) y[ib * 32 + j] = (float)(int8_t)b[2 + j] * d;
      }
      return;
    case NLO_Q4_0:
      for (int64_t ib = 0; ib < n / 32; ++ib) {
        const uint8_t* b = s + ib * 18;
        const float d = rd_half(b, 0);
        for (int j = 0; j < 16; ++j) {
          const uint8_t q = b[2 + j];
          y[ib * 32 + j] = (float)((int)(q & 0xF) - 8) * d;
          y[ib * 32 + j + 16] = (float)((int)(q >> 4) - 8) * d;
        }
      }
      return;
    case NLO_Q6_K:
      for (int64_t ib = 0; ib < n / 256; ++ib) {
        const uint8_t* b = s + ib * 210;
        float* yb = y + ib * 256;
        const float d = rd_half(b, 208);
        int qlo = 0, qho = 128, sco = 192, yo = 0;
        for (int h = 0; h < 2; ++h) {
          for (int l = 0; l < 32; ++l) {
            const int isc = l / 16;
            const uint8_t qh = b[qho + l];
            const int q1 = (int)((b[qlo + l] & 0xF) | (((qh >> 0) & 3) << 4)) - 32;
            const int q2 = (int)((b[qlo + l + 32] & 0xF) | (((qh >> 2) & 3) << 4)) - 32;
            const int q3 = (int)((b[qlo + l] >> 4) | (((qh >> 4) & 3) << 4)) - 32;
            const int q4 = (int)((b[qlo + l + 32] >> 4) | (((qh >> 6) & 3) << 4)) - 32;
            yb[yo + l] = d * (float)(int8_t)b[sco + isc] * (float)q1;
            yb[yo + l + 32] = d * (float)(int8_t)b[sco + isc + 2] * (float)q2;
            yb[yo + l + 64] = d * (float)(int8_t)b[sco + isc + 4] * (float)q3;
            yb[yo + l + 96] = d * (float)(int8_t)b[sco + isc + 6] * (float)q4;
          }
          yo += 128;
          qlo += 64;
          qho += 32;
          sco += 8;
        }
      }
      return;
    default:
      return;
  }
}

/* dotQ8_0i (quant.nim:762-772); off is the activation offset b*cols. */
static float dot_q8_0i(const uint8_t* w, const float* ad, const int8_t* aq, int64_t off, int64_t n) {
  float acc = 0.0f;
  for (int64_t ib = 0; ib < n / 32; ++ib) {
    const int64_t o = ib * 34, ab = off / 32 + ib;
    const int8_t* q8 = aq + ab * 32;
    int32_t s = 0;
    for (int l = 0; l < 32; ++l) s += (int32_t)(int8_t)w[o + 2 + l] * (int32_t)q8[l];
    acc += rd_half(w, o) * ad[ab] * (float)s;
  }
  return acc;
}

/* dotQ4_0i (quant.nim:774-786). */
static float dot_q4_0i(const uint8_t* w, const float* ad, const int8_t* aq, int64_t off, int64_t n) {
  float acc = 0.0f;
  for (int64_t ib = 0; ib < n / 32; ++ib) {
    const int64_t o = ib * 18, ab = off / 32 + ib;
    const int8_t* q8 = aq + ab * 32;
    int32_t s = 0;
    for (int l = 0; l < 16; ++l) {
      const uint8_t q = w[o + 2 + l];
      s += ((int32_t)(q & 0xF) - 8) * (int32_t)q8[l] + ((int32_t)(q >> 4) - 8) * (int32_t)q8[l + 16];
    }
    acc += rd_half(w, o) * ad[ab] * (float)s;
  }
  return acc;
}

/* dotQ6K (quant.nim:731-760). */
static float dot_q6k(const uint8_t* w, const float* ad, const int8_t* aq, int64_t off, int64_t n) {
  float acc = 0.0f;
  for (int64_t ib = 0; ib < n / 256; ++ib) {
    const uint8_t* b = w + ib * 210;
    const int64_t ab = off / 256 + ib;
    const int8_t* q8 = aq + ab * 256;
    const float d = rd_half(b, 208);
    const int8_t* sc = (const int8_t*)(b + 192);
    int32_t sumi = 0;
    for (int h = 0; h < 2; ++h) {
      const int ql = 64 * h, qh = 128 + 32 * h;
      for (int half = 0; half < 2; ++half) {
        int32_t s0 = 0, s1 = 0, s2 = 0, s3 = 0;
        for (int l = 16 * half; l < 16 * half + 16; ++l) {
          const uint8_t hb = b[qh + l];
          const int32_t q1 = (int32_t)((b[ql + l] & 0xF) | ((hb & 3) << 4)) - 32;
          const int32_t q2 = (int32_t)((b[ql + l + 32] & 0xF) | (((hb >> 2) & 3) << 4)) - 32;
          const int32_t q3 = (int32_t)((b[ql + l] >> 4) | (((hb >> 4) & 3) << 4)) - 32;
          const int32_t q4 = (int32_t)((b[ql + l + 32] >> 4) | (((hb >> 6) & 3) << 4)) - 32;
          const int base = 128 * h + l;
          s0 += q1 * (int32_t)q8[base];
          s1 += q2 * (int32_t)q8[base + 32];
          s2 += q3 * (int32_t)q8[base + 64];
          s3 += q4 * (int32_t)q8[base + 96];
        }
        const int so = 8 * h + half;
        sumi += (int32_t)sc[so] * s0 + (int32_t)sc[so + 2] * s1 + (int32_t)sc[so + 4] * s2 +
                (int32_t)sc[so + 6] * s3;
      }
    }
    acc += ad[ab] * d * (float)sumi;
  }
  return acc;
}

typedef struct {
  const uint8_t* w;
  int32_t t;
  int64_t rows, cols, rb, nb;
  const float* x;
  float* y;
  const float* ad; /* NULL: float path */
  const int8_t* aq;
  int64_t r0, r1;
} task_t;

static void* run_rows(void* p) {
  const task_t* c = (const task_t*)p;
  float* tmp = c->ad ? NULL : (float*)malloc((size_t)c->cols * sizeof(float));
  for (int64_t r = c->r0; r < c->r1; ++r) {
    const uint8_t* rp = c->w + r * c->rb;
    if (c->ad) {
      for (int64_t b = 0; b < c->nb; ++b) {
        float v = 0.0f;
        if (c->t == NLO_Q8_0) v = dot_q8_0i(rp, c->ad, c->aq, b * c->cols, c->cols);
        else if (c->t == NLO_Q4_0) v = dot_q4_0i(rp, c->ad, c->aq, b * c->cols, c->cols);
        else v = dot_q6k(rp, c->ad, c->aq, b * c->cols, c->cols);
        c->y[b * c->rows + r] = v;
      }
    } else {
      dequant_row(c->t, rp, tmp, c->cols);
      for (int64_t b = 0; b < c->nb; ++b) c->y[b * c->rows + r] = dot_f32(tmp, c->x + b * c->cols, c->cols);
    }
  }
  free(tmp);
  return NULL;
}

int nlo_lm_head(const uint8_t* w, int32_t t, int64_t rows, int64_t cols, const float* x, int64_t nb,
                float* y, int32_t exact_matmul, int32_t threads) {
  const int64_t rb = nlo_row_bytes(t, cols);
  if (rb < 0 || rows < 0 || nb < 0) return -1;
  if (rows == 0 || nb == 0) return 0;
  const int64_t bl = act_block_len(t);
  float* ad = NULL;
  int8_t* aq = NULL;
  if (!exact_matmul && bl > 0 && cols % bl == 0 && (nb <= 4 || t != NLO_Q8_0)) {
    ad = (float*)malloc((size_t)(nb * cols / bl) * sizeof(float));
    aq = (int8_t*)malloc((size_t)(nb * cols));
    nlo_quantize_act(x, nb * cols, bl, ad, aq);
  }
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (threads > rows) threads = (int32_t)rows;
  pthread_t th[256];
  task_t tk[256];
  for (int i = 0; i < threads; ++i) {
    tk[i] = (task_t){w, t, rows, cols, rb, nb, x, y, ad, aq, rows * i / threads, rows * (i + 1) / threads};
    if (threads > 1) pthread_create(&th[i], NULL, run_rows, &tk[i]);
  }
  if (threads == 1) run_rows(&tk[0]);
  else
    for (int i = 0; i < threads; ++i) pthread_join(th[i], NULL);
  free(ad);
  free(aq);
  return 0;
}
