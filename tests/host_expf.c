/*
 * tests/host_expf.c -- host-side checker for the sampler's exponential.
 *
 * TEST INFRASTRUCTURE ONLY (compiled by tests/test_expf.py into a temporary
 * directory). The reference's softmax calls Nim's exp(float32), which is the
 * C library's expf (sampler.nim:56): on the reference's x86-64 Linux builds,
 * glibc's. This file counts, over ranges of float bit patterns and on all
 * host threads, where glibc's expf differs from
 *   - (float)exp((double)x), the correctly rounded value in practice;
 *   - method_expf(x) below, a C restatement of the method glibc ships
 *     (Arm optimized-routines' expf), the same operations as the device
 *     function ref_expf in nim.llm_b200/csrc/nls_common.cuh;
 *   - an array of device results copied to the host.
 * Built with -ffp-contract=off so that only the explicit fma() calls fuse.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

static float f_of(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t b_of(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

static const uint64_t kTab[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};

/* 2^(j/32) rounded to double, with j/32 taken out of the exponent field */
uint64_t nhx_table(int j) { return kTab[j & 31]; }

float method_expf(float x) {
  const double inv_ln2_n = 0x1.71547652b82fep0 * 32.0, shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
  const double c1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
  const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  if (x != x) return x + x;
  if (x < -0x1.9fe368p6f) return 0.0f;
  if (x > 0x1.62e42ep6f) return INFINITY;
  const double xd = x;
  double kd = fma(inv_ln2_n, xd, shift);
  uint64_t ki;
  memcpy(&ki, &kd, 8);
  kd -= shift;
  const double r = fma(inv_ln2_n, xd, -kd);
  const uint64_t t = kTab[ki & 31] + (ki << 47);
  double s;
  memcpy(&s, &t, 8);
  const double z = fma(c0, r, c1);
  double y = fma(c2, r, 1.0);
  y = fma(z, r * r, y);
  return (float)(y * s);
}

typedef struct {
  int what; /* 0: vs double exp, 1: vs method, 2: vs device array */
  uint32_t first;
  int64_t lo, hi;
  const float* dev;
  int64_t count;
  int64_t first_bad;
} job_t;

static int same(float a, float b) {
  if (a != a && b != b) return 1;
  return b_of(a) == b_of(b);
}

static void* worker(void* p) {
  job_t* j = (job_t*)p;
  j->count = 0;
  j->first_bad = -1;
  for (int64_t i = j->lo; i < j->hi; ++i) {
    const float x = f_of(j->first + (uint32_t)i);
    const float g = expf(x);
    float o;
    if (j->what == 0) o = (float)exp((double)x);
    else if (j->what == 1) o = method_expf(x);
    else o = j->dev[i];
    if (!same(g, o)) {
      if (j->first_bad < 0) j->first_bad = i;
      j->count++;
    }
  }
  return NULL;
}

/* Number of i in [0, n) where glibc expf(x_i) differs from the chosen
 * comparison (x_i = float with bits first + i); *first_bad = the smallest
 * such i, or -1. */
int64_t nhx_count(int what, uint32_t first, int64_t n, const float* dev, int threads,
                  int64_t* first_bad) {
  if (threads < 1) threads = 1;
  if (threads > 64) threads = 64;
  job_t jobs[64];
  pthread_t th[64];
  for (int t = 0; t < threads; ++t) {
    jobs[t].what = what;
    jobs[t].first = first;
    jobs[t].lo = n * t / threads;
    jobs[t].hi = n * (t + 1) / threads;
    jobs[t].dev = dev;
    pthread_create(&th[t], NULL, worker, &jobs[t]);
  }
  int64_t total = 0, fb = -1;
  for (int t = 0; t < threads; ++t) {
    pthread_join(th[t], NULL);
    total += jobs[t].count;
    if (jobs[t].first_bad >= 0 && (fb < 0 || jobs[t].first_bad < fb)) fb = jobs[t].first_bad;
  }
  if (first_bad) *first_bad = fb;
  return total;
}
