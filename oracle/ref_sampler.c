/*
 * oracle/ref_sampler.c -- CPU restatement of nimllm's logits->token sampler.
 *
 * TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and
 * bench.py (cpu_baseline leg and --impl reference) may load this library;
 * the product path (nim.llm_b200/) never links or calls it.
 *
 * Parity status: UNPINNED against the reference itself (no Nim toolchain here
 * and no golden vectors for the stochastic branches in the reference's tests).
 * Cross-checked against oracle/translit.py, a separate line-by-line Python
 * transliteration, and against hand-derived known-answer tests.
 *
 * Every step follows src/nimllm/sampler.nim (reference repository) and keeps
 * Nim's numeric conversion points:
 *   - Nim `float` is IEEE double, `float32` is IEEE single; `x.float32` rounds
 *     to nearest; `exp(float32)` is C expf (glibc here, as on the reference's
 *     Linux builds).
 *   - Compiled with -ffp-contract=off so `cnt*freq + pres` is not fused,
 *     matching an x86-64 build without -march=native (tests/config.nims).
 *   - Sums are sequential fp32 in candidate order, exactly as the Nim loops.
 */
#include "ref_sampler.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* Nim system.cmp for floats: 0 when ==, -1 when <, else 1. */
static int nim_cmp_f32(float x, float y) {
  if (x == y) return 0;
  if (x < y) return -1;
  return 1;
}

/* argmax (sampler.nim:45-49): first index of the maximum, strict `>`. */
int64_t nlo_argmax(const float* x, int64_t n) {
  int64_t best = 0;
  for (int64_t i = 1; i < n; ++i)
    if (x[i] > x[best]) best = i;
  return best;
}

/* Nim max(x, y) on float32: returns y when x <= y. Only the sign of a zero
 * can differ between definitions, and v - mx is the same either way. */
static float nim_max_f32(float x, float y) { return (x <= y) ? y : x; }

/* softmaxInPlace (sampler.nim:51-57): max, expf(v - mx) with a sequential
 * fp32 sum in array order, then a true division by the sum. */
void nlo_softmax_inplace(float* x, int64_t n) {
  float mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i) mx = nim_max_f32(mx, x[i]);
  float s = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    x[i] = expf(x[i] - mx);
    s += x[i];
  }
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] / s;
}

/* ---- std/heapqueue on (float32, int) tuples (sampler.nim:88-95) ----------
 * A binary min-heap with the push / replace / pop steps of the published
 * heapq algorithm; Nim's tuple `<` is lexicographic, so the min is the
 * smallest value and, among equal values, the smallest index. */
typedef struct { float v; int64_t i; } hitem;

static int hless(hitem a, hitem b) {
  int c = nim_cmp_f32(a.v, b.v);
  if (c != 0) return c < 0;
  return a.i < b.i;
}

static void h_siftdown(hitem* h, int64_t startpos, int64_t pos) {
  hitem newitem = h[pos];
  while (pos > startpos) {
    int64_t parentpos = (pos - 1) >> 1;
    hitem parent = h[parentpos];
    if (hless(newitem, parent)) {
      h[pos] = parent;
      pos = parentpos;
    } else {
      break;
    }
  }
  h[pos] = newitem;
}

static void h_siftup(hitem* h, int64_t len, int64_t pos) {
  int64_t endpos = len, startpos = pos;
  hitem newitem = h[pos];
  int64_t childpos = 2 * pos + 1;
  while (childpos < endpos) {
    int64_t rightpos = childpos + 1;
    if (rightpos < endpos && !hless(h[childpos], h[rightpos])) childpos = rightpos;
    h[pos] = h[childpos];
    pos = childpos;
    childpos = 2 * pos + 1;
  }
  h[pos] = newitem;
  h_siftdown(h, startpos, pos);
}

static void h_push(hitem* h, int64_t* len, hitem it) {
  h[*len] = it;
  *len += 1;
  h_siftdown(h, 0, *len - 1);
}

static hitem h_pop(hitem* h, int64_t* len) {
  hitem last = h[*len - 1];
  *len -= 1;
  if (*len > 0) {
    hitem ret = h[0];
    h[0] = last;
    h_siftup(h, *len, 0);
    return ret;
  }
  return last;
}

static void h_replace(hitem* h, int64_t len, hitem it) {
  h[0] = it;
  h_siftup(h, len, 0);
}

/* ---- algorithm.sort: stable merge sort, comparator cmp(x[b], x[a]) -------
 * (sampler.nim:97). A stable sort's output is unique, so any stable merge
 * sort reproduces it: descending value, ties by ascending index. */
static int sort_cmp(const float* x, int64_t a, int64_t b) { return nim_cmp_f32(x[b], x[a]); }

static void merge_sort_idx(const float* x, int64_t* a, int64_t* tmp, int64_t n) {
  for (int64_t width = 1; width < n; width *= 2) {
    for (int64_t lo = 0; lo < n; lo += 2 * width) {
      int64_t mid = lo + width < n ? lo + width : n;
      int64_t hi = lo + 2 * width < n ? lo + 2 * width : n;
      int64_t i = lo, j = mid, k = lo;
      while (i < mid && j < hi) {
        if (sort_cmp(x, a[i], a[j]) <= 0) tmp[k++] = a[i++];
        else tmp[k++] = a[j++];
      }
      while (i < mid) tmp[k++] = a[i++];
      while (j < hi) tmp[k++] = a[j++];
    }
    memcpy(a, tmp, (size_t)n * sizeof(int64_t));
  }
}

static int cmp_i64(const void* pa, const void* pb) {
  int64_t a = *(const int64_t*)pa, b = *(const int64_t*)pb;
  return (a > b) - (a < b);
}

static double dmin(double a, double b) { return a < b ? a : b; }

/* sample (sampler.nim:59-121). */
int64_t nlo_sample(const nlo_params* p, const int64_t* hist, int64_t hist_len,
                   const int64_t* bias_ids, const double* bias_vals, int64_t n_bias,
                   const float* logits_in, int64_t V, double uniform, nlo_diag* diag) {
  if (V <= 0) return -1;
  nlo_diag dg;
  memset(&dg, 0, sizeof dg);
  dg.margin = 1e30;
  /* var logits = @logitsIn (:62) */
  float* x = (float*)malloc((size_t)V * sizeof(float));
  memcpy(x, logits_in, (size_t)V * sizeof(float));

  /* penalties (:64-74): CountTable over the last repeatLastN ids. Iteration
   * order over distinct ids does not matter: each touches only its own
   * logit. */
  if (hist_len > 0 && (p->repeat_penalty != 1.0 || p->presence_penalty != 0 ||
                       p->frequency_penalty != 0)) {
    int64_t start = 0;
    if (p->repeat_last_n > 0) {
      start = hist_len - p->repeat_last_n;
      if (start < 0) start = 0;
    }
    int64_t wl = hist_len - start;
    int64_t* w = (int64_t*)malloc((size_t)wl * sizeof(int64_t));
    memcpy(w, hist + start, (size_t)wl * sizeof(int64_t));
    qsort(w, (size_t)wl, sizeof(int64_t), cmp_i64);
    for (int64_t i = 0; i < wl;) {
      int64_t tok = w[i], cnt = 0;
      while (i < wl && w[i] == tok) { ++cnt; ++i; }
      if (tok < 0 || tok >= V) continue;
      if (p->repeat_penalty != 1.0) {
        if (x[tok] > 0) x[tok] = x[tok] / (float)p->repeat_penalty;
        else x[tok] = x[tok] * (float)p->repeat_penalty;
      }
      x[tok] = x[tok] - (float)((double)cnt * p->frequency_penalty + p->presence_penalty);
    }
    free(w);
  }
  /* logit bias (:75-76), after the penalties. */
  for (int64_t b = 0; b < n_bias; ++b) {
    int64_t tok = bias_ids[b];
    if (tok >= 0 && tok < V) x[tok] = x[tok] + (float)bias_vals[b];
  }
  /* greedy (:77-78): argmax before temperature; no uniform consumed. */
  if (p->temperature <= 0) {
    int64_t id = nlo_argmax(x, V);
    free(x);
    dg.ncand = V; dg.n = 1; dg.pos = 0; dg.prob = 1.0f;
    if (diag) *diag = dg;
    return id;
  }
  /* temperature (:80-81) */
  float invT = (float)(1.0 / p->temperature);
  for (int64_t i = 0; i < V; ++i) x[i] = x[i] * invT;

  /* candidates (:83-97) */
  int64_t k = (p->top_k > 0) ? (p->top_k < V ? p->top_k : V) : V;
  int64_t* idx;
  int64_t nidx;
  if (k < V) {
    hitem* h = (hitem*)malloc((size_t)k * sizeof(hitem));
    int64_t hl = 0;
    for (int64_t i = 0; i < V; ++i) {
      if (hl < k) {
        hitem it = {x[i], i};
        h_push(h, &hl, it);
      } else if (x[i] > h[0].v) {
        hitem it = {x[i], i};
        h_replace(h, hl, it);
      }
    }
    idx = (int64_t*)malloc((size_t)k * sizeof(int64_t));
    nidx = 0;
    while (hl > 0) idx[nidx++] = h_pop(h, &hl).i;
    for (int64_t a = 0, b = nidx - 1; a < b; ++a, --b) {  /* idx.reverse() */
      int64_t t = idx[a]; idx[a] = idx[b]; idx[b] = t;
    }
    free(h);
  } else {
    idx = (int64_t*)malloc((size_t)V * sizeof(int64_t));
    int64_t* tmp = (int64_t*)malloc((size_t)V * sizeof(int64_t));
    for (int64_t i = 0; i < V; ++i) idx[i] = i;
    merge_sort_idx(x, idx, tmp, V);
    free(tmp);
    nidx = V;
  }
  dg.ncand = nidx;
  /* softmax over the candidates (:98-100) */
  float* probs = (float*)malloc((size_t)nidx * sizeof(float));
  for (int64_t i = 0; i < nidx; ++i) probs[i] = x[idx[i]];
  {
    float mx = -INFINITY;
    for (int64_t i = 0; i < nidx; ++i) mx = nim_max_f32(mx, probs[i]);
    float s = 0.0f;
    for (int64_t i = 0; i < nidx; ++i) {
      probs[i] = expf(probs[i] - mx);
      s += probs[i];
    }
    for (int64_t i = 0; i < nidx; ++i) probs[i] = probs[i] / s;
    dg.denom = s;
  }
  int64_t n = nidx;
  /* top-p (:102-108): fp32 running sum, float64 comparison. */
  if (p->top_p > 0 && p->top_p < 1) {
    float cum = 0.0f, prev = 0.0f;
    int hit = 0;
    for (int64_t i = 0; i < n; ++i) {
      prev = cum;
      cum += probs[i];
      if ((double)cum >= p->top_p) {
        n = i + 1;
        hit = 1;
        dg.margin = dmin(dg.margin, dmin((double)cum - p->top_p, p->top_p - (double)prev));
        break;
      }
    }
    if (!hit) dg.margin = dmin(dg.margin, p->top_p - (double)cum);
  }
  /* min-p (:109-114), after top-p and bounded by n. */
  if (p->min_p > 0) {
    float thr = probs[0] * (float)p->min_p;
    int64_t m = 1;
    while (m < n && probs[m] >= thr) ++m;
    if (m < n) dg.margin = dmin(dg.margin, (double)thr - (double)probs[m]);
    if (m > 1) dg.margin = dmin(dg.margin, (double)probs[m - 1] - (double)thr);
    n = m;
  }
  /* draw (:115-121) */
  float total = 0.0f;
  for (int64_t i = 0; i < n; ++i) total += probs[i];
  float r = (float)uniform * total;
  int64_t pos = n - 1;
  float rprev = r;
  for (int64_t i = 0; i < n; ++i) {
    rprev = r;
    r -= probs[i];
    if (r <= 0) { pos = i; break; }
  }
  int64_t id = idx[pos];
  dg.n = n;
  dg.pos = pos;
  dg.prob = probs[pos];
  dg.total = total;
  if (total > 0) {
    double m = (r <= 0) ? dmin((double)rprev, -(double)r) : (double)r;
    dg.margin = dmin(dg.margin, m / (double)total);
  }
  free(probs);
  free(idx);
  free(x);
  if (diag) *diag = dg;
  return id;
}

/* topTokens (sampler.nim:123-130): softmax over all V in index order, then a
 * stable descending sort. */
int64_t nlo_top_tokens(const float* logits, int64_t V, int64_t n, int64_t* out_ids,
                       float* out_probs) {
  if (V <= 0 || n <= 0) return 0;
  float* probs = (float*)malloc((size_t)V * sizeof(float));
  memcpy(probs, logits, (size_t)V * sizeof(float));
  nlo_softmax_inplace(probs, V);
  int64_t* idx = (int64_t*)malloc((size_t)V * sizeof(int64_t));
  int64_t* tmp = (int64_t*)malloc((size_t)V * sizeof(int64_t));
  for (int64_t i = 0; i < V; ++i) idx[i] = i;
  merge_sort_idx(probs, idx, tmp, V);
  int64_t m = n < V ? n : V;
  for (int64_t i = 0; i < m; ++i) {
    out_ids[i] = idx[i];
    out_probs[i] = probs[idx[i]];
  }
  free(tmp);
  free(idx);
  free(probs);
  return m;
}

/* perplexity's per-position term (model.nim:580-584): mx = the fp32 maximum
 * of the row (:581), s = the float64 sum, in index order, of
 * exp(float64(x_k - mx)) with the difference in fp32 (:582-583), and the
 * term -(float64(x_target - mx) - ln(s)) (:584). Nim's exp/ln on float64 are
 * C's exp/log. */
double nlo_token_nll(const float* logits, int64_t V, int64_t target) {
  float mx = -INFINITY;
  for (int64_t k = 0; k < V; ++k) mx = logits[k] > mx ? logits[k] : mx;
  double s = 0.0;
  for (int64_t k = 0; k < V; ++k) {
    const float d = logits[k] - mx;
    s += exp((double)d);
  }
  const float dt = logits[target] - mx;
  return -((double)dt - log(s));
}

typedef struct {
  const float* logits; int64_t ld, rows, V;
  const nlo_params* params;
  const int64_t *hist, *hist_off, *bias_ids, *bias_off;
  const double *bias_vals, *uniforms;
  int64_t* out_ids; nlo_diag* diag;
  int tid, nthreads;
} batch_job;

static void* batch_worker(void* arg) {
  batch_job* j = (batch_job*)arg;
  for (int64_t r = j->tid; r < j->rows; r += j->nthreads) {
    const int64_t* h = j->hist ? j->hist + j->hist_off[r] : NULL;
    int64_t hl = j->hist ? j->hist_off[r + 1] - j->hist_off[r] : 0;
    const int64_t* bi = j->bias_ids ? j->bias_ids + j->bias_off[r] : NULL;
    const double* bv = j->bias_vals ? j->bias_vals + j->bias_off[r] : NULL;
    int64_t nb = j->bias_ids ? j->bias_off[r + 1] - j->bias_off[r] : 0;
    j->out_ids[r] = nlo_sample(&j->params[r], h, hl, bi, bv, nb, j->logits + r * j->ld, j->V,
                               j->uniforms ? j->uniforms[r] : 0.0,
                               j->diag ? &j->diag[r] : NULL);
  }
  return NULL;
}

void nlo_sample_batch(const float* logits, int64_t ld, int64_t rows, int64_t V,
                      const nlo_params* params, const int64_t* hist, const int64_t* hist_off,
                      const int64_t* bias_ids, const double* bias_vals, const int64_t* bias_off,
                      const double* uniforms, int64_t* out_ids, nlo_diag* diag, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  batch_job jobs[256];
  pthread_t th[256];
  for (int t = 0; t < threads; ++t) {
    batch_job j = {logits, ld, rows, V, params, hist, hist_off, bias_ids, bias_off,
                   bias_vals, uniforms, out_ids, diag, t, threads};
    jobs[t] = j;
  }
  if (threads == 1) {
    batch_worker(&jobs[0]);
    return;
  }
  for (int t = 0; t < threads; ++t) pthread_create(&th[t], NULL, batch_worker, &jobs[t]);
  for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
}
