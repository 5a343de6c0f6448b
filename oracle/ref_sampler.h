/*
 * oracle/ref_sampler.h -- CPU restatement of nimllm's sampler (TEST INFRASTRUCTURE).
 *
 * This is the checker, never the product: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline / --impl reference leg may load it.
 *
 * Parity status: UNPINNED against the reference itself. The reference is Nim
 * (src/nimllm/sampler.nim) and no Nim toolchain exists on these machines; its
 * own tests hold no golden vectors for the stochastic branches. The restatement
 * is cross-checked against an independent line-by-line Python transliteration
 * (oracle/translit.py) and against hand-derived known-answer tests.
 */
#ifndef NLS_ORACLE_REF_SAMPLER_H
#define NLS_ORACLE_REF_SAMPLER_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors SamplerParams (sampler.nim:11-21) minus seed/logitBias, which are
 * passed separately (the RNG stays with the caller; bias is a CSR list). */
typedef struct {
  double temperature;       /* sampler.nim:12 */
  double top_p;             /* sampler.nim:14 */
  double min_p;             /* sampler.nim:15 */
  double repeat_penalty;    /* sampler.nim:16 */
  double presence_penalty;  /* sampler.nim:18 */
  double frequency_penalty; /* sampler.nim:19 */
  int64_t top_k;            /* sampler.nim:13 */
  int64_t repeat_last_n;    /* sampler.nim:17 */
} nlo_params;

/* Extra outputs of one draw, for parity diagnostics. */
typedef struct {
  float prob;       /* softmax probability of the drawn candidate (probs[i]) */
  int64_t ncand;    /* candidates before cut-offs (k, or V for the full sort) */
  int64_t n;        /* candidates kept after top-p and min-p */
  int64_t pos;      /* position of the drawn token in the candidate order */
  double margin;    /* smallest decision margin seen: draw, top-p, min-p */
  float total;      /* sequential sum of the kept probabilities */
  float denom;      /* softmax denominator (sequential fp32 sum) */
} nlo_diag;

int64_t nlo_argmax(const float* x, int64_t n);                 /* sampler.nim:45-49 */
void nlo_softmax_inplace(float* x, int64_t n);                 /* sampler.nim:51-57 */

/* One call of Sampler.sample (sampler.nim:59-121). `hist` is the full
 * history (the window of repeat_last_n is applied here, sampler.nim:67).
 * `uniform` is the value rng.rand(1.0) returned; it is ignored for greedy
 * rows (temperature <= 0), which consume no uniform. Returns the token id,
 * or -1 when n_vocab <= 0 (the reference raises IndexDefect there). */
int64_t nlo_sample(const nlo_params* p, const int64_t* hist, int64_t hist_len,
                   const int64_t* bias_ids, const double* bias_vals, int64_t n_bias,
                   const float* logits, int64_t n_vocab, double uniform,
                   nlo_diag* diag);

/* topTokens (sampler.nim:123-130): the n most probable tokens. Returns the
 * number written (min(n, n_vocab)). */
int64_t nlo_top_tokens(const float* logits, int64_t n_vocab, int64_t n,
                       int64_t* out_ids, float* out_probs);

/* Batch driver: row r uses params[r], hist[hist_off[r]..hist_off[r+1]),
 * bias[bias_off[r]..bias_off[r+1]), logits + r*ld, uniforms[r]. Rows are
 * independent and spread over `threads` POSIX threads (the reference sampler
 * itself is single-threaded per call). diag may be NULL. */
void nlo_sample_batch(const float* logits, int64_t ld, int64_t rows, int64_t n_vocab,
                      const nlo_params* params,
                      const int64_t* hist, const int64_t* hist_off,
                      const int64_t* bias_ids, const double* bias_vals, const int64_t* bias_off,
                      const double* uniforms, int64_t* out_ids, nlo_diag* diag,
                      int threads);

/* perplexity's per-position term (model.nim:580-584) for one row. */
double nlo_token_nll(const float* logits, int64_t V, int64_t target);

#ifdef __cplusplus
}
#endif
#endif
