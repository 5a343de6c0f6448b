/*
 * tests/nim_abi_harness.c -- the library bound the way Nim binds it.
 *
 * TEST INFRASTRUCTURE (compiled and run by tests/test_nim_binding.py).
 * A Nim module that declares
 *     proc nls_sample_batch(...): NlsStatus {.importc, dynlib: nlsLib, cdecl.}
 * does not link against the library: at start-up it dlopen()s
 * "libnimllm_sample.so" and dlsym()s every importc name, calling each through
 * a function pointer whose C type Nim's code generator derives from the Nim
 * declaration (int32 -> NI32 = int32_t, int64 -> NI64 = int64_t, uint32 ->
 * NU32 = uint32_t, float32 -> NF32 = float, float64 -> NF = double, ptr T ->
 * T*, pointer -> void*, cstring -> char*, an {.bycopy.} object -> a struct
 * with the same fields). This program does exactly that for the names the
 * binding module of INTEGRATION.md imports, with those types, and then runs
 * the generation loop of chat.nim:204-208 -- `let id = s.sample(logits)`,
 * `s.accept id`, next logits -- through the binding's `sample` (the unchanged
 * reference signature, sampler.nim:59), re-expressed in C:
 *   - one module-level handle, created on the first call;
 *   - u = s.rng.rand(1.0) drawn only when temperature > 0 (sampler.nim:77-78,117);
 *   - the whole history passed as CSR (the library applies repeatLastN, :67);
 *   - the logitBias table passed as CSR lists (ids int64, values float64);
 *   - an empty logitsIn handled as the reference does: greedy returns 0, a
 *     sampling call raises (the reference indexes probs[0] or idx[n - 1]).
 *
 * Usage:  nim_abi_harness <lib.so> --resolve-only
 *         nim_abi_harness <lib.so> <input.bin> <output.bin>
 * Input (little endian): int64 V, steps_a, steps_b, n_hist0, n_bias, n_unif;
 * params A and B (64-byte records); the initial history (int64 x n_hist0);
 * bias ids (int64) and values (float64) of sampler A; the uniform stream
 * (float64 x n_unif); logits of A's steps then of B's (float32 x V each).
 * Output: ids of A's steps, ids of B's steps (int64), uniforms consumed
 * (int64), then the results of the empty-logits probes (int64 x 2).
 */
#include <dlfcn.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef int32_t NI32;
typedef int64_t NI64;
typedef uint32_t NU32;
typedef float NF32;
typedef double NF;

/* NlsRowParams* {.bycopy.} = object  (nls_row_params, 64 bytes) */
typedef struct {
  NF temperature, topP, minP;
  NF repeatPenalty, presencePenalty, frequencyPenalty;
  NI64 topK, repeatLastN;
} NlsRowParams;

/* the importc declarations of the binding module, as Nim types them */
typedef NI32 (*nls_create_t)(void** outH, NI32 device, NI32 maxRows, NI32 maxVocab);
typedef void (*nls_destroy_t)(void* h);
typedef NI32 (*nls_sample_batch_t)(void* h, NF32* logits, NI64 ld, NI32 rows, NI32 vocab,
                                   NlsRowParams* params, NI64* histIds, NI64* histOff,
                                   NI64* biasIds, NF* biasVals, NI64* biasOff, NF* uniforms,
                                   NI64* outIds, NF32* outProbs, NU32 flags, void* stream);
typedef NI32 (*nls_argmax_batch_t)(void* h, NF32* logits, NI64 ld, NI32 rows, NI32 vocab,
                                   NI64* outIds, NU32 flags, void* stream);
typedef NI32 (*nls_top_tokens_t)(void* h, NF32* logits, NI64 ld, NI32 rows, NI32 vocab, NI32 n,
                                 NI64* outIds, NF32* outProbs, NU32 flags, void* stream);
typedef NI32 (*nls_token_nll_t)(void* h, NF32* logits, NI64 ld, NI32 rows, NI32 vocab,
                                NI64* targets, NF* outNll, NU32 flags, void* stream);
typedef NI32 (*nls_stream_status_t)(void* h, void* stream);
typedef char* (*nls_status_str_t)(NI32 s);
typedef char* (*nls_last_error_t)(void* h);
typedef char* (*nls_version_t)(void);
typedef NI32 (*nls_lm_head_t)(void* h, void* weights, NI32 wtype, NI32 rows, NI32 cols, NF32* x,
                              NI32 nb, NF32* y, NU32 flags, void* stream);
typedef NI32 (*nls_lm_head_sample_t)(void* h, void* weights, NI32 wtype, NI32 vocab, NI32 cols,
                                     NF32* x, NI32 rows, NlsRowParams* params, NI64* histIds,
                                     NI64* histOff, NI64* biasIds, NF* biasVals, NI64* biasOff,
                                     NF* uniforms, NI64* outIds, NF32* outProbs, NU32 flags,
                                     void* stream);
typedef NI32 (*nls_device_upload_t)(void* h, void* host, uint64_t bytes, void** outDev);
typedef void (*nls_device_free_t)(void* h, void* dev);

static struct {
  nls_create_t create;
  nls_destroy_t destroy;
  nls_sample_batch_t sample_batch;
  nls_argmax_batch_t argmax_batch;
  nls_top_tokens_t top_tokens;
  nls_token_nll_t token_nll;
  nls_stream_status_t stream_status;
  nls_status_str_t status_str;
  nls_last_error_t last_error;
  nls_version_t version;
  nls_lm_head_t lm_head;
  nls_lm_head_sample_t lm_head_sample;
  nls_device_upload_t device_upload;
  nls_device_free_t device_free;
} L;

/* what Nim's dynlib loader does at start-up (one dlsym per importc name) */
static int load(const char* path) {
  void* lib = dlopen(path, RTLD_NOW);
  if (!lib) { fprintf(stderr, "could not load: %s\n", dlerror()); return 1; }
#define SYM(field, name)                                          \
  do {                                                            \
    *(void**)&L.field = dlsym(lib, name);                         \
    if (!L.field) { fprintf(stderr, "could not import: %s\n", name); return 1; } \
  } while (0)
  SYM(create, "nls_create");
  SYM(destroy, "nls_destroy");
  SYM(sample_batch, "nls_sample_batch");
  SYM(argmax_batch, "nls_argmax_batch");
  SYM(top_tokens, "nls_top_tokens");
  SYM(token_nll, "nls_token_nll");
  SYM(stream_status, "nls_stream_status");
  SYM(status_str, "nls_status_str");
  SYM(last_error, "nls_last_error");
  SYM(version, "nls_version");
  SYM(lm_head, "nls_lm_head");
  SYM(lm_head_sample, "nls_lm_head_sample");
  SYM(device_upload, "nls_device_upload");
  SYM(device_free, "nls_device_free");
#undef SYM
  return 0;
}

/* ---- the Nim side: Sampler (params, rng, history) and sample ---------- */
typedef struct {
  NlsRowParams params;
  const NF* unif;   /* s.rng: the stream of rand(1.0) values */
  NI64 n_unif, used;
  NI64* history;    /* s.history (seq[int]) */
  NI64 hist_len, hist_cap;
  const NI64* bias_ids;  /* s.params.logitBias, as the binding flattens it */
  const NF* bias_vals;
  NI64 n_bias;
} Sampler;

static void* g_handle = NULL;  /* the module's handle, made on first use */
static const NI32 kMaxVocab = 262144;

/* raise CatchableError: the harness reports and exits */
static void raise_error(const char* what, NI32 st) {
  fprintf(stderr, "%s: %s (%s)\n", what, st ? L.status_str(st) : "",
          g_handle ? L.last_error(g_handle) : "");
  exit(3);
}

static NF rng_rand(Sampler* s) {
  if (s->used >= s->n_unif) { fprintf(stderr, "uniform stream exhausted\n"); exit(4); }
  return s->unif[s->used++];
}

/* proc sample*(s: Sampler; logitsIn: openArray[float32]): int  (sampler.nim:59) */
static NI64 sample(Sampler* s, const NF32* logitsIn, NI64 len, int* raised) {
  *raised = 0;
  if (len == 0) {
    /* greedy: argmax of nothing is 0 (sampler.nim:46-49); sampling indexes
       probs[0] (min-p) or, after drawing, idx[n - 1] of an empty seq */
    if (s->params.temperature <= 0) return 0;
    if (!(s->params.minP > 0)) (void)rng_rand(s);
    *raised = 1;
    return -1;
  }
  if (!g_handle) {
    NI32 st = L.create(&g_handle, 0, 1, kMaxVocab);
    if (st != 0) raise_error("nls_create", st);
  }
  NlsRowParams prm = s->params;
  NF u = (s->params.temperature > 0) ? rng_rand(s) : 0.0;
  NI64 hoff[2] = {0, s->hist_len};
  NI64 boff[2] = {0, s->n_bias};
  NI64 outId = -1;
  /* an empty list is passed as NULL ids and NULL offsets together */
  NI32 st = L.sample_batch(g_handle, (NF32*)logitsIn, len, 1, (NI32)len, &prm,
                           s->hist_len ? s->history : NULL, s->hist_len ? hoff : NULL,
                           s->n_bias ? (NI64*)s->bias_ids : NULL,
                           s->n_bias ? (NF*)s->bias_vals : NULL, s->n_bias ? boff : NULL, &u,
                           &outId, NULL, 0u, NULL);
  if (st != 0) raise_error("nls_sample_batch", st);
  return outId;
}

/* proc accept*(s: Sampler; tok: int)  (sampler.nim:41-43) */
static void accept(Sampler* s, NI64 tok) {
  if (s->hist_len == s->hist_cap) {
    s->hist_cap = s->hist_cap ? 2 * s->hist_cap : 64;
    s->history = (NI64*)realloc(s->history, (size_t)s->hist_cap * sizeof(NI64));
  }
  s->history[s->hist_len++] = tok;
}

static void rd(void* p, size_t n, FILE* f) {
  if (n && fread(p, 1, n, f) != n) { fprintf(stderr, "short input\n"); exit(2); }
}

int main(int argc, char** argv) {
  if (argc < 3) { fprintf(stderr, "usage: %s lib.so (--resolve-only | in out)\n", argv[0]); return 2; }
  if (load(argv[1])) return 1;
  if (!strcmp(argv[2], "--resolve-only")) {
    printf("%s\n", L.version());
    return 0;
  }
  FILE* f = fopen(argv[2], "rb");
  if (!f) return 2;
  NI64 hdr[6];
  rd(hdr, sizeof hdr, f);
  const NI64 V = hdr[0], steps_a = hdr[1], steps_b = hdr[2], n_hist0 = hdr[3], n_bias = hdr[4],
             n_unif = hdr[5];
  NlsRowParams pa, pb;
  rd(&pa, sizeof pa, f);
  rd(&pb, sizeof pb, f);
  NI64* hist0 = (NI64*)malloc((size_t)(n_hist0 + 1) * 8);
  NI64* bids = (NI64*)malloc((size_t)(n_bias + 1) * 8);
  NF* bvals = (NF*)malloc((size_t)(n_bias + 1) * 8);
  NF* unif = (NF*)malloc((size_t)(n_unif + 1) * 8);
  NF32* la = (NF32*)malloc((size_t)(steps_a * V + 1) * 4);
  NF32* lb = (NF32*)malloc((size_t)(steps_b * V + 1) * 4);
  rd(hist0, (size_t)n_hist0 * 8, f);
  rd(bids, (size_t)n_bias * 8, f);
  rd(bvals, (size_t)n_bias * 8, f);
  rd(unif, (size_t)n_unif * 8, f);
  rd(la, (size_t)(steps_a * V) * 4, f);
  rd(lb, (size_t)(steps_b * V) * 4, f);
  fclose(f);

  /* sampler A (sampling) and sampler B (greedy) share the uniform stream, so
     a greedy call that drew a uniform would shift every later draw of A */
  NI64 used = 0;
  Sampler a = {pa, unif, n_unif, 0, NULL, 0, 0, bids, bvals, n_bias};
  Sampler b = {pb, unif, n_unif, 0, NULL, 0, 0, NULL, NULL, 0};
  for (NI64 i = 0; i < n_hist0; ++i) accept(&a, hist0[i]);
  NI64* ids_a = (NI64*)malloc((size_t)(steps_a + 1) * 8);
  NI64* ids_b = (NI64*)malloc((size_t)(steps_b + 1) * 8);
  int raised;
  NI64 ib = 0;
  for (NI64 t = 0; t < steps_a; ++t) {
    /* chat.nim:204-208: let id = s.sample(logits); s.accept id */
    a.used = used;
    const NI64 id = sample(&a, la + t * V, V, &raised);
    used = a.used;
    ids_a[t] = id;
    accept(&a, id);
    if (t % 4 == 3 && ib < steps_b) {  /* interleave the greedy sampler */
      b.used = used;
      const NI64 g = sample(&b, lb + ib * V, V, &raised);
      used = b.used;
      ids_b[ib++] = g;
      accept(&b, g);
    }
  }
  /* empty logitsIn: greedy gives 0; sampling raises (after drawing when
     min-p is off, as the reference draws before idx[n - 1]) */
  NI64 probes[2];
  b.used = used;
  probes[0] = sample(&b, la, 0, &raised);
  used = b.used;
  a.used = used;
  (void)sample(&a, la, 0, &raised);
  used = a.used;
  probes[1] = raised;

  FILE* o = fopen(argv[3], "wb");
  if (!o) return 2;
  fwrite(ids_a, 8, (size_t)steps_a, o);
  fwrite(ids_b, 8, (size_t)steps_b, o);
  fwrite(&used, 8, 1, o);
  fwrite(probes, 8, 2, o);
  fclose(o);
  if (g_handle) L.destroy(g_handle);
  return 0;
}
