/*
 * nimllm_sample.h -- C ABI of libnimllm_sample.so, the B200 (sm_100a) token
 * sampler for nimllm.
 *
 * The library replaces the logits->token path of nimllm's Nim sampler
 * (src/nimllm/sampler.nim in the reference repository) and the output
 * projection that produces those logits (model.nim:466-470), plus
 * topTokens and perplexity's per-position term. Nim reaches it through
 * {.importc, dynlib: "libnimllm_sample.so".}; the Nim `Sampler` object keeps
 * its params, its history and its RNG on the host and passes one uniform per
 * sampled row. Every entry point below cites the reference interface it
 * replaces.
 *
 * Conventions
 *  - Plain C: pointers, sizes and status codes; no exceptions cross the ABI.
 *  - The caller owns every buffer; inputs are never written.
 *  - Token ids are Nim `int` (int64). Ids outside [0, vocab) in histories and
 *    bias lists are ignored, as in sampler.nim:70,76.
 *  - Rows are independent. Row r reads params[r], the history
 *    hist_ids[hist_off[r] .. hist_off[r+1]), the bias entries
 *    bias_ids/bias_vals[bias_off[r] .. bias_off[r+1]), logits + r*ld and
 *    uniforms[r].
 *  - Without NLS_DEVICE_INPUTS every input pointer is host memory; with it,
 *    every input pointer (logits, params, histories, bias, uniforms) is device
 *    memory of the handle's device. Likewise NLS_DEVICE_OUTPUTS for outputs.
 *  - A call whose outputs are host memory returns after the results are
 *    written (it synchronises `stream`). A call with device outputs is
 *    stream-ordered and returns at once; its kernel-side status (NaN rows,
 *    capacity) is read with nls_stream_status().
 *  - One handle per host thread / stream; calls on one handle must not
 *    overlap in time on the host.
 */
#ifndef NIMLLM_SAMPLE_H
#define NIMLLM_SAMPLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NLS_ABI_VERSION 1

#if defined(__GNUC__)
#define NLS_API __attribute__((visibility("default")))
#else
#define NLS_API
#endif

typedef int32_t nls_status;
enum {
  NLS_OK = 0,
  NLS_ERR_INVALID_ARG = 1, /* bad pointer/size/flag, duplicate bias id in a row */
  NLS_ERR_CUDA = 2,        /* a CUDA runtime call failed; see nls_last_error() */
  NLS_ERR_NCCL = 3,        /* a collective failed (vocab-sharded mode) */
  NLS_ERR_TIMEOUT = 4,     /* a bounded wait ran out */
  NLS_ERR_NAN_LOGITS = 5,  /* a full-sort row (top_k <= 0 or >= vocab) holds NaN after
                              penalties/bias/temperature; its out id is -1 (the
                              reference's stable sort then meets a comparator that
                              is not an order, and its output depends on the sort's
                              internals). Top-k rows with NaN return the
                              reference's own answer (see nls_sample_batch). */
  NLS_ERR_CAPACITY = 6,    /* rows/vocab beyond the handle's limits (a penalty window
                              or bias list of any length is supported) */
  NLS_ERR_NO_DEVICE = 7    /* no usable CUDA device */
};

/* flags */
#define NLS_DEVICE_INPUTS 1u  /* all input pointers are device memory */
#define NLS_DEVICE_OUTPUTS 2u /* out_ids / out_probs are device memory (async call) */

/* Per-row generation parameters: SamplerParams (sampler.nim:11-21) without
 * `seed` (the RNG stays in the Nim Sampler, sampler.nim:25,39) and without
 * `logitBias` (passed as the CSR bias lists). 64 bytes, no padding. */
typedef struct nls_row_params {
  double temperature;       /* sampler.nim:12  <= 0: greedy argmax                */
  double top_p;             /* sampler.nim:14  active iff 0 < top_p < 1           */
  double min_p;             /* sampler.nim:15  active iff min_p > 0               */
  double repeat_penalty;    /* sampler.nim:16  1.0 = off                          */
  double presence_penalty;  /* sampler.nim:18                                     */
  double frequency_penalty; /* sampler.nim:19                                     */
  int64_t top_k;            /* sampler.nim:13  <= 0 or >= vocab: full sort        */
  int64_t repeat_last_n;    /* sampler.nim:17  <= 0: the whole history            */
} nls_row_params;

typedef struct nls_handle nls_handle;

/* Create a handle bound to CUDA `device`, sized for up to max_rows rows of up
 * to max_vocab logits (1 <= max_vocab <= 262144). Replaces newSampler
 * (sampler.nim:37-39) as the owner of per-stream state: the handle owns the
 * device staging buffers and scratch; params/RNG/history stay with the
 * caller. */
NLS_API nls_status nls_create(nls_handle** out, int32_t device, int32_t max_rows, int32_t max_vocab);

/* Release a handle and its device memory. NULL is accepted. */
NLS_API void nls_destroy(nls_handle* h);

/* Sample one token per row: Sampler.sample (sampler.nim:59-121) for a batch of
 * independent samplers. Per row, in the reference's order: repeat/frequency/
 * presence penalties over the last repeat_last_n history ids (:63-74), logit
 * bias (:75-76), greedy argmax when temperature <= 0 (:77-78, no uniform
 * consumed), temperature (:80-81), top-k by the reference's heap rule or the
 * full stable sort (:83-97), softmax over the candidates (:98-100), top-p
 * (:102-108), min-p (:109-114) and the inverse-CDF draw with
 * uniforms[r] = rng.rand(1.0) (:115-121).
 *
 *  logits     [rows x ld] fp32, row-major, ld >= vocab
 *  params     [rows]
 *  hist_ids   history ids, CSR by hist_off[rows+1]; NULL = no history
 *  bias_ids, bias_vals, bias_off  logit bias, CSR; NULL = no bias.
 *             Ids must be unique within a row (a Nim Table); bias_vals are
 *             Nim floats and are rounded to float32 like `b.float32`.
 *  uniforms   [rows] in [0, 1); NULL only if every row is greedy
 *  out_ids    [rows] sampled token ids (-1 for a failed row)
 *  out_probs  [rows] softmax probability of the sampled token among the
 *             candidates (probs[i] in sampler.nim:100,120); NULL = not wanted.
 *             Greedy rows report 1.0.
 *  stream     cudaStream_t (NULL = legacy default stream)
 *
 * NaN after penalties, bias and temperature: a top-k row (0 < top_k < vocab)
 * gets the reference's answer. A NaN past the first top_k positions is never
 * pushed into its heap (:91) and is left out; a NaN among them stays in the
 * heap, every candidate probability is NaN, and the token is idx[0] when
 * min_p > 0, else idx[top_k - 1], in the heap's output order (:94-121), with
 * probability NaN. A full-sort row with a NaN fails (NLS_ERR_NAN_LOGITS). */
NLS_API nls_status nls_sample_batch(nls_handle* h, const float* logits, int64_t ld, int32_t rows,
                            int32_t vocab, const nls_row_params* params,
                            const int64_t* hist_ids, const int64_t* hist_off,
                            const int64_t* bias_ids, const double* bias_vals,
                            const int64_t* bias_off, const double* uniforms,
                            int64_t* out_ids, float* out_probs, uint32_t flags, void* stream);

/* argmax (sampler.nim:45-49) per row: first index of the maximum with the
 * reference's strict `>` (a NaN never wins unless it sits at index 0). */
NLS_API nls_status nls_argmax_batch(nls_handle* h, const float* logits, int64_t ld, int32_t rows,
                            int32_t vocab, int64_t* out_ids, uint32_t flags, void* stream);

/* topTokens (sampler.nim:123-130) per row: the n most probable tokens of the
 * softmax over the whole row (its fp32 sum taken in index order, as
 * softmaxInPlace does, sampler.nim:51-57), ordered by probability descending,
 * equal probabilities by ascending index. No penalties, bias or temperature
 * (the reference applies none). out_ids/out_probs are [rows x n]; entries
 * past min(n, vocab) get id -1 and probability 0. 1 <= n <= 256. A row with a
 * NaN or a non-finite maximum gets ids -1 and NLS_ERR_NAN_LOGITS (the
 * reference's probabilities are NaN there). Flags as nls_sample_batch. */
NLS_API nls_status nls_top_tokens(nls_handle* h, const float* logits, int64_t ld, int32_t rows,
                                  int32_t vocab, int32_t n, int64_t* out_ids, float* out_probs,
                                  uint32_t flags, void* stream);

/* Allocation-free sampling. No counterpart in the reference. Some callers
 * cannot call cudaMalloc -- a serving process that has given nearly all of
 * the GPU's memory to its own pool (an allocation would fail there), a host
 * whose memory policy forbids allocating after start-up, or a latency-critical
 * decode loop that cannot afford the device-wide synchronisation that
 * cudaMalloc/cudaFree imply -- and so cannot use nls_create. Same semantics
 * and arguments as nls_sample_batch with NLS_DEVICE_INPUTS |
 * NLS_DEVICE_OUTPUTS: every pointer is device memory of the current device,
 * the call is stream-ordered and returns after the launches; a row that fails
 * in the kernels gets out id -1 (its reason: nls_noalloc_status). It calls no
 * cudaMalloc/cudaFree and no allocating library routine: its scratch is one
 * fixed device array in the library (about 16 MiB, held by every GPU that
 * loads the library until the process exits). Limits: rows <= 4096 and
 * vocab <= 262144, else NLS_ERR_CAPACITY. The first call on a device looks up
 * that array's address and caches it: make that first call before any stream
 * capture begins, and do not call this entry point after cudaDeviceReset.
 * All calls share the array, which keeps the last call's contents (the
 * status word and counters are cleared by each call); calls that overlap on
 * the GPU race on it. */
NLS_API nls_status nls_sample_batch_noalloc(const float* logits, int64_t ld, int32_t rows,
                                            int32_t vocab, const nls_row_params* params,
                                            const int64_t* hist_ids, const int64_t* hist_off,
                                            const int64_t* bias_ids, const double* bias_vals,
                                            const int64_t* bias_off, const double* uniforms,
                                            int64_t* out_ids, float* out_probs, void* stream);

/* Kernel-side status of the last nls_sample_batch_noalloc call on the current
 * device (NLS_ERR_NAN_LOGITS, NLS_ERR_TIMEOUT, NLS_ERR_INVALID_ARG for a
 * duplicate bias id or a sampling row without uniforms; NLS_OK if none),
 * copied from the library's status word in stream order. With
 * NLS_DEVICE_OUTPUTS, `out` is device memory and the copy is asynchronous;
 * otherwise `out` is host memory and the call waits for `stream`. Allocates
 * nothing. No counterpart in the reference. */
NLS_API nls_status nls_noalloc_status(int32_t* out, uint32_t flags, void* stream);

/* ---- vocab-sharded mode ----------------------------------------------------
 * For logits produced by a tensor-parallel lm_head: each of P ranks (one
 * process and GPU each) holds the columns [r*Vs, min(vocab, (r+1)*Vs)) of
 * every row, Vs = ceil(vocab / P). No counterpart in the reference, which
 * samples one host row (sampler.nim:59); the results equal nls_sample_batch
 * on the whole rows bit for bit. The exact sequential sums need each row's
 * whole candidate order, so the call exchanges data rather than partial sums:
 * an NCCL send/recv transpose gives rank q every column of the rows it owns
 * (rows [floor(B*q/P), floor(B*(q+1)/P))), rank q samples those rows with the
 * batch kernels, and an NCCL all-gather returns every row's id (and prob) to
 * every rank. NCCL is the process's own libnccl.so.2, found at run time. */
typedef struct nls_comm nls_comm;

/* An NCCL unique id (128 bytes) for nls_comm_create; make it on one rank and
 * send it to the others out of band. */
NLS_API nls_status nls_comm_unique_id(uint8_t* out128);

/* Join the communicator of `nranks` ranks as `rank`, on CUDA `device` (the
 * device of the handle used with it). Collective: every rank calls it. The
 * communicator is non-blocking: the library polls its state against a host
 * deadline (120 s here, then nls_comm_set_timeout), and a rank that does not
 * join in time ends the call with NLS_ERR_TIMEOUT instead of a hang. */
NLS_API nls_status nls_comm_create(nls_comm** out, const uint8_t* id128, int32_t nranks,
                                   int32_t rank, int32_t device);
NLS_API void nls_comm_destroy(nls_comm* c);

/* Host deadline, in milliseconds, of each later vocab-sharded call on `c`
 * (default 120000): a call whose collectives have not finished by then --
 * another rank left, died or never made the call -- aborts the communicator
 * (ncclCommAbort, which ends the collectives in flight) and returns
 * NLS_ERR_TIMEOUT; later calls on it return NLS_ERR_NCCL. No counterpart in
 * the reference (single process). */
NLS_API nls_status nls_comm_set_timeout(nls_comm* c, uint64_t ms);

/* Abort the communicator at once (ncclCommAbort): for a rank that learns
 * out of band that a peer is gone. Local; later calls on `c` return
 * NLS_ERR_NCCL; release it with nls_comm_destroy. */
NLS_API nls_status nls_comm_abort(nls_comm* c);

/* Sample B rows whose vocabulary is split over the communicator's ranks (see
 * above). Collective and synchronous: every rank calls it with the same rows,
 * vocab, params, histories, bias and uniforms (replicated; ids are global
 * token ids) and its own shard `logits` [rows x ld], ld >= its column count.
 * Every pointer is device memory of the handle's device; out_ids (and
 * out_probs, optional) receive all B rows on every rank. Returns the first
 * non-zero status of any rank (NLS_ERR_NCCL for a failed collective), or
 * NLS_ERR_TIMEOUT when the collectives did not finish within the
 * communicator's deadline (the communicator is then aborted). */
NLS_API nls_status nls_sample_batch_vocab_sharded(
    nls_handle* h, nls_comm* c, const float* logits, int64_t ld, int32_t rows, int32_t vocab,
    const nls_row_params* params, const int64_t* hist_ids, const int64_t* hist_off,
    const int64_t* bias_ids, const double* bias_vals, const int64_t* bias_off,
    const double* uniforms, int64_t* out_ids, float* out_probs, void* stream);

/* Limit, in nanoseconds, of the bounded waits in which the streaming kernel
 * (greedy and top-k <= 256 rows) waits for its bulk copies of logits, and
 * in which the tensor-core path of nls_lm_head waits between its pipeline
 * stages (default 200 ms; later calls on this handle use it). A wait that
 * runs out fails its row (id -1) or the projection with NLS_ERR_TIMEOUT,
 * after the kernel has waited, with the default limit, for the copies (and
 * MMAs) it has in flight. A limit of 0 is a
 * deadline already past: every such wait gives up at once, which drives that
 * failure path on purpose (tests of the timeout handling). No counterpart in
 * the reference (its sampler runs on the host and waits for nothing). */
NLS_API nls_status nls_set_wait_limit(nls_handle* h, uint64_t ns);

/* Kernel-side status of the last asynchronous call on this handle: waits for
 * `stream` and returns the first error the kernels recorded (NLS_OK if none). */
NLS_API nls_status nls_stream_status(nls_handle* h, void* stream);

/* The per-position term of perplexity (model.nim:570-589): for each row r,
 * out_nll[r] = -(float64(x[targets[r]] - mx) - ln(s)), where mx is the row's
 * fp32 maximum, the difference is taken in fp32, and s is the float64 sum of
 * exp(float64(x_k - mx)) over the row (model.nim:581-584). The caller sums
 * the terms and takes exp(total / count) (:589). The sum runs in a tree order
 * rather than index order (float64 rounding differences only). A row with a
 * NaN or a non-finite maximum gets NaN and NLS_ERR_NAN_LOGITS; a target
 * outside [0, vocab) gets NaN and NLS_ERR_INVALID_ARG. Flags as
 * nls_sample_batch (targets is an input, out_nll an output). */
NLS_API nls_status nls_token_nll(nls_handle* h, const float* logits, int64_t ld, int32_t rows,
                                 int32_t vocab, const int64_t* targets, double* out_nll,
                                 uint32_t flags, void* stream);

/* ---- output projection ----------------------------------------------------
 * The matmul that produces the sampler's logits, matmul(m.output, xb, logits,
 * nb) (model.nim:466-470 -> :179-189, row task :144-169), computed on the GPU
 * bit for bit: the same path choice (int8 activations by default, the float
 * path under exactMatmul), the same integer block products and the same fp32
 * rounding order per output. No LoRA (the reference adds LoRA after the
 * projection, model.nim:190-195). */

/* ggml weight types accepted (GgmlType codes, quant.nim:14-19) */
#define NLS_WT_F32 0
#define NLS_WT_F16 1
#define NLS_WT_Q4_0 2
#define NLS_WT_Q8_0 8
#define NLS_WT_Q6_K 14
/* flag: the reference's `exactMatmul = true` (model.nim:173): float path
 * (dequantRow + dotF32) for every weight type */
#define NLS_EXACT_MATMUL 4u
/* flag: the rows are independent sequences (separate Chats sharing one
 * model, each evaluating one token): choose the matmul path as
 * model.nim:185 does for nb = 1, so that every row's logits equal a
 * one-row call's (without it, Q8_0 weights with nb > 4 take the float path
 * as one nb-row matmul would) */
#define NLS_ROWS_INDEPENDENT 8u

/* y[b*rows + r] = weight row r . x[b*cols ..] for b < nb (matmul, model.nim:179).
 *  weights  device memory of the handle's device, 16-byte aligned: `rows`
 *           rows of `cols` values in the ggml layout of `wtype` (rowBytes,
 *           quant.nim:65-71), rows back to back (QMatrix.data, model.nim:88)
 *  x        [nb x cols] fp32 activations (the normalised hidden state)
 *  y        [nb x rows] fp32
 * Path, as model.nim:185: with int8 activations (quantizeAct per block of 32,
 * or 256 for Q6_K, then integer block dot products) unless NLS_EXACT_MATMUL
 * is set, the type is F32/F16, or the type is Q8_0 and nb > 4; otherwise
 * dequantised weights and the eight-accumulator fp32 dot product.
 * cols must be a whole number of blocks (32 for Q4_0/Q8_0, 256 for Q6_K) and
 * at most 16384 for F32/F16. Non-finite activations on the int8 path give
 * NLS_ERR_NAN_LOGITS (the reference's int8 conversion of them is undefined).
 * On the int8 path, Q6_K and Q4_0 at 8 or more batch rows, and Q8_0 rows
 * that are separate sequences (NLS_ROWS_INDEPENDENT) at 8 or more, run on
 * the tensor cores with the same results (up to 5376, 4352 and 6144 columns
 * for Q6_K, Q8_0 and Q4_0); a wait of that pipeline that runs out
 * (nls_set_wait_limit) gives NLS_ERR_TIMEOUT, after the copies and MMAs in
 * flight have finished under the default limit, and leaves the logits
 * undefined.
 * Flags: NLS_DEVICE_INPUTS (x), NLS_DEVICE_OUTPUTS (y), NLS_EXACT_MATMUL,
 * NLS_ROWS_INDEPENDENT. */
NLS_API nls_status nls_lm_head(nls_handle* h, const void* weights, int32_t wtype, int32_t rows,
                               int32_t cols, const float* x, int32_t nb, float* y,
                               uint32_t flags, void* stream);

/* Device copies of caller data (no counterpart in the reference): allocate
 * `bytes` on the handle's device and copy `host` there (synchronously);
 * *out_dev receives the device address (256-byte aligned). For the output
 * layer's weights (QMatrix.data, model.nim:88), uploaded once after loading
 * the model. Free with nls_device_free. */
NLS_API nls_status nls_device_upload(nls_handle* h, const void* host, uint64_t bytes, void** out_dev);
NLS_API void nls_device_free(nls_handle* h, void* dev);

/* The output projection followed by sampling, the two steps of one decode
 * step's tail (model.nim:466-470, then Sampler.sample, sampler.nim:59-121):
 * logits = nls_lm_head(weights, wtype, vocab, cols, x, rows) stay in the
 * handle's device memory (never copied to the host) and nls_sample_batch
 * samples them with the given params, histories, bias and uniforms.
 * Flags and outputs as nls_sample_batch (NLS_DEVICE_INPUTS covers x and the
 * sampling inputs; weights are always device memory), plus NLS_EXACT_MATMUL
 * and NLS_ROWS_INDEPENDENT (one decode step of `rows` separate Chats).
 * rows <= the handle's max_rows, vocab <= its max_vocab. */
NLS_API nls_status nls_lm_head_sample(nls_handle* h, const void* weights, int32_t wtype,
                                      int32_t vocab, int32_t cols, const float* x, int32_t rows,
                                      const nls_row_params* params, const int64_t* hist_ids,
                                      const int64_t* hist_off, const int64_t* bias_ids,
                                      const double* bias_vals, const int64_t* bias_off,
                                      const double* uniforms, int64_t* out_ids, float* out_probs,
                                      uint32_t flags, void* stream);

/* Per-kernel timing of later calls on this handle (tracing; no counterpart
 * in the reference, which only times whole generations with epochTime,
 * chat.nim:191,246-247). With `on` set, every sampling call records CUDA
 * events around each of its kernels on the call's stream. */
NLS_API nls_status nls_set_profiling(nls_handle* h, int32_t on);

/* Device times in milliseconds of the last profiled call, each measured from
 * the call's start on its stream: out_ms[0] to the end of the streaming
 * kernel (greedy and top-k <= 256 rows), out_ms[1] to the end of the
 * full-sort kernel (the other rows; above 8 rows it runs concurrently with the
 * streaming kernel, else after it), out_ms[2] to the end of the call's last
 * kernel (above 8 rows, a second full-sort
 * launch over rows the streaming kernel handed back). Waits for those events.
 * `n` is the capacity of out_ms (up to 3 values are written). */
NLS_API nls_status nls_last_kernel_ms(nls_handle* h, float* out_ms, int32_t n);

/* The exponential the sampling kernels use for the reference's expf (Nim's
 * exp(float32), i.e. the C library's expf, sampler.nim:56), evaluated on the
 * current device for the n consecutive float bit patterns starting at
 * first_bits: out[i] = expf(float with bits first_bits + i). out_estimate
 * (optional) receives the cheaper estimate the full-sort kernel uses only to
 * decide rounding units. Both are device memory; stream-ordered. For tests
 * that hold the device function against the host's expf bit for bit.
 * No counterpart in the reference (a numerics check of the library). */
NLS_API nls_status nls_ref_expf_range(uint32_t first_bits, int64_t n, float* out,
                                      float* out_estimate, void* stream);

/* Human-readable text of a status code / of the handle's last CUDA error. */
NLS_API const char* nls_status_str(nls_status s);
NLS_API const char* nls_last_error(const nls_handle* h);

/* Library version string, e.g. "nimllm-sample-b200 0.1.0 (sm_100a)". */
NLS_API const char* nls_version(void);

#ifdef __cplusplus
}
#endif
#endif /* NIMLLM_SAMPLE_H */
