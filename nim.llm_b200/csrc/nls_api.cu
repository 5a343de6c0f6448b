// nls_api.cu -- the C ABI of libnimllm_sample.so (include/nimllm_sample.h).
//
// Host glue only: argument checks, staging of host inputs into device
// buffers owned by the handle, the two kernel launches, and the read-back of
// results and status. No sampling arithmetic happens on the host, and there
// is no CPU fallback: without a usable CUDA device every call fails with
// NLS_ERR_NO_DEVICE or NLS_ERR_CUDA.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <new>

#include "nls_kernels.h"
#include "nls_nccl.h"
#include "nimllm_sample.h"

struct nls_handle {
  int device = 0;
  int max_rows = 0;
  int max_vocab = 0;
  int sm_count = 0;
  // staging for host inputs (grown on demand)
  float* d_logits = nullptr;
  size_t logits_cap = 0;
  nls_row_params* d_params = nullptr;
  double* d_uniforms = nullptr;
  int64_t* d_hist_off = nullptr;
  int64_t* d_bias_off = nullptr;
  int64_t* d_hist = nullptr;
  size_t hist_cap = 0;
  int64_t* d_bias_ids = nullptr;
  double* d_bias_vals = nullptr;
  size_t bias_cap = 0;
  size_t bias_vals_cap = 0;
  // outputs for host-output calls
  int64_t* d_out_ids = nullptr;
  float* d_out_probs = nullptr;
  // [0] status, [1] full_count, [2] row_claim, [3] claim_count,
  // [4 .. 4+max_rows) full_list, [4+max_rows .. 4+2*max_rows) claim_list
  int* d_work = nullptr;
  // full-sort scratch: slots x 4 x vpad words
  uint32_t* d_scratch = nullptr;
  int vpad = 0;
  int slots = 0;
  int* h_status = nullptr;  // pinned
  // the streaming kernel runs on `side`, forked from and joined back into the
  // caller's stream, concurrently with the full-sort kernel
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  // profiling: [0] start, [1] streaming kernel done, [2] full-sort kernel
  // done, [3] fallback launch done
  int profiling = 0;
  int profiled = 0;
  // limit of the streaming kernel's bulk-copy waits and of the tensor-core
  // output projection's pipeline waits (nls_set_wait_limit)
  unsigned long long wait_ns = 200ull * 1000ull * 1000ull;
  cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
  // vocab-sharded calls: packed shard, received shards, gathered ids/probs
  float* d_sh_send = nullptr;
  size_t sh_send_cap = 0;
  float* d_sh_recv = nullptr;
  size_t sh_recv_cap = 0;
  int64_t* d_sh_mine = nullptr;
  size_t sh_mine_cap = 0;
  int64_t* d_sh_all = nullptr;
  size_t sh_all_cap = 0;
  float* d_sh_pmine = nullptr;
  size_t sh_pmine_cap = 0;
  float* d_sh_pall = nullptr;
  size_t sh_pall_cap = 0;
  int64_t* h_sh_status = nullptr;  // pinned, one per rank (up to kMaxRanks)
  // nls_token_nll with host buffers: targets in, terms out
  int64_t* d_tgt = nullptr;
  size_t tgt_cap = 0;
  double* d_nll = nullptr;
  size_t nll_cap = 0;
  // output projection: staged activations, host-output logits
  float* d_lmx = nullptr;
  size_t lmx_cap = 0;
  uint8_t* d_lmq = nullptr;  // the tensor-core projection's quantized activations
  size_t lmq_cap = 0;
  float* d_lmy = nullptr;
  size_t lmy_cap = 0;
  char last_err[256] = {0};
};

struct nls_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
  int device = 0;
  // host deadline of each collective call (nls_comm_set_timeout)
  unsigned long long timeout_ms = 120000ull;
  bool aborted = false;  // ncclCommAbort has run: the communicator is dead
};

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

nls_status cuda_fail(nls_handle* h, cudaError_t e, const char* what) {
  if (h) snprintf(h->last_err, sizeof h->last_err, "%s: %s", what, cudaGetErrorString(e));
  return NLS_ERR_CUDA;
}

#define NLS_CUDA(h, call)                                   \
  do {                                                      \
    cudaError_t e_ = (call);                                \
    if (e_ != cudaSuccess) return cuda_fail((h), e_, #call); \
  } while (0)

template <class T>
nls_status grow(nls_handle* h, T** p, size_t* cap, size_t n) {
  if (n <= *cap && *p) return NLS_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  size_t want = n < 1024 ? 1024 : n;
  NLS_CUDA(h, cudaMalloc((void**)p, want * sizeof(T)));
  *cap = want;
  return NLS_OK;
}

bool csr_ok(const int64_t* off, int rows) {
  if (off[0] < 0) return false;
  for (int r = 0; r < rows; ++r)
    if (off[r + 1] < off[r]) return false;
  return true;
}

int pick_cluster(const nls_handle* h, int rows, int vocab) {
  const char* env = getenv("NLS_CLUSTER");
  int C = 1;
  if (env && *env) {
    C = atoi(env);
  } else if (vocab >= 8192) {
    C = (h->sm_count + rows - 1) / (rows > 0 ? rows : 1);  // split rows only when SMs are left
  }
  int maxc = vocab / 2048;
  if (C > maxc) C = maxc;
  if (C > 8) {
    const int big = nls::light_max_cluster(vocab);
    if (C > big) C = big;
  }
  if (C < 1) C = 1;
  return C;
}

constexpr int kSmallBatch = 8;
constexpr int kMaxRanks = 64;

// One batch: the streaming kernel (greedy and top-k <= 256 rows) on the side
// stream, concurrently with the full-sort kernel, which claims the full-path
// rows itself; then a second full-sort launch for the rows the streaming
// kernel handed back (ties or thresholds it could not settle; usually none).
// Batches of at most kSmallBatch rows run the two kernels one after the
// other instead (the fork/join costs more than the overlap gains).
// keep_status: d_work[0] already holds the status of an earlier kernel of
// the same call (the output projection), which must survive.
nls_status run_batch(nls_handle* h, const nls::BatchArgs& a_in, uint32_t flags, cudaStream_t st,
                     bool keep_status = false) {
  nls::BatchArgs a = a_in;
  a.wait_ns = h->wait_ns;
  a.status = h->d_work;
  a.full_count = h->d_work + 1;
  a.full_list = h->d_work + 4;
  a.row_claim = nullptr;
  a.skip_full = 0;
  if (keep_status)
    NLS_CUDA(h, cudaMemsetAsync(h->d_work + 1, 0, 3 * sizeof(int), st));
  else
    NLS_CUDA(h, cudaMemsetAsync(h->d_work, 0, 4 * sizeof(int), st));
  const int C = pick_cluster(h, a.rows, a.V);
  int chunk = (a.V + C - 1) / C;
  chunk = (chunk + 3) & ~3;
  const bool prof = h->profiling != 0;
  if (prof) NLS_CUDA(h, cudaEventRecord(h->ev[0], st));
  if (a.argmax_only) {
    NLS_CUDA(h, nls::launch_light(a, C, chunk, st));
    if (prof) {
      NLS_CUDA(h, cudaEventRecord(h->ev[1], st));
      NLS_CUDA(h, cudaEventRecord(h->ev[2], st));
      NLS_CUDA(h, cudaEventRecord(h->ev[3], st));
    }
  } else if (a.rows <= kSmallBatch) {
    // a few rows: the streaming kernel hands full-path rows to one
    // full-sort launch after it (two launches, no fork/join)
    // (no event between the two: the full-sort launch is the streaming
    // kernel's programmatic dependent; profiling reports the pair's time)
    NLS_CUDA(h, nls::launch_light(a, C, chunk, st));
    NLS_CUDA(h, nls::launch_full(a, h->d_scratch, h->vpad, h->slots, st, true));
    if (prof) {
      NLS_CUDA(h, cudaEventRecord(h->ev[1], st));
      NLS_CUDA(h, cudaEventRecord(h->ev[2], st));
      NLS_CUDA(h, cudaEventRecord(h->ev[3], st));
    }
  } else {
    nls::BatchArgs af = a;
    af.row_claim = h->d_work + 2;
    if (a.rows > 4 * h->sm_count) {
      // many rows: the full-path rows are listed first, so that each claim
      // is one atomic (walking thousands of rows per claim held every SM
      // for ~0.1 ms on config 4); a few hundred rows are walked directly
      af.claim_count = h->d_work + 3;
      af.claim_list = h->d_work + 4 + h->max_rows;
      NLS_CUDA(h, nls::launch_classify(af, h->d_work + 4 + h->max_rows, h->d_work + 3, st));
    }
    // The streaming kernel forks only now, so that the full-sort kernel,
    // whose slowest row sets the call's time, is dispatched onto the SMs
    // first (its CTAs cannot share an SM with streaming CTAs).
    NLS_CUDA(h, cudaEventRecord(h->fork, st));
    NLS_CUDA(h, cudaStreamWaitEvent(h->side, h->fork, 0));
    NLS_CUDA(h, nls::launch_full(af, h->d_scratch, h->vpad, h->slots, st));
    if (prof) NLS_CUDA(h, cudaEventRecord(h->ev[2], st));
    nls::BatchArgs al = a;
    al.skip_full = 1;
    NLS_CUDA(h, nls::launch_light(al, C, chunk, h->side));
    if (prof) NLS_CUDA(h, cudaEventRecord(h->ev[1], h->side));
    NLS_CUDA(h, cudaEventRecord(h->join, h->side));
    NLS_CUDA(h, cudaStreamWaitEvent(st, h->join, 0));
    NLS_CUDA(h, nls::launch_full(a, h->d_scratch, h->vpad, h->slots, st));
    if (prof) NLS_CUDA(h, cudaEventRecord(h->ev[3], st));
  }
  h->profiled = prof ? 1 : 0;
  // host-output calls read the status at their end; device-output calls
  // leave it in d_work for nls_stream_status (no copy in their stream)
  if (!(flags & NLS_DEVICE_OUTPUTS))
    NLS_CUDA(h, cudaMemcpyAsync(h->h_status, h->d_work, sizeof(int), cudaMemcpyDeviceToHost, st));
  return NLS_OK;
}

}  // namespace

extern "C" {

const char* nls_version(void) { return "nimllm-sample-b200 0.1.0 (sm_100a)"; }

const char* nls_status_str(nls_status s) {
  switch (s) {
    case NLS_OK: return "ok";
    case NLS_ERR_INVALID_ARG: return "invalid argument";
    case NLS_ERR_CUDA: return "CUDA error";
    case NLS_ERR_NCCL: return "NCCL error";
    case NLS_ERR_TIMEOUT: return "timeout";
    case NLS_ERR_NAN_LOGITS: return "NaN logits in a sampling row";
    case NLS_ERR_CAPACITY: return "capacity exceeded";
    case NLS_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

const char* nls_last_error(const nls_handle* h) { return h ? h->last_err : "null handle"; }

nls_status nls_set_wait_limit(nls_handle* h, uint64_t ns) {
  if (!h) return NLS_ERR_INVALID_ARG;
  h->wait_ns = ns;
  return NLS_OK;
}

void nls_destroy(nls_handle* h) {
  if (!h) return;
  {
    DeviceGuard g(h->device);
    cudaFree(h->d_logits);
    cudaFree(h->d_params);
    cudaFree(h->d_uniforms);
    cudaFree(h->d_hist_off);
    cudaFree(h->d_bias_off);
    cudaFree(h->d_hist);
    cudaFree(h->d_bias_ids);
    cudaFree(h->d_bias_vals);
    cudaFree(h->d_out_ids);
    cudaFree(h->d_out_probs);
    cudaFree(h->d_work);
    cudaFree(h->d_scratch);
    if (h->h_status) cudaFreeHost(h->h_status);
    if (h->side) cudaStreamDestroy(h->side);
    cudaFree(h->d_sh_send);
    cudaFree(h->d_sh_recv);
    cudaFree(h->d_sh_mine);
    cudaFree(h->d_sh_all);
    cudaFree(h->d_sh_pmine);
    cudaFree(h->d_sh_pall);
    if (h->h_sh_status) cudaFreeHost(h->h_sh_status);
    cudaFree(h->d_tgt);
    cudaFree(h->d_nll);
    cudaFree(h->d_lmx);
    cudaFree(h->d_lmq);
    cudaFree(h->d_lmy);
    if (h->fork) cudaEventDestroy(h->fork);
    if (h->join) cudaEventDestroy(h->join);
    for (cudaEvent_t e : h->ev)
      if (e) cudaEventDestroy(e);
  }
  delete h;
}

nls_status nls_create(nls_handle** out, int32_t device, int32_t max_rows, int32_t max_vocab) {
  if (!out) return NLS_ERR_INVALID_ARG;
  *out = nullptr;
  if (max_rows < 1 || max_vocab < 1 || max_vocab > nls::kMaxVocab) return NLS_ERR_INVALID_ARG;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) return NLS_ERR_NO_DEVICE;
  if (device < 0 || device >= ndev) return NLS_ERR_INVALID_ARG;
  nls_handle* h = new (std::nothrow) nls_handle();
  if (!h) return NLS_ERR_CAPACITY;
  h->device = device;
  h->max_rows = max_rows;
  h->max_vocab = max_vocab;
  DeviceGuard g(device);
  nls_status st = NLS_OK;
  auto fail = [&](cudaError_t e, const char* what) {
    st = cuda_fail(h, e, what);
    return st;
  };
  cudaError_t e;
  if ((e = cudaDeviceGetAttribute(&h->sm_count, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) {
    fail(e, "cudaDeviceGetAttribute");
  } else if ((e = cudaMalloc(&h->d_params, sizeof(nls_row_params) * max_rows)) != cudaSuccess) {
    fail(e, "cudaMalloc(params)");
  } else if ((e = cudaMalloc(&h->d_uniforms, sizeof(double) * max_rows)) != cudaSuccess) {
    fail(e, "cudaMalloc(uniforms)");
  } else if ((e = cudaMalloc(&h->d_hist_off, sizeof(int64_t) * (max_rows + 1))) != cudaSuccess) {
    fail(e, "cudaMalloc(hist_off)");
  } else if ((e = cudaMalloc(&h->d_bias_off, sizeof(int64_t) * (max_rows + 1))) != cudaSuccess) {
    fail(e, "cudaMalloc(bias_off)");
  } else if ((e = cudaMalloc(&h->d_out_ids, sizeof(int64_t) * max_rows)) != cudaSuccess) {
    fail(e, "cudaMalloc(out_ids)");
  } else if ((e = cudaMalloc(&h->d_out_probs, sizeof(float) * max_rows)) != cudaSuccess) {
    fail(e, "cudaMalloc(out_probs)");
  } else if ((e = cudaMalloc(&h->d_work, sizeof(int) * (4 + 2 * (size_t)max_rows))) != cudaSuccess) {
    fail(e, "cudaMalloc(work)");
  } else if ((e = cudaStreamCreateWithFlags(&h->side, cudaStreamNonBlocking)) != cudaSuccess) {
    fail(e, "cudaStreamCreate(side)");
  } else if ((e = cudaEventCreateWithFlags(&h->fork, cudaEventDisableTiming)) != cudaSuccess) {
    fail(e, "cudaEventCreate(fork)");
  } else if ((e = cudaEventCreateWithFlags(&h->join, cudaEventDisableTiming)) != cudaSuccess) {
    fail(e, "cudaEventCreate(join)");
  } else if ((e = cudaMallocHost(&h->h_status, sizeof(int))) != cudaSuccess) {
    fail(e, "cudaMallocHost(status)");
  }
  if (st == NLS_OK) {
    h->vpad = (max_vocab + 31) & ~31;
    h->slots = h->sm_count;
    size_t words = (size_t)h->slots * 4 * (size_t)h->vpad;
    if ((e = cudaMalloc(&h->d_scratch, words * sizeof(uint32_t))) != cudaSuccess)
      fail(e, "cudaMalloc(scratch)");
  }
  if (st != NLS_OK) {
    nls_destroy(h);
    return st;
  }
  *h->h_status = 0;
  *out = h;
  return NLS_OK;
}

}  // extern "C"

namespace {

// nls_sample_batch after its argument checks. logits_dev: the logits are
// device memory even when the other inputs are host memory (the output
// projection wrote them); keep_status as run_batch.
nls_status sample_impl(nls_handle* h, const float* logits, int64_t ld, bool logits_dev,
                       bool keep_status, int32_t rows, int32_t vocab,
                       const nls_row_params* params, const int64_t* hist_ids,
                       const int64_t* hist_off, const int64_t* bias_ids,
                       const double* bias_vals, const int64_t* bias_off,
                       const double* uniforms, int64_t* out_ids, float* out_probs,
                       uint32_t flags, cudaStream_t st) {
  const bool dev_in = (flags & NLS_DEVICE_INPUTS) != 0;
  const bool dev_out = (flags & NLS_DEVICE_OUTPUTS) != 0;

  nls::BatchArgs a{};
  a.rows = rows;
  a.V = vocab;
  a.argmax_only = 0;
  if (dev_in) {
    a.logits = logits;
    a.ld = ld;
    a.params = params;
    a.hist_ids = hist_ids;
    a.hist_off = hist_off;
    a.bias_ids = bias_ids;
    a.bias_vals = bias_vals;
    a.bias_off = bias_off;
    a.uniforms = uniforms;
  } else {
    nls_status s;
    if (logits_dev) {
      a.logits = logits;
      a.ld = ld;
    } else {
      if ((s = grow(h, &h->d_logits, &h->logits_cap, (size_t)rows * vocab)) != NLS_OK) return s;
      NLS_CUDA(h, cudaMemcpy2DAsync(h->d_logits, (size_t)vocab * sizeof(float), logits,
                                    (size_t)ld * sizeof(float), (size_t)vocab * sizeof(float), rows,
                                    cudaMemcpyHostToDevice, st));
      a.logits = h->d_logits;
      a.ld = vocab;
    }
    NLS_CUDA(h, cudaMemcpyAsync(h->d_params, params, sizeof(nls_row_params) * rows,
                                cudaMemcpyHostToDevice, st));
    a.params = h->d_params;
    if (uniforms) {
      NLS_CUDA(h, cudaMemcpyAsync(h->d_uniforms, uniforms, sizeof(double) * rows,
                                  cudaMemcpyHostToDevice, st));
      a.uniforms = h->d_uniforms;
    }
    if (hist_ids) {
      if (!csr_ok(hist_off, rows)) return NLS_ERR_INVALID_ARG;
      const size_t n = (size_t)hist_off[rows];
      if ((s = grow(h, &h->d_hist, &h->hist_cap, n)) != NLS_OK) return s;
      if (n) NLS_CUDA(h, cudaMemcpyAsync(h->d_hist, hist_ids, n * sizeof(int64_t), cudaMemcpyHostToDevice, st));
      NLS_CUDA(h, cudaMemcpyAsync(h->d_hist_off, hist_off, sizeof(int64_t) * (rows + 1),
                                  cudaMemcpyHostToDevice, st));
      a.hist_ids = h->d_hist;
      a.hist_off = h->d_hist_off;
    }
    if (bias_ids) {
      if (!csr_ok(bias_off, rows)) return NLS_ERR_INVALID_ARG;
      const size_t n = (size_t)bias_off[rows];
      if ((s = grow(h, &h->d_bias_ids, &h->bias_cap, n)) != NLS_OK) return s;
      if ((s = grow(h, &h->d_bias_vals, &h->bias_vals_cap, n)) != NLS_OK) return s;
      if (n) {
        NLS_CUDA(h, cudaMemcpyAsync(h->d_bias_ids, bias_ids, n * sizeof(int64_t), cudaMemcpyHostToDevice, st));
        NLS_CUDA(h, cudaMemcpyAsync(h->d_bias_vals, bias_vals, n * sizeof(double), cudaMemcpyHostToDevice, st));
      }
      NLS_CUDA(h, cudaMemcpyAsync(h->d_bias_off, bias_off, sizeof(int64_t) * (rows + 1),
                                  cudaMemcpyHostToDevice, st));
      a.bias_ids = h->d_bias_ids;
      a.bias_vals = h->d_bias_vals;
      a.bias_off = h->d_bias_off;
    }
  }
  a.out_ids = dev_out ? out_ids : h->d_out_ids;
  a.out_probs = dev_out ? out_probs : (out_probs ? h->d_out_probs : nullptr);
  nls_status s = run_batch(h, a, flags, st, keep_status);
  if (s != NLS_OK) return s;
  if (dev_out) return NLS_OK;
  NLS_CUDA(h, cudaMemcpyAsync(out_ids, h->d_out_ids, sizeof(int64_t) * rows, cudaMemcpyDeviceToHost, st));
  if (out_probs)
    NLS_CUDA(h, cudaMemcpyAsync(out_probs, h->d_out_probs, sizeof(float) * rows, cudaMemcpyDeviceToHost, st));
  NLS_CUDA(h, cudaStreamSynchronize(st));
  return (nls_status)*h->h_status;
}

// Output projection into dy [nb x rows] (device) from x (host or device per
// x_dev); the kernel status goes to d_work[0], which the caller has cleared.
nls_status lm_head_impl(nls_handle* h, const void* weights, int32_t wtype, int32_t rows,
                        int32_t cols, const float* x, bool x_dev, int32_t nb, float* dy,
                        uint32_t flags, cudaStream_t st) {
  const bool exact = (flags & NLS_EXACT_MATMUL) != 0;
  const int path_nb = (flags & NLS_ROWS_INDEPENDENT) ? 1 : nb;
  nls_status s;
  const float* dx = x;
  if (!x_dev) {
    if ((s = grow(h, &h->d_lmx, &h->lmx_cap, (size_t)nb * cols)) != NLS_OK) return s;
    NLS_CUDA(h, cudaMemcpyAsync(h->d_lmx, x, sizeof(float) * (size_t)nb * cols, cudaMemcpyHostToDevice, st));
    dx = h->d_lmx;
  }
  // the tensor-core path (8 or more batch rows) quantizes the activations
  // once per launch into this scratch
  if (nb >= 8 && (s = grow(h, &h->d_lmq, &h->lmq_cap, nls::lm_head_act_scratch_bytes(cols))) != NLS_OK) return s;
  NLS_CUDA(h, nls::launch_lm_head(static_cast<const uint8_t*>(weights), wtype, rows, cols, dx, nb,
                                  path_nb, dy, exact, h->d_work, h->sm_count, h->wait_ns, h->d_lmq, st));
  return NLS_OK;
}

bool lm_head_args_ok(const void* weights, int32_t wtype, int32_t rows, int32_t cols) {
  int64_t rb = 0;
  if (!weights || (reinterpret_cast<uintptr_t>(weights) & 15) != 0) return false;
  if (rows < 1 || cols < 1 || !nls::lm_head_row_bytes(wtype, cols, &rb)) return false;
  // the float path keeps a batch row of x in shared memory
  return (wtype != 0 && wtype != 1) || cols <= 16384;
}

}  // namespace

extern "C" {

nls_status nls_sample_batch(nls_handle* h, const float* logits, int64_t ld, int32_t rows,
                            int32_t vocab, const nls_row_params* params,
                            const int64_t* hist_ids, const int64_t* hist_off,
                            const int64_t* bias_ids, const double* bias_vals,
                            const int64_t* bias_off, const double* uniforms, int64_t* out_ids,
                            float* out_probs, uint32_t flags, void* stream) {
  if (!h) return NLS_ERR_INVALID_ARG;
  if (flags & ~(NLS_DEVICE_INPUTS | NLS_DEVICE_OUTPUTS)) return NLS_ERR_INVALID_ARG;
  if (rows < 0 || vocab < 1 || ld < vocab) return NLS_ERR_INVALID_ARG;
  if (rows == 0) return NLS_OK;
  if (!logits || !params || !out_ids) return NLS_ERR_INVALID_ARG;
  if ((hist_ids == nullptr) != (hist_off == nullptr)) return NLS_ERR_INVALID_ARG;
  if ((bias_ids == nullptr) != (bias_off == nullptr) || (bias_ids == nullptr) != (bias_vals == nullptr))
    return NLS_ERR_INVALID_ARG;
  if (rows > h->max_rows || vocab > h->max_vocab) return NLS_ERR_CAPACITY;
  DeviceGuard g(h->device);
  return sample_impl(h, logits, ld, (flags & NLS_DEVICE_INPUTS) != 0, false, rows, vocab, params,
                     hist_ids, hist_off, bias_ids, bias_vals, bias_off, uniforms, out_ids,
                     out_probs, flags, (cudaStream_t)stream);
}

nls_status nls_device_upload(nls_handle* h, const void* host, uint64_t bytes, void** out_dev) {
  if (!h || !out_dev || (bytes && !host)) return NLS_ERR_INVALID_ARG;
  *out_dev = nullptr;
  DeviceGuard g(h->device);
  void* d = nullptr;
  NLS_CUDA(h, cudaMalloc(&d, bytes ? bytes : 16));
  if (bytes) {
    const cudaError_t e = cudaMemcpy(d, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(d);
      return cuda_fail(h, e, "cudaMemcpy (nls_device_upload)");
    }
  }
  *out_dev = d;
  return NLS_OK;
}

void nls_device_free(nls_handle* h, void* dev) {
  if (!h || !dev) return;
  DeviceGuard g(h->device);
  cudaFree(dev);
}

nls_status nls_lm_head(nls_handle* h, const void* weights, int32_t wtype, int32_t rows,
                       int32_t cols, const float* x, int32_t nb, float* y, uint32_t flags,
                       void* stream) {
  if (!h) return NLS_ERR_INVALID_ARG;
  if (flags & ~(NLS_DEVICE_INPUTS | NLS_DEVICE_OUTPUTS | NLS_EXACT_MATMUL | NLS_ROWS_INDEPENDENT))
    return NLS_ERR_INVALID_ARG;
  if (nb < 0 || rows < 0) return NLS_ERR_INVALID_ARG;
  if (nb == 0 || rows == 0) return NLS_OK;
  if (!x || !y || !lm_head_args_ok(weights, wtype, rows, cols)) return NLS_ERR_INVALID_ARG;
  DeviceGuard g(h->device);
  cudaStream_t st = (cudaStream_t)stream;
  const bool dev_out = (flags & NLS_DEVICE_OUTPUTS) != 0;
  nls_status s;
  float* dy = y;
  if (!dev_out) {
    if ((s = grow(h, &h->d_lmy, &h->lmy_cap, (size_t)nb * rows)) != NLS_OK) return s;
    dy = h->d_lmy;
  }
  NLS_CUDA(h, cudaMemsetAsync(h->d_work, 0, sizeof(int), st));
  if ((s = lm_head_impl(h, weights, wtype, rows, cols, x, (flags & NLS_DEVICE_INPUTS) != 0, nb, dy,
                        flags, st)) != NLS_OK)
    return s;
  if (dev_out) return NLS_OK;
  NLS_CUDA(h, cudaMemcpyAsync(h->h_status, h->d_work, sizeof(int), cudaMemcpyDeviceToHost, st));
  NLS_CUDA(h, cudaMemcpyAsync(y, dy, sizeof(float) * (size_t)nb * rows, cudaMemcpyDeviceToHost, st));
  NLS_CUDA(h, cudaStreamSynchronize(st));
  return (nls_status)*h->h_status;
}

nls_status nls_lm_head_sample(nls_handle* h, const void* weights, int32_t wtype, int32_t vocab,
                              int32_t cols, const float* x, int32_t rows,
                              const nls_row_params* params, const int64_t* hist_ids,
                              const int64_t* hist_off, const int64_t* bias_ids,
                              const double* bias_vals, const int64_t* bias_off,
                              const double* uniforms, int64_t* out_ids, float* out_probs,
                              uint32_t flags, void* stream) {
  if (!h) return NLS_ERR_INVALID_ARG;
  if (flags & ~(NLS_DEVICE_INPUTS | NLS_DEVICE_OUTPUTS | NLS_EXACT_MATMUL | NLS_ROWS_INDEPENDENT))
    return NLS_ERR_INVALID_ARG;
  if (rows < 0) return NLS_ERR_INVALID_ARG;
  if (rows == 0) return NLS_OK;
  if (!x || !params || !out_ids || !lm_head_args_ok(weights, wtype, vocab, cols))
    return NLS_ERR_INVALID_ARG;
  if ((hist_ids == nullptr) != (hist_off == nullptr)) return NLS_ERR_INVALID_ARG;
  if ((bias_ids == nullptr) != (bias_off == nullptr) || (bias_ids == nullptr) != (bias_vals == nullptr))
    return NLS_ERR_INVALID_ARG;
  if (rows > h->max_rows || vocab > h->max_vocab) return NLS_ERR_CAPACITY;
  DeviceGuard g(h->device);
  cudaStream_t st = (cudaStream_t)stream;
  nls_status s;
  if ((s = grow(h, &h->d_logits, &h->logits_cap, (size_t)rows * vocab)) != NLS_OK) return s;
  NLS_CUDA(h, cudaMemsetAsync(h->d_work, 0, sizeof(int), st));
  if ((s = lm_head_impl(h, weights, wtype, vocab, cols, x, (flags & NLS_DEVICE_INPUTS) != 0, rows,
                        h->d_logits, flags, st)) != NLS_OK)
    return s;
  return sample_impl(h, h->d_logits, vocab, true, true, rows, vocab, params, hist_ids, hist_off,
                     bias_ids, bias_vals, bias_off, uniforms, out_ids, out_probs,
                     flags & ~(NLS_EXACT_MATMUL | NLS_ROWS_INDEPENDENT), st);
}

nls_status nls_argmax_batch(nls_handle* h, const float* logits, int64_t ld, int32_t rows,
                            int32_t vocab, int64_t* out_ids, uint32_t flags, void* stream) {
  if (!h) return NLS_ERR_INVALID_ARG;
  if (flags & ~(NLS_DEVICE_INPUTS | NLS_DEVICE_OUTPUTS)) return NLS_ERR_INVALID_ARG;
  if (rows < 0 || vocab < 1 || ld < vocab) return NLS_ERR_INVALID_ARG;
  if (rows == 0) return NLS_OK;
  if (!logits || !out_ids) return NLS_ERR_INVALID_ARG;
  if (rows > h->max_rows || vocab > h->max_vocab) return NLS_ERR_CAPACITY;
  DeviceGuard g(h->device);
  cudaStream_t st = (cudaStream_t)stream;
  nls::BatchArgs a{};
  a.rows = rows;
  a.V = vocab;
  a.argmax_only = 1;
  if (flags & NLS_DEVICE_INPUTS) {
    a.logits = logits;
    a.ld = ld;
  } else {
    nls_status s;
    if ((s = grow(h, &h->d_logits, &h->logits_cap, (size_t)rows * vocab)) != NLS_OK) return s;
    NLS_CUDA(h, cudaMemcpy2DAsync(h->d_logits, (size_t)vocab * sizeof(float), logits,
                                  (size_t)ld * sizeof(float), (size_t)vocab * sizeof(float), rows,
                                  cudaMemcpyHostToDevice, st));
    a.logits = h->d_logits;
    a.ld = vocab;
  }
  const bool dev_out = (flags & NLS_DEVICE_OUTPUTS) != 0;
  a.out_ids = dev_out ? out_ids : h->d_out_ids;
  nls_status s = run_batch(h, a, flags, st);
  if (s != NLS_OK) return s;
  if (dev_out) return NLS_OK;
  NLS_CUDA(h, cudaMemcpyAsync(out_ids, h->d_out_ids, sizeof(int64_t) * rows, cudaMemcpyDeviceToHost, st));
  NLS_CUDA(h, cudaStreamSynchronize(st));
  return (nls_status)*h->h_status;
}

nls_status nls_top_tokens(nls_handle* h, const float* logits, int64_t ld, int32_t rows,
                          int32_t vocab, int32_t n, int64_t* out_ids, float* out_probs,
                          uint32_t flags, void* stream) {
  if (!h) return NLS_ERR_INVALID_ARG;
  if (flags & ~(NLS_DEVICE_INPUTS | NLS_DEVICE_OUTPUTS)) return NLS_ERR_INVALID_ARG;
  if (rows < 0 || vocab < 1 || ld < vocab || n < 1 || n > 256) return NLS_ERR_INVALID_ARG;
  if (rows == 0) return NLS_OK;
  if (!logits || !out_ids) return NLS_ERR_INVALID_ARG;
  if (rows > h->max_rows || vocab > h->max_vocab) return NLS_ERR_CAPACITY;
  DeviceGuard g(h->device);
  cudaStream_t st = (cudaStream_t)stream;
  nls_status s;
  const float* dl = logits;
  int64_t dld = ld;
  if (!(flags & NLS_DEVICE_INPUTS)) {
    if ((s = grow(h, &h->d_logits, &h->logits_cap, (size_t)rows * vocab)) != NLS_OK) return s;
    NLS_CUDA(h, cudaMemcpy2DAsync(h->d_logits, (size_t)vocab * sizeof(float), logits,
                                  (size_t)ld * sizeof(float), (size_t)vocab * sizeof(float), rows,
                                  cudaMemcpyHostToDevice, st));
    dl = h->d_logits;
    dld = vocab;
  }
  const bool dev_out = (flags & NLS_DEVICE_OUTPUTS) != 0;
  int64_t* oid = out_ids;
  float* opr = out_probs;
  if (!dev_out) {
    if ((s = grow(h, &h->d_sh_mine, &h->sh_mine_cap, (size_t)rows * n)) != NLS_OK) return s;
    if ((s = grow(h, &h->d_sh_pmine, &h->sh_pmine_cap, (size_t)rows * n)) != NLS_OK) return s;
    oid = h->d_sh_mine;
    opr = out_probs ? h->d_sh_pmine : nullptr;
  }
  NLS_CUDA(h, cudaMemsetAsync(h->d_work, 0, sizeof(int), st));
  NLS_CUDA(h, nls::launch_top(dl, dld, rows, vocab, n, oid, opr, h->d_work, h->d_scratch, h->vpad,
                              h->slots, st));
  if (dev_out) return NLS_OK;
  NLS_CUDA(h, cudaMemcpyAsync(h->h_status, h->d_work, sizeof(int), cudaMemcpyDeviceToHost, st));
  NLS_CUDA(h, cudaMemcpyAsync(out_ids, oid, sizeof(int64_t) * rows * n, cudaMemcpyDeviceToHost, st));
  if (out_probs)
    NLS_CUDA(h, cudaMemcpyAsync(out_probs, opr, sizeof(float) * rows * n, cudaMemcpyDeviceToHost, st));
  NLS_CUDA(h, cudaStreamSynchronize(st));
  return (nls_status)*h->h_status;
}

nls_status nls_token_nll(nls_handle* h, const float* logits, int64_t ld, int32_t rows,
                         int32_t vocab, const int64_t* targets, double* out_nll, uint32_t flags,
                         void* stream) {
  if (!h) return NLS_ERR_INVALID_ARG;
  if (flags & ~(NLS_DEVICE_INPUTS | NLS_DEVICE_OUTPUTS)) return NLS_ERR_INVALID_ARG;
  if (rows < 0 || vocab < 1 || ld < vocab) return NLS_ERR_INVALID_ARG;
  if (rows == 0) return NLS_OK;
  if (!logits || !targets || !out_nll) return NLS_ERR_INVALID_ARG;
  if (rows > h->max_rows || vocab > h->max_vocab) return NLS_ERR_CAPACITY;
  DeviceGuard g(h->device);
  cudaStream_t st = (cudaStream_t)stream;
  nls_status s;
  const float* dl = logits;
  int64_t dld = ld;
  const int64_t* dt = targets;
  if (!(flags & NLS_DEVICE_INPUTS)) {
    if ((s = grow(h, &h->d_logits, &h->logits_cap, (size_t)rows * vocab)) != NLS_OK) return s;
    if ((s = grow(h, &h->d_tgt, &h->tgt_cap, (size_t)rows)) != NLS_OK) return s;
    NLS_CUDA(h, cudaMemcpy2DAsync(h->d_logits, (size_t)vocab * sizeof(float), logits,
                                  (size_t)ld * sizeof(float), (size_t)vocab * sizeof(float), rows,
                                  cudaMemcpyHostToDevice, st));
    NLS_CUDA(h, cudaMemcpyAsync(h->d_tgt, targets, sizeof(int64_t) * rows, cudaMemcpyHostToDevice, st));
    dl = h->d_logits;
    dld = vocab;
    dt = h->d_tgt;
  }
  const bool dev_out = (flags & NLS_DEVICE_OUTPUTS) != 0;
  double* dout = out_nll;
  if (!dev_out) {
    if ((s = grow(h, &h->d_nll, &h->nll_cap, (size_t)rows)) != NLS_OK) return s;
    dout = h->d_nll;
  }
  NLS_CUDA(h, cudaMemsetAsync(h->d_work, 0, sizeof(int), st));
  NLS_CUDA(h, nls::launch_nll(dl, dld, rows, vocab, dt, dout, h->d_work, h->sm_count, st));
  if (dev_out) return NLS_OK;
  NLS_CUDA(h, cudaMemcpyAsync(h->h_status, h->d_work, sizeof(int), cudaMemcpyDeviceToHost, st));
  NLS_CUDA(h, cudaMemcpyAsync(out_nll, dout, sizeof(double) * rows, cudaMemcpyDeviceToHost, st));
  NLS_CUDA(h, cudaStreamSynchronize(st));
  return (nls_status)*h->h_status;
}

nls_status nls_set_profiling(nls_handle* h, int32_t on) {
  if (!h) return NLS_ERR_INVALID_ARG;
  DeviceGuard g(h->device);
  if (on && !h->ev[0]) {
    for (cudaEvent_t& e : h->ev) NLS_CUDA(h, cudaEventCreate(&e));
  }
  h->profiling = on ? 1 : 0;
  return NLS_OK;
}

nls_status nls_last_kernel_ms(nls_handle* h, float* out_ms, int32_t n) {
  if (!h || !out_ms || n < 1) return NLS_ERR_INVALID_ARG;
  if (!h->profiled) return NLS_ERR_INVALID_ARG;
  DeviceGuard g(h->device);
  NLS_CUDA(h, cudaEventSynchronize(h->ev[3]));
  NLS_CUDA(h, cudaEventSynchronize(h->ev[1]));
  for (int i = 0; i < n && i < 3; ++i) {
    float ms = 0.0f;
    NLS_CUDA(h, cudaEventElapsedTime(&ms, h->ev[0], h->ev[i + 1]));
    out_ms[i] = ms;
  }
  return NLS_OK;
}

nls_status nls_stream_status(nls_handle* h, void* stream) {
  if (!h) return NLS_ERR_INVALID_ARG;
  DeviceGuard g(h->device);
  NLS_CUDA(h, cudaStreamSynchronize((cudaStream_t)stream));
  int status = 0;
  NLS_CUDA(h, cudaMemcpy(&status, h->d_work, sizeof(int), cudaMemcpyDeviceToHost));
  return (nls_status)status;
}


}  // extern "C"

namespace {

unsigned long long now_ms() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (unsigned long long)ts.tv_sec * 1000ull + (unsigned long long)ts.tv_nsec / 1000000ull;
}

void pause_us(long us) {
  timespec ts{0, us * 1000L};
  nanosleep(&ts, nullptr);
}

// End the communicator at once (pending collectives on it end too).
void abort_comm(const nls::NcclApi& n, nls_comm* c) {
  if (c->comm && !c->aborted) {
    DeviceGuard g(c->device);
    n.CommAbort(c->comm);
  }
  c->aborted = true;
}

// Non-blocking communicator: wait until its state leaves ncclInProgress.
// An error aborts it (NLS_ERR_NCCL); so does the deadline (NLS_ERR_TIMEOUT).
nls_status comm_settle(const nls::NcclApi& n, nls_comm* c, unsigned long long deadline,
                       char* err, size_t errlen, const char* what) {
  for (;;) {
    ncclResult_t r = ncclSuccess;
    if (n.CommGetAsyncError(c->comm, &r) != ncclSuccess) r = ncclInternalError;
    if (r == ncclSuccess) return NLS_OK;
    if (r != ncclInProgress) {
      if (err) snprintf(err, errlen, "%s: %s", what, n.GetErrorString(r));
      abort_comm(n, c);
      return NLS_ERR_NCCL;
    }
    if (now_ms() > deadline) {
      if (err) snprintf(err, errlen, "%s: no progress within %llu ms", what, c->timeout_ms);
      abort_comm(n, c);
      return NLS_ERR_TIMEOUT;
    }
    pause_us(20);
  }
}

}  // namespace

extern "C" {

nls_status nls_comm_unique_id(uint8_t* out) {
  if (!out) return NLS_ERR_INVALID_ARG;
  const nls::NcclApi& n = nls::nccl_api();
  if (!n.ok) return NLS_ERR_NCCL;
  ncclUniqueId id;
  if (n.GetUniqueId(&id) != ncclSuccess) return NLS_ERR_NCCL;
  memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
  return NLS_OK;
}

nls_status nls_comm_create(nls_comm** out, const uint8_t* id, int32_t nranks, int32_t rank,
                           int32_t device) {
  if (!out) return NLS_ERR_INVALID_ARG;
  *out = nullptr;
  if (!id || nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks) return NLS_ERR_INVALID_ARG;
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) return NLS_ERR_NO_DEVICE;
  if (device < 0 || device >= ndev) return NLS_ERR_INVALID_ARG;
  const nls::NcclApi& n = nls::nccl_api();
  if (!n.ok) return NLS_ERR_NCCL;
  DeviceGuard g(device);
  ncclUniqueId uid;
  memcpy(uid.internal, id, NCCL_UNIQUE_ID_BYTES);
  nls_comm* c = new (std::nothrow) nls_comm();
  if (!c) return NLS_ERR_CAPACITY;
  c->nranks = nranks;
  c->rank = rank;
  c->device = device;
  // non-blocking: every call returns at once and the library polls the
  // communicator's state against a host deadline, so a rank that never
  // joins (or leaves) ends in NLS_ERR_TIMEOUT and ncclCommAbort, not a hang
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const ncclResult_t r = n.CommInitRankConfig(&c->comm, nranks, uid, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (c->comm) n.CommAbort(c->comm);
    delete c;
    return NLS_ERR_NCCL;
  }
  const nls_status st = comm_settle(n, c, now_ms() + c->timeout_ms, nullptr, 0, "ncclCommInitRankConfig");
  if (st != NLS_OK) {
    delete c;
    return st;
  }
  *out = c;
  return NLS_OK;
}

nls_status nls_comm_set_timeout(nls_comm* c, uint64_t ms) {
  if (!c || ms == 0) return NLS_ERR_INVALID_ARG;
  c->timeout_ms = ms;
  return NLS_OK;
}

nls_status nls_comm_abort(nls_comm* c) {
  if (!c) return NLS_ERR_INVALID_ARG;
  const nls::NcclApi& n = nls::nccl_api();
  if (!n.ok) return NLS_ERR_NCCL;
  abort_comm(n, c);
  return NLS_OK;
}

void nls_comm_destroy(nls_comm* c) {
  if (!c) return;
  const nls::NcclApi& n = nls::nccl_api();
  if (n.ok && c->comm && !c->aborted) {
    DeviceGuard g(c->device);
    // a non-blocking communicator may report ncclInProgress while it tears
    // down; wait for that within its deadline (abort if it runs out)
    const ncclResult_t r = n.CommDestroy(c->comm);
    if (r == ncclInProgress) {
      const unsigned long long deadline = now_ms() + c->timeout_ms;
      ncclResult_t a = ncclInProgress;
      while (n.CommGetAsyncError(c->comm, &a) == ncclSuccess && a == ncclInProgress && now_ms() <= deadline)
        pause_us(20);
    } else if (r != ncclSuccess) {
      n.CommAbort(c->comm);
    }
  }
  delete c;
}

nls_status nls_sample_batch_vocab_sharded(nls_handle* h, nls_comm* c, const float* logits,
                                          int64_t ld, int32_t rows, int32_t vocab,
                                          const nls_row_params* params, const int64_t* hist_ids,
                                          const int64_t* hist_off, const int64_t* bias_ids,
                                          const double* bias_vals, const int64_t* bias_off,
                                          const double* uniforms, int64_t* out_ids,
                                          float* out_probs, void* stream) {
  if (!h || !c) return NLS_ERR_INVALID_ARG;
  const int P = c->nranks, me = c->rank;
  if (rows < 0 || vocab < 1) return NLS_ERR_INVALID_ARG;
  const int Vs = (vocab + P - 1) / P;  // columns per rank (the last may have fewer)
  auto vq = [&](int q) { const int v = vocab - q * Vs; return v < 0 ? 0 : (v < Vs ? v : Vs); };
  if (vq(P - 1) < 1) return NLS_ERR_INVALID_ARG;  // every rank holds at least one column
  const int Vr = vq(me);
  if (ld < Vr) return NLS_ERR_INVALID_ARG;
  if (rows == 0) return NLS_OK;
  if (!logits || !params || !out_ids) return NLS_ERR_INVALID_ARG;
  if ((hist_ids == nullptr) != (hist_off == nullptr)) return NLS_ERR_INVALID_ARG;
  if ((bias_ids == nullptr) != (bias_off == nullptr) || (bias_ids == nullptr) != (bias_vals == nullptr))
    return NLS_ERR_INVALID_ARG;
  if (c->device != h->device) return NLS_ERR_INVALID_ARG;
  if (c->aborted) return NLS_ERR_NCCL;
  if (rows > h->max_rows || vocab > h->max_vocab) return NLS_ERR_CAPACITY;
  const nls::NcclApi& n = nls::nccl_api();
  if (!n.ok) return NLS_ERR_NCCL;
  const unsigned long long deadline = now_ms() + c->timeout_ms;
  DeviceGuard g(h->device);
  cudaStream_t st = (cudaStream_t)stream;
  auto r0 = [&](int q) { return (int)((int64_t)rows * q / P); };  // rank q owns rows [r0(q), r0(q+1))
  const int R0 = r0(me), Bown = r0(me + 1) - R0;
  const int Bmax = (rows + P - 1) / P;
  nls_status s;
  if ((s = grow(h, &h->d_logits, &h->logits_cap, (size_t)Bown * vocab)) != NLS_OK) return s;
  if ((s = grow(h, &h->d_sh_recv, &h->sh_recv_cap, (size_t)Bown * vocab)) != NLS_OK) return s;
  if ((s = grow(h, &h->d_sh_mine, &h->sh_mine_cap, (size_t)Bmax + 1)) != NLS_OK) return s;
  if ((s = grow(h, &h->d_sh_all, &h->sh_all_cap, (size_t)P * (Bmax + 1))) != NLS_OK) return s;
  if ((s = grow(h, &h->d_sh_pmine, &h->sh_pmine_cap, (size_t)Bmax)) != NLS_OK) return s;
  if ((s = grow(h, &h->d_sh_pall, &h->sh_pall_cap, (size_t)P * Bmax)) != NLS_OK) return s;
  if (!h->h_sh_status) NLS_CUDA(h, cudaMallocHost(&h->h_sh_status, sizeof(int64_t) * kMaxRanks));
  // 1. transpose: rank q receives every rank's columns of the rows it owns
  const float* src = logits;
  if (ld != Vr) {
    if ((s = grow(h, &h->d_sh_send, &h->sh_send_cap, (size_t)rows * Vr)) != NLS_OK) return s;
    NLS_CUDA(h, cudaMemcpy2DAsync(h->d_sh_send, (size_t)Vr * sizeof(float), logits,
                                  (size_t)ld * sizeof(float), (size_t)Vr * sizeof(float), rows,
                                  cudaMemcpyDeviceToDevice, st));
    src = h->d_sh_send;
  }
  // (a non-blocking communicator may answer ncclInProgress: the operation
  // is being enqueued; the communicator is settled before the next one)
  auto ncclok = [&](ncclResult_t r, const char* what) {
    if (r == ncclSuccess || r == ncclInProgress) return true;
    snprintf(h->last_err, sizeof h->last_err, "%s: %s", what, n.GetErrorString(r));
    abort_comm(n, c);
    return false;
  };
  auto settle = [&](const char* what) {
    return comm_settle(n, c, deadline, h->last_err, sizeof h->last_err, what);
  };
  if (!ncclok(n.GroupStart(), "ncclGroupStart")) return NLS_ERR_NCCL;
  bool ok = true;
  for (int q = 0; q < P && ok; ++q) {
    const int nq = r0(q + 1) - r0(q);
    if (nq > 0)
      ok = ncclok(n.Send(src + (size_t)r0(q) * Vr, (size_t)nq * Vr, ncclFloat, q, c->comm, st), "ncclSend");
    if (ok && Bown > 0)
      ok = ncclok(n.Recv(h->d_sh_recv + (size_t)Bown * q * Vs, (size_t)Bown * vq(q), ncclFloat, q,
                         c->comm, st), "ncclRecv");
  }
  if (!ncclok(n.GroupEnd(), "ncclGroupEnd") || !ok) return NLS_ERR_NCCL;
  if ((s = settle("ncclGroupEnd")) != NLS_OK) return s;
  // 2. assemble the owned rows and sample them like any batch
  if (Bown > 0) {
    for (int q = 0; q < P; ++q)
      NLS_CUDA(h, cudaMemcpy2DAsync(h->d_logits + (size_t)q * Vs, (size_t)vocab * sizeof(float),
                                    h->d_sh_recv + (size_t)Bown * q * Vs, (size_t)vq(q) * sizeof(float),
                                    (size_t)vq(q) * sizeof(float), Bown, cudaMemcpyDeviceToDevice, st));
    nls::BatchArgs a{};
    a.logits = h->d_logits;
    a.ld = vocab;
    a.rows = Bown;
    a.V = vocab;
    a.params = params + R0;
    a.hist_ids = hist_ids;
    a.hist_off = hist_off ? hist_off + R0 : nullptr;
    a.bias_ids = bias_ids;
    a.bias_vals = bias_vals;
    a.bias_off = bias_off ? bias_off + R0 : nullptr;
    a.uniforms = uniforms ? uniforms + R0 : nullptr;
    a.out_ids = h->d_sh_mine;
    a.out_probs = out_probs ? h->d_sh_pmine : nullptr;
    if ((s = run_batch(h, a, NLS_DEVICE_INPUTS | NLS_DEVICE_OUTPUTS, st)) != NLS_OK) return s;
  }
  // 3. every rank gets every row's result, and every rank's status
  NLS_CUDA(h, cudaMemsetAsync(h->d_sh_mine + Bmax, 0, sizeof(int64_t), st));
  if (Bown > 0) NLS_CUDA(h, cudaMemcpyAsync(h->d_sh_mine + Bmax, h->d_work, sizeof(int), cudaMemcpyDeviceToDevice, st));
  if (!ncclok(n.AllGather(h->d_sh_mine, h->d_sh_all, (size_t)Bmax + 1, ncclInt64, c->comm, st), "ncclAllGather"))
    return NLS_ERR_NCCL;
  if ((s = settle("ncclAllGather")) != NLS_OK) return s;
  if (out_probs &&
      !ncclok(n.AllGather(h->d_sh_pmine, h->d_sh_pall, (size_t)Bmax, ncclFloat, c->comm, st), "ncclAllGather"))
    return NLS_ERR_NCCL;
  if (out_probs && (s = settle("ncclAllGather")) != NLS_OK) return s;
  for (int q = 0; q < P; ++q) {
    const int nq = r0(q + 1) - r0(q);
    if (nq > 0) {
      NLS_CUDA(h, cudaMemcpyAsync(out_ids + r0(q), h->d_sh_all + (size_t)q * (Bmax + 1), sizeof(int64_t) * nq,
                                  cudaMemcpyDeviceToDevice, st));
      if (out_probs)
        NLS_CUDA(h, cudaMemcpyAsync(out_probs + r0(q), h->d_sh_pall + (size_t)q * Bmax, sizeof(float) * nq,
                                    cudaMemcpyDeviceToDevice, st));
    }
    NLS_CUDA(h, cudaMemcpyAsync(h->h_sh_status + q, h->d_sh_all + (size_t)q * (Bmax + 1) + Bmax,
                                sizeof(int64_t), cudaMemcpyDeviceToHost, st));
  }
  // wait for the stream against the deadline: a rank that does not take part
  // (gone, or stuck before this call) leaves the collectives waiting, and the
  // library then aborts the communicator instead of waiting for good
  for (;;) {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) return cuda_fail(h, q, "cudaStreamQuery");
    ncclResult_t ae = ncclSuccess;
    if (n.CommGetAsyncError(c->comm, &ae) != ncclSuccess || (ae != ncclSuccess && ae != ncclInProgress)) {
      snprintf(h->last_err, sizeof h->last_err, "NCCL: %s", n.GetErrorString(ae));
      abort_comm(n, c);
      return NLS_ERR_NCCL;
    }
    if (now_ms() > deadline) {
      snprintf(h->last_err, sizeof h->last_err, "vocab-sharded call: the collectives did not finish "
               "within %llu ms; communicator aborted", c->timeout_ms);
      abort_comm(n, c);
      // the aborted collectives end; let the stream drain (bounded)
      const unsigned long long drain = now_ms() + 10000ull;
      while (cudaStreamQuery(st) == cudaErrorNotReady && now_ms() <= drain) pause_us(100);
      return NLS_ERR_TIMEOUT;
    }
    pause_us(20);
  }
  for (int q = 0; q < P; ++q)
    if (h->h_sh_status[q] != 0) return (nls_status)h->h_sh_status[q];
  return NLS_OK;
}

}  // extern "C"
