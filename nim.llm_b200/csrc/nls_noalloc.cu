// nls_noalloc.cu -- nls_sample_batch_noalloc: sampling without allocating.
//
// Some callers cannot call cudaMalloc: a serving process that has given
// nearly all of the GPU's memory to its own pool (an allocation would fail),
// a host whose memory policy forbids allocating after start-up, or a
// latency-critical decode loop that cannot afford the device-wide
// synchronisation cudaMalloc/cudaFree imply. The handle-based entry points
// allocate their staging and scratch in nls_create, so those callers get this
// entry instead. It takes device pointers for every input and output, as the
// handle path does with NLS_DEVICE_INPUTS | NLS_DEVICE_OUTPUTS, and runs the
// same two kernels. The full-sort kernel's scratch and the work counters live
// in one file-scope device array, g_noalloc_scratch, of fixed size: every GPU
// that loads the library holds it (about 16 MiB) until the process exits.
//
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress while that device is current, and caches it for the
// life of the process: make that first call before any stream capture, and
// do not use the entry point after cudaDeviceReset (the module is reloaded
// and the cached address goes stale). All calls share the one array and it
// keeps the last call's contents; the status word and the counters are
// cleared at the start of every call. Calls whose work overlaps on the GPU
// (different streams, or different host threads on one device) race on the
// array. nls_noalloc_status reads the status word the last call's kernels
// left (a NaN row of a full sort, a timeout, a bad history offset).
#include <mutex>

#include "nimllm_sample.h"
#include "nls_kernels.h"

namespace {

constexpr int kNoallocMaxRows = 4096;                 // rows per call
constexpr int kNoallocSlots = 4;                      // full-sort CTAs (scratch slots)
constexpr int kNoallocVpad = nls::kMaxVocab;          // words per slot array (vocab limit)
constexpr int kWorkWords = ((2 + kNoallocMaxRows) + 63) / 64 * 64;  // status, count, list
constexpr size_t kScratchWords =
    (size_t)kWorkWords + (size_t)kNoallocSlots * 4 * (size_t)kNoallocVpad;

static __device__ __align__(256) uint32_t g_noalloc_scratch[kScratchWords];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint32_t* g_base[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (cached).
cudaError_t scratch_base(int dev, uint32_t** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_base[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_base[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_base[dev];
  return cudaSuccess;
}

// CTAs per row of the streaming kernel: the handle path's choice (split rows
// only when SMs are left, at least 2048 logits per CTA), within the portable
// cluster size.
int noalloc_cluster(int rows, int vocab, int sm_count) {
  int C = 1;
  if (vocab >= 8192) C = (sm_count + rows - 1) / rows;
  if (C > vocab / 2048) C = vocab / 2048;
  if (C > 8) C = 8;
  if (C < 1) C = 1;
  return C;
}

}  // namespace

extern "C" nls_status nls_sample_batch_noalloc(
    const float* logits, int64_t ld, int32_t rows, int32_t vocab, const nls_row_params* params,
    const int64_t* hist_ids, const int64_t* hist_off, const int64_t* bias_ids,
    const double* bias_vals, const int64_t* bias_off, const double* uniforms, int64_t* out_ids,
    float* out_probs, void* stream) {
  if (rows < 0 || vocab < 1 || ld < vocab) return NLS_ERR_INVALID_ARG;
  if (rows == 0) return NLS_OK;
  if (!logits || !params || !out_ids) return NLS_ERR_INVALID_ARG;
  if ((hist_ids == nullptr) != (hist_off == nullptr)) return NLS_ERR_INVALID_ARG;
  if ((bias_ids == nullptr) != (bias_off == nullptr) || (bias_ids == nullptr) != (bias_vals == nullptr))
    return NLS_ERR_INVALID_ARG;
  if (rows > kNoallocMaxRows || vocab > kNoallocVpad) return NLS_ERR_CAPACITY;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NLS_ERR_NO_DEVICE;
  if (dev < 0 || dev >= kMaxDevices) return NLS_ERR_CAPACITY;
  uint32_t* base = nullptr;
  if (scratch_base(dev, &base) != cudaSuccess) return NLS_ERR_CUDA;
  int sm_count = 0;
  if (cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return NLS_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;

  nls::BatchArgs a{};
  a.logits = logits;
  a.ld = ld;
  a.rows = rows;
  a.V = vocab;
  a.params = params;
  a.hist_ids = hist_ids;
  a.hist_off = hist_off;
  a.bias_ids = bias_ids;
  a.bias_vals = bias_vals;
  a.bias_off = bias_off;
  a.uniforms = uniforms;
  a.out_ids = out_ids;
  a.out_probs = out_probs;
  int* work = reinterpret_cast<int*>(base);
  a.status = work;
  a.full_count = work + 1;
  a.full_list = work + 2;
  a.argmax_only = 0;
  a.wait_ns = 200ull * 1000ull * 1000ull;  // the library's default wait limit
  uint32_t* scratch = base + kWorkWords;

  if (cudaMemsetAsync(work, 0, 2 * sizeof(int), st) != cudaSuccess) return NLS_ERR_CUDA;
  const int C = noalloc_cluster(rows, vocab, sm_count);
  int chunk = (vocab + C - 1) / C;
  chunk = (chunk + 3) & ~3;
  if (nls::launch_light(a, C, chunk, st) != cudaSuccess) return NLS_ERR_CUDA;
  if (nls::launch_full(a, scratch, kNoallocVpad, kNoallocSlots, st) != cudaSuccess) return NLS_ERR_CUDA;
  return NLS_OK;
}

extern "C" nls_status nls_noalloc_status(int32_t* out, uint32_t flags, void* stream) {
  if (!out) return NLS_ERR_INVALID_ARG;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NLS_ERR_NO_DEVICE;
  if (dev < 0 || dev >= kMaxDevices) return NLS_ERR_CAPACITY;
  uint32_t* base = nullptr;
  if (scratch_base(dev, &base) != cudaSuccess) return NLS_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;
  if (flags & NLS_DEVICE_OUTPUTS) {
    if (cudaMemcpyAsync(out, base, sizeof(int32_t), cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return NLS_ERR_CUDA;
    return NLS_OK;
  }
  if (cudaMemcpyAsync(out, base, sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return NLS_ERR_CUDA;
  return NLS_OK;
}
