// nls_check.cu -- the device exponential evaluated over ranges of float bit
// patterns, so that a test can hold it against the host C library's expf
// (the function Nim's exp(float32) calls in the reference, sampler.nim:56).
//
// ref_expf (nls_common.cuh) is the value every sampling kernel uses for a
// softmax term that reaches an output; texp_estimate is the cheaper estimate
// the full-sort kernel uses only to decide grid units, under the bracket
// kBracketRel. Both are written out here for n consecutive bit patterns.
#include "nls_common.cuh"
#include "nimllm_sample.h"

namespace {

__global__ void expf_range_kernel(uint32_t first, long long n, float* out, float* est) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float x = __uint_as_float(first + (uint32_t)i);
    out[i] = nls::ref_expf(x);
    if (est) est[i] = nls::texp_estimate(x);
  }
}

}  // namespace

extern "C" nls_status nls_ref_expf_range(uint32_t first_bits, int64_t n, float* out,
                                         float* out_estimate, void* stream) {
  if (n < 0 || (n > 0 && !out) || (uint64_t)first_bits + (uint64_t)n > 0x100000000ull)
    return NLS_ERR_INVALID_ARG;
  if (n == 0) return NLS_OK;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NLS_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return NLS_ERR_CUDA;
  const long long blocks_needed = (n + 255) / 256;
  const int blocks = (int)(blocks_needed < (long long)sms * 8 ? blocks_needed : (long long)sms * 8);
  expf_range_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(first_bits, (long long)n, out, out_estimate);
  return cudaGetLastError() == cudaSuccess ? NLS_OK : NLS_ERR_CUDA;
}
