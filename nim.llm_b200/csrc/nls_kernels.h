// nls_kernels.h -- host-side launchers of the sampler kernels.
#pragma once

#include <cstddef>
#include <cuda_runtime.h>

#include "nls_common.cuh"

namespace nls {

// Streaming kernel (greedy rows and top-k rows with k <= kLightKMax): one
// cluster of C CTAs per row, CTA c owning positions [c*chunk, (c+1)*chunk).
size_t light_smem_bytes(int C, int chunk);
cudaError_t launch_light(const BatchArgs& a, int C, int chunk, cudaStream_t stream);
// the largest cluster (CTAs per row) the device schedules for this vocab:
// 16 where a GPC has room for it, else 8 (checked once per device)
int light_max_cluster(int V);

// Full-sort kernel over the rows listed in a.full_list (count in a.full_count):
// `slots` persistent CTAs, each with 4*vpad words of `scratch`.
size_t full_smem_bytes(int V);
// after_light: launched right behind the streaming kernel on the same
// stream as its programmatic dependent (it waits for that grid in-kernel).
cudaError_t launch_full(const BatchArgs& a, uint32_t* scratch, int vpad, int slots,
                        cudaStream_t stream, bool after_light = false);

// The rows whose parameters select the full path, ascending, into
// list[0 .. *count): what a row-claiming full-sort launch claims from.
cudaError_t launch_classify(const BatchArgs& a, int* list, int* count, cudaStream_t stream);

// topTokens: one CTA per row (up to `slots`), scratch slots as launch_full.
size_t top_smem_bytes();
cudaError_t launch_top(const float* logits, int64_t ld, int rows, int V, int n, int64_t* out_ids,
                       float* out_probs, int* status, uint32_t* scratch, int vpad, int slots,
                       cudaStream_t stream);

// perplexity's per-position negative log-likelihood: out[r] for row r and
// target token targets[r] (grid-stride over rows, up to 4 CTAs per SM).
cudaError_t launch_nll(const float* logits, int64_t ld, int rows, int V, const int64_t* targets,
                       double* out, int* status, int sm_count, cudaStream_t stream);

// Output projection (matmul(m.output, x, y, nb), model.nim:179-189): y[b*rows + r]
// for ggml-layout weights w (rows x row bytes, 16-byte aligned, device) and
// activations x [nb x cols] (device). wtype: 0 F32, 1 F16, 2 Q4_0, 8 Q8_0,
// 14 Q6_K. The int8 path quantises x in each CTA (no scratch).
int lm_head_row_bytes(int wtype, int64_t cols, int64_t* out);
bool lm_head_int8_path(int wtype, int cols, int nb, bool exact);
// path_nb: the batch size the path choice sees (nb, or 1 for independent rows)
cudaError_t launch_lm_head(const uint8_t* w, int wtype, int rows, int cols, const float* x, int nb,
                           int path_nb, float* y, bool exact, int* status, int sm_count,
                           unsigned long long wait_ns, uint8_t* act_scratch, cudaStream_t st);
// Q6_K / Q8_0 / Q4_0 on the int8 path at lm_head_mma_min_rows or more batch rows:
// tcgen05 int8 MMAs (nls_lmhead_mma.cu), launches of up to 16 batch rows (with
// act_scratch: lm_head_act_scratch_bytes, else the CUDA-core path);
// y[b * ldy + r]
bool lm_head_mma_path(int wtype, int cols, int nb);
int lm_head_mma_min_rows(int wtype);
// the float path (dequantRow + dotF32) for F16 / Q8_0 / Q4_0 weights whose
// rows and 256-value chunks are 16-byte multiples (nls_lmhead_float.cu);
// x 16-byte aligned; launches of up to 16 batch rows
bool lm_head_float_tiled(int wtype, int cols, int64_t row_bytes);
cudaError_t launch_lm_head_float(const uint8_t* w, int wtype, int64_t row_bytes, int rows, int cols,
                                 const float* x, int nb, float* y, int64_t ldy, int sm_count,
                                 cudaStream_t st);
size_t lm_head_mma_smem(int wtype, int cols);
// device scratch of the tensor-core path: the quantized activations of one
// launch (16-byte aligned)
size_t lm_head_act_scratch_bytes(int cols);
cudaError_t launch_lm_head_mma(const uint8_t* w, int wtype, int64_t row_bytes, int rows, int cols, const float* x,
                               int nb, float* y, int64_t ldy, int* status, int sm_count,
                               unsigned long long wait_ns, uint8_t* act_scratch, cudaStream_t st);
}  // namespace nls
