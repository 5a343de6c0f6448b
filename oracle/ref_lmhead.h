/* oracle/ref_lmhead.h -- CPU restatement of nimllm's output projection
 * (TEST INFRASTRUCTURE; see ref_lmhead.c). */
#ifndef NLO_REF_LMHEAD_H
#define NLO_REF_LMHEAD_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type codes (quant.nim:14-19) of the weight formats restated here */
enum { NLO_F32 = 0, NLO_F16 = 1, NLO_Q4_0 = 2, NLO_Q8_0 = 8, NLO_Q6_K = 14 };

/* rowBytes (quant.nim:65-71): bytes of one weight row of `cols` values;
 * -1 for an unsupported type or a length that is not a whole number of blocks. */
int64_t nlo_row_bytes(int32_t wtype, int64_t cols);

/* quantizeAct (quant.nim:646-662) without the 16-value sums (only the K
 * types with mins use them): n floats in blocks of block_len -> per-block
 * scales d[n / block_len] and int8 values qs[n]. */
void nlo_quantize_act(const float* x, int64_t n, int64_t block_len, float* d, int8_t* qs);

/* matmul (model.nim:179-189) with its row task (model.nim:144-169), no LoRA:
 * y[b*rows + r] = row r of w (ggml layout, rows x nlo_row_bytes) . x[b*cols ..].
 * exact_matmul mirrors the module variable `exactMatmul` (model.nim:173).
 * Rows are split over `threads` POSIX threads (order within a row is the
 * reference's). Returns 0, or -1 for an unsupported type or shape. */
int nlo_lm_head(const uint8_t* w, int32_t wtype, int64_t rows, int64_t cols, const float* x,
                int64_t nb, float* y, int32_t exact_matmul, int32_t threads);

#ifdef __cplusplus
}
#endif
#endif
