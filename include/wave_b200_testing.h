/*
 * wave_b200_testing.h -- test hooks of libwave_b200.so.
 *
 * These expose internal kernels for unit tests.  They have no counterpart in
 * the reference and are not part of the drop-in boundary (wave_b200.h).
 */
#ifndef WAVE_B200_TESTING_H
#define WAVE_B200_TESTING_H

#include "wave_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* C[m][n] = sum_k A[m][k] * B[n][k] + bias[n] on the tcgen05 bf16 GEMM used
 * for out_proj.  A [M][K] and B [N][K] are bf16 (uint16 storage), C [M][N]
 * and bias [N] fp32; all DEVICE pointers; K a multiple of 8.  Asynchronous
 * on the context's stream. */
WB_API int wb_test_gemm_bf16(wb_context *ctx, const uint16_t *A, const uint16_t *B, const float *bias,
                             float *C, int M, int N, int K);

/* Same with fp32 A, B on the kind::tf32 path (wide layers' out_proj);
 * K a multiple of 4. */
WB_API int wb_test_gemm_tf32(wb_context *ctx, const float *A, const float *B, const float *bias, float *C, int M,
                             int N, int K);

#ifdef __cplusplus
}
#endif
#endif /* WAVE_B200_TESTING_H */
