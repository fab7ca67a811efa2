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

/* The dot-product attention core alone (compute.rs:357-414, between c_attn
 * and c_proj): qkv [B*T][3*n_embd] -> o [B*T][n_embd], DEVICE pointers.
 * mode 0: the tensor-core core (head_dim <= 128) with its fp32 fallback for
 * query tiles past the fixed-shift bound; 1: the same with every tile sent
 * to the fallback; 2: the fp32 FMA core.  Asynchronous on the context's
 * stream. */
WB_API int wb_test_dot_core(wb_context *ctx, const float *qkv, int batch, int seq_len, int n_embd, int n_head,
                            int mode, float *o);

#ifdef __cplusplus
}
#endif
#endif /* WAVE_B200_TESTING_H */
