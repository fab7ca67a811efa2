// wb_tc.h -- tensor-core (tcgen05) path: device weight layouts and the
// prefill / decode sequences of WB_PATH_TENSOR.
#pragma once
#include "wave_b200.h"
#include "wb_internal.h"
#include "wb_proj.h"

#include <string>

namespace wb {

struct TcLayerWeights {
    int E = 0, H = 0, hd = 0, C = 0;
    ProjWeights pw{};                  // fp32 projection weights (shared with the SIMT path)
    ProjTcWeights proj;                // 3xTF32 tensor-core projection weights
    const float *harmonic_n = nullptr; // [H] softplus(harmonic_raw)
    const float *b_o = nullptr;        // [E] out_proj bias
    const float *wo_t = nullptr;       // [E][E] out_proj, input-major fp32 (decode rows)
    const float *wrs_h = nullptr;      // [H][E][2] phase projection, one head's weights contiguous (decode)
    float *w_o32 = nullptr;            // [E][E] out_proj rows, fp32 (tf32 B operand)
};

int tc_layer_upload(TcLayerWeights *t, const wb_attn_weights_desc *w, std::string *msg);
void tc_layer_free(TcLayerWeights *t);

// Prefill forward of heads h0 .. h1 - 1 (h1 < 0: all heads); with a head
// range y is that range's share of the output, o_range W_o[:, range]^T,
// plus the bias when add_bias.
int tc_attn_forward(const TcLayerWeights &t, const float *x, int B, int T, bool use_content, float *y,
                    float *phases_out, Workspace *ws, uint32_t *dev_err, int sm_count, cudaStream_t st,
                    std::string *msg, int h0 = 0, int h1 = -1, bool add_bias = true);
int tc_kv_prefill(const TcLayerWeights &t, const WbSeqView &sv, const float *x, int n_seq, int T, float *y,
                  Workspace *ws, uint32_t *dev_err, int sm_count, cudaStream_t st, std::string *msg);
int tc_gemm_bf16(const __nv_bfloat16 *A, const __nv_bfloat16 *B, const float *bias, float *C, int M, int N, int K,
                 uint32_t *dev_err, cudaStream_t st, std::string *msg);
int tc_gemm_tf32(const float *A, const float *B, const float *bias, float *C, int M, int N, int K, uint32_t *dev_err,
                 cudaStream_t st, std::string *msg);

// bf16 split of fp32 data (hi = bf16(x), lo = bf16(x - hi)) and the product
// C = A W^T (+ bias) from the three terms A_hi W_hi + A_lo W_hi + A_hi W_lo on
// the tcgen05 bf16 GEMM (~16 mantissa bits: the tensor path of the serve
// layer's FFN out_proj and vocabulary products).  K a multiple of 8.
int split_bf16(const float *x, long long n, __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t st);
int tc_gemm_bf16x3(const __nv_bfloat16 *A_hi, const __nv_bfloat16 *A_lo, const __nv_bfloat16 *W_hi,
                   const __nv_bfloat16 *W_lo, const float *bias, float *C, int M, int N, int K, uint32_t *dev_err,
                   cudaStream_t st, std::string *msg);
// Decode step for n_seq sequences of one layer: attention over the cache
// with the new position appended, then out_proj and the length update;
// scratch (the cache's, fixed size, tickets zero) holds the attention
// kernel's partials.
// chain: the attention grid may launch as a programmatic dependent of the
// kernel before it (allowed unless that kernel is the decode out_proj of
// the same cache layer); *ends_with_out: the step's last kernel is the SIMT
// decode out_proj (fewer than 64 rows), which lets such a dependent launch.
int tc_kv_decode(const TcLayerWeights &t, const WbSeqView &sv, int32_t *len, int cap, int n_slots, const float *x,
                 int n_seq, float *y, void *scratch, size_t scratch_bytes, uint32_t *dev_err, int sm_count,
                 cudaStream_t st, std::string *msg, bool chain = false, bool *ends_with_out = nullptr);

// Dot-product attention core (compute.rs:357-414) on the tcgen05 attention
// kernel: qkv [B*T][3E] (device) -> o [B*T][E], head_dim <= 128 (WB_ENOTSUP
// above; features and values padded to 64 or 128 columns).  ws:
// tc_dot_core_bytes(B, T, E, H) bytes of device scratch.  Query tiles whose
// scores could overflow the fixed shift are recomputed by the fp32 core;
// force_fallback (testing) sends every tile there.
size_t tc_dot_core_bytes(int B, int T, int E, int H);
int tc_dot_attention(const float *qkv, int B, int T, int E, int H, float *o, void *ws, int force_fallback,
                     uint32_t *dev_err, int sm_count, cudaStream_t st, std::string *msg);

// Row counts below this have tc_kv_decode write y with plain stores of its
// SIMT out_proj kernel (no tensor map), so y may then be the device alias of
// pinned host memory.
int tc_decode_plain_store_rows();

}  // namespace wb
