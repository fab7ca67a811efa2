// wb_proj.h -- tensor-core (3xTF32) projections of the tensor path.
#pragma once
#include "wave_b200.h"
#include "wb_internal.h"

namespace wb {

struct ProjTcWeights {
    int E = 0, H = 0, hd = 0, C = 0;
    int n_v = 0, n_c = 0, n_rs = 0, N = 0;  // value / content / phase column counts
    float *w_hi = nullptr;                  // [N][E] tf32 heads of the weights
    float *w_lo = nullptr;                  // [N][E] fp32 remainders
    float *bias = nullptr;                  // [N]
};

int proj_weights_upload(ProjTcWeights *p, const wb_attn_weights_desc *w, std::string *msg);
void proj_weights_free(ProjTcWeights *p);

// Values into sv.v, phases + buckets into sv.theta / sv.bucket, content
// vectors into content [R][H*C] (skipped when content is null) for the
// R = B*T rows of x [R][E], for heads h0 .. h0 + Hg - 1 (all heads: 0, H).
// wrs_t/brs: phase weights [E][H][2] and biases; wv_t/bv: value weights
// [H][hd(in)][hd(out)] and biases (head_dim <= 64: values and phases in one
// fp32 SIMT pass, the GEMM only for content).
int launch_proj_tc(const ProjTcWeights &p, const float *wrs_t, const float *brs, const float *wv_t, const float *bv,
                   const float *x, int B, int T, const WbSeqView &sv, float *content, int h0, int Hg,
                   uint32_t *dev_err, cudaStream_t st, std::string *msg);

}  // namespace wb
