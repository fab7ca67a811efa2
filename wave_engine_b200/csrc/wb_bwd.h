// wb_bwd.h -- attention backward (src/common/attn.rs:346-430) on the GPU.
#pragma once
#include "wave_b200.h"
#include "wb_internal.h"

namespace wb {

// Device weights the backward reads (the layer's own copies).
struct BwdLayer {
    int E, H, hd, C;
    const float *w_out;  // [E][E] out_proj rows ([out][in])
    const float *hn;     // [H] softplus(harmonic_raw)
    const float *raw;    // [H] harmonic_raw
    const float *wrs_t;  // [E][H][2]
    const float *wv_t;   // [H][hd(in)][hd(out)]
    const float *wc_t;   // [E][H*C] or nullptr
};

// The forward cache on the device, WaveAttnCache (attn.rs:51-70) per
// sequence stacked over the batch.
struct BwdCache {
    const float *phases;     // [B][H][T]
    const float *phase_rs;   // [B][H][T][2]
    const float *v_all;      // [B][H][T][hd]
    const float *content;    // [B][H][T][C] or nullptr
    const float *att_w;      // [B][H][T][T]
    const float *out_merged; // [B][T][E]
};

// Gradient outputs on the device (any may be nullptr: not computed).
struct BwdGrads {
    float *harmonic_raw, *phase_proj_w, *phase_proj_b, *v_proj_w, *v_proj_b, *content_proj_w, *content_proj_b,
        *out_proj_w, *out_proj_b;
};

size_t attn_backward_scratch_bytes(int B, int H, int T, int hd, int C, int E);
// d_x [B][T][E] and the weight gradients summed over the batch.
int attn_backward(const BwdLayer &w, const BwdCache &cache, const float *x, const float *d_y, int B, int T,
                  float *d_x, const BwdGrads &g, void *scratch, cudaStream_t st, std::string *msg);

// [B][T][H][K] -> [B][H][T][K] (the cache's per-head layouts).
void launch_rows_to_heads(const float *src, int B, int T, int H, int K, float *dst, cudaStream_t st);

}  // namespace wb
