// wb_serve.h -- kernels of the serve-tier layer around the attention
// (wb_serve.cu): LayerNorm, maestro, AGC, Kerr ODE, FFN out_proj, residual,
// embedding and the decoders.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wb {

// agc.rs OdeAgc, device resident (the reference's process-wide instance,
// ffn.rs:76, made explicit): updated by every FFN call it is passed to.
struct AgcDev {
    float ema_mean, ema_var, headroom, decay, min_threshold, max_threshold, threshold;
    int count;  // observations so far (the first 9 replace the EMA)
};

struct MaestroArgs {
    const float *x;       // [rows][E] input
    const float *base;    // [rows][E] residual base (nullptr: x)
    const float *sq_w, *sq_b, *pr_wt, *pr_b;  // squeeze [M][E] + [M], process_1 transposed [M][E] + [E]
    long long rows;
    int E, M;
    float *y;             // [rows][E] = base + process_1 . gelu(squeeze . x)
};

struct OdeArgs {
    const float *pre;         // [rows][2 n_bands] precond (before the AGC compression)
    const float *thresholds;  // AGC threshold per segment of rows_per_seg rows
    long long rows_per_seg;
    const float *gamma_raw, *omega, *rk4_w, *corrector;  // corrector nullptr: no corrector plate
    float alpha, beta;
    int n_bands, steps, fft_len;  // fft_len 0: plain stencil; else circular over fft_len points
    float *out;               // [rows][2 n_bands]
};

int launch_layer_norm(const float *x, int rows, int n, const float *w, const float *b, float *y, cudaStream_t st);
int launch_maestro(const MaestroArgs &a, cudaStream_t st);
// AGC observations of n_seg consecutive segments of seg_mags band
// magnitudes each, in order; *thresholds (inside scratch) receives each
// segment's threshold.  scratch: agc_scratch_floats(n_seg, seg_mags) floats.
size_t agc_scratch_floats(int n_seg, long long seg_mags);
int launch_agc_observe(const float *pre, int n_seg, long long seg_mags, AgcDev *agc, float *scratch,
                       float **thresholds, cudaStream_t st);
int launch_kerr_ode(const OdeArgs &a, long long rows, cudaStream_t st);
int launch_out_proj_exact(const float *x, long long rows, int E, int groups, const float *w, const float *b, float *y,
                          cudaStream_t st);
int launch_residual(float *h, const float *a, const float *b, long long n, cudaStream_t st);
int launch_embed(const int32_t *tok, const int32_t *widx, int rows, int E, const float *wte, int vocab,
                 const float *wpe, int n_pos, float *out, uint32_t *dev_err, cudaStream_t st);
int launch_rotate_bands(const float *x, long long rows, int n_bands, const float *corr, float *y, cudaStream_t st);
int launch_vocab_dot(const float *x, int rows, int E, const float *w, int vocab, float *logits, cudaStream_t st);

}  // namespace wb
