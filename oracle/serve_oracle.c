/*
 * serve_oracle.c -- CPU restatement of the serve-tier layer around the
 * attention (src/common/kv_cache.rs:93-236 prefill, :241-381 forward_one):
 * token embedding, LayerNorm, the dual-maestro Kerr-ODE FFN as those
 * functions run it (src/common/ffn.rs:39-230 with freeze_ode, no memory and
 * the stencil ODE of src/common/fft_ode.rs:171-250), the parallel residual,
 * the final LayerNorm and phase_native_decode / lm_head.  Test
 * infrastructure only (the parity checker of the GPU serve-layer kernels);
 * nothing in the product path links or calls this file.
 *
 * PARITY STATUS: parity unpinned, like the attention oracle (the Rust
 * reference cannot be built here).  One restatement choice: for n_bands >=
 * 256 the reference forms the ODE's neighbour sums by an FFT convolution
 * (rustfft, fft_ode.rs:60-120) over fft_len = next_power_of_two(n_bands)
 * zero-padded points; this file sums the same four neighbours directly with
 * the same circular indexing (a neighbour j contributes when j mod fft_len
 * < n_bands), so it differs from the reference by the FFT's rounding only.
 *
 * fp32 throughout, products rounded before the add (-ffp-contract=off),
 * sums in the reference's sequential order, glibc sqrtf/tanhf/sinf/cosf.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

float wo_softplus(float x);

/* src/common/model.rs:154-165 layer_norm. */
void wo_layer_norm(const float *x, int n, const float *w, const float *b, float *y) {
    float sum = 0.0f;
    for (int i = 0; i < n; i++) sum += x[i];
    const float mean = sum / (float)n;
    float var = 0.0f;
    for (int i = 0; i < n; i++) {
        const float d = x[i] - mean;
        var += d * d;
    }
    var = var / (float)n;
    const float sd = sqrtf(var + 1e-5f);
    for (int i = 0; i < n; i++) y[i] = (x[i] - mean) / sd * w[i] + b[i];
}

/* compute.rs:113-119 gelu_batch (tanh approximation, c = 0.7978845608). */
static float gelu(float v) {
    const float c = 0.7978845608f;
    const float inner = c * (v + 0.044715f * v * v * v);
    return 0.5f * v * (1.0f + tanhf(inner));
}

/* compute.rs:441-452 linear_batch_cpu: y[i] = b[i] + sum_j w[i][j] x[j]. */
static void linear(const float *w, const float *b, int n_out, int n_in, const float *x, float *y) {
    for (int i = 0; i < n_out; i++) {
        float s = 0.0f;
        const float *row = w + (size_t)i * n_in;
        for (int j = 0; j < n_in; j++) s += row[j] * x[j];
        y[i] = b[i] + s;
    }
}

/* src/common/agc.rs OdeAgc: the adaptive knee compression ahead of the ODE.
 * The reference keeps one process-wide instance (ffn.rs:76) that every FFN
 * call of every layer updates; here the state is explicit. */
typedef struct {
    float ema_mean, ema_var, headroom, decay, min_threshold, max_threshold, threshold;
    int64_t count;
} wo_agc;

/* agc.rs OdeAgc::new() = from_coupling(0.1, 0.1) -> with_ceiling. */
void wo_agc_init(wo_agc *a, float alpha, float beta) {
    float ceiling = sqrtf(1.57079637050628662109f / (alpha + 4.0f * beta));
    ceiling = fmaxf(ceiling, 0.5f);
    a->ema_mean = 1.0f;
    a->ema_var = 0.5f;
    a->headroom = 3.0f;
    a->decay = 0.995f;
    a->min_threshold = fmaxf(ceiling * 0.3f, 0.5f);
    a->max_threshold = ceiling;
    a->threshold = fmaxf(ceiling * 0.75f, 0.5f);
    a->count = 0;
}

/* agc.rs:134-165 observe. */
static void agc_observe(wo_agc *a, const float *mags, size_t n) {
    if (n == 0) return;
    const float ceiling_2x = a->max_threshold * 2.0f;
    size_t nc = 0;
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++)
        if (isfinite(mags[i]) && mags[i] < ceiling_2x) {
            sum += mags[i];
            nc++;
        }
    if (nc == 0) return;
    const float cn = (float)nc;
    const float mean = sum / cn;
    float var = 0.0f;
    for (size_t i = 0; i < n; i++)
        if (isfinite(mags[i]) && mags[i] < ceiling_2x) {
            const float d = mags[i] - mean;
            var += d * d;
        }
    var = var / cn;
    if (!isfinite(mean) || !isfinite(var)) return;
    a->count += 1;
    if (a->count < 10) {
        a->ema_mean = mean;
        a->ema_var = var;
    } else {
        a->ema_mean = a->decay * a->ema_mean + (1.0f - a->decay) * mean;
        a->ema_var = a->decay * a->ema_var + (1.0f - a->decay) * var;
    }
    const float sd = fmaxf(sqrtf(a->ema_var), 0.01f);
    a->threshold = fminf(fmaxf(a->ema_mean + a->headroom * sd, a->min_threshold), a->max_threshold);
}

/* agc.rs:174-213 process over t positions of n_embd = 2 * n_bands. */
static void agc_process(wo_agc *a, float *pre, int t, int n_bands) {
    const int E = 2 * n_bands;
    float *mags = (float *)malloc(sizeof(float) * (size_t)t * n_bands + 1);
    for (int p = 0; p < t; p++)
        for (int k = 0; k < n_bands; k++) {
            const float r = pre[(size_t)p * E + 2 * k], s = pre[(size_t)p * E + 2 * k + 1];
            mags[(size_t)p * n_bands + k] = sqrtf(r * r + s * s);
        }
    agc_observe(a, mags, (size_t)t * n_bands);
    free(mags);
    const float thr = a->threshold;
    for (int p = 0; p < t; p++)
        for (int k = 0; k < n_bands; k++) {
            float *rs = pre + (size_t)p * E + 2 * k;
            const float mag = sqrtf(rs[0] * rs[0] + rs[1] * rs[1]);
            if (mag > thr && mag > 0.001f) {
                /* agc.rs knee_compress */
                const float excess = mag - thr;
                const float compressed = thr + thr * tanhf(excess / thr);
                const float scale = compressed / mag;
                rs[0] *= scale;
                rs[1] *= scale;
            }
        }
}

/* fft_ode.rs:123-141 deriv_sequential_into (n_bands < 256), and the same
 * with the FFT path's circular neighbour indexing (n_bands >= 256). */
static void kerr_deriv(const float *r, const float *s, int n, const float *gamma, const float *omega, float alpha,
                       float beta, int fft_len, float *msq, float *dr, float *ds) {
    for (int k = 0; k < n; k++) msq[k] = r[k] * r[k] + s[k] * s[k];
    for (int k = 0; k < n; k++) {
        float ns = 0.0f;
        if (fft_len == 0) {
            if (k >= 2) ns += r[k - 2] * r[k - 2] + s[k - 2] * s[k - 2];
            if (k >= 1) ns += r[k - 1] * r[k - 1] + s[k - 1] * s[k - 1];
            if (k + 1 < n) ns += r[k + 1] * r[k + 1] + s[k + 1] * s[k + 1];
            if (k + 2 < n) ns += r[k + 2] * r[k + 2] + s[k + 2] * s[k + 2];
        } else {
            const int off[4] = {-2, -1, 1, 2};
            for (int u = 0; u < 4; u++) {
                const int j = ((k + off[u]) % fft_len + fft_len) % fft_len;
                if (j < n) ns += msq[j];
            }
        }
        const float phi = omega[k] + alpha * msq[k] + beta * ns;
        dr[k] = -gamma[k] * r[k] - phi * s[k];
        ds[k] = -gamma[k] * s[k] + phi * r[k];
    }
}

typedef struct {
    int n_embd, maestro_dim, out_groups, rk4_steps, use_corrector;
    const float *mi_sq_w, *mi_sq_b, *mi_pr_w, *mi_pr_b;  /* maestro_in: squeeze [M][E], process_1 [E][M] */
    const float *mo_sq_w, *mo_sq_b, *mo_pr_w, *mo_pr_b;  /* maestro_out */
    const float *gamma_raw, *omega;                      /* [n_bands] */
    float alpha, beta;
    const float *phase_correction;                      /* [n_bands] */
    const float *rk4_w;                                  /* [4] */
    const float *op_w, *op_b;  /* out_proj: dense [E][E] + [E], or groups x ([gs][gs] + [gs]) packed in order */
} wo_ffn;

/* fft_ode.rs:171-250 kerr_ode_fft for one position x [E] -> out [E]. */
static void kerr_ode(const wo_ffn *f, const float *x, float *out) {
    const int n = f->n_embd / 2;
    int fft_len = 0;
    if (n >= 256) {
        fft_len = 1;
        while (fft_len < n) fft_len <<= 1;
    }
    const float dt = 1.0f / (float)f->rk4_steps;
    float *buf = (float *)malloc(sizeof(float) * (size_t)n * 14);
    float *r = buf, *s = r + n, *rt = s + n, *st = rt + n, *k1r = st + n, *k1s = k1r + n, *k2r = k1s + n,
          *k2s = k2r + n, *k3r = k2s + n, *k3s = k3r + n, *k4r = k3s + n, *k4s = k4r + n, *gamma = k4s + n,
          *msq = gamma + n;
    for (int k = 0; k < n; k++) {
        gamma[k] = wo_softplus(f->gamma_raw[k]);
        r[k] = x[2 * k];
        s[k] = x[2 * k + 1];
    }
    const float *w = f->rk4_w;
    for (int step = 0; step < f->rk4_steps; step++) {
        kerr_deriv(r, s, n, gamma, f->omega, f->alpha, f->beta, fft_len, msq, k1r, k1s);
        for (int i = 0; i < n; i++) rt[i] = r[i] + 0.5f * dt * k1r[i];
        for (int i = 0; i < n; i++) st[i] = s[i] + 0.5f * dt * k1s[i];
        kerr_deriv(rt, st, n, gamma, f->omega, f->alpha, f->beta, fft_len, msq, k2r, k2s);
        for (int i = 0; i < n; i++) rt[i] = r[i] + 0.5f * dt * k2r[i];
        for (int i = 0; i < n; i++) st[i] = s[i] + 0.5f * dt * k2s[i];
        kerr_deriv(rt, st, n, gamma, f->omega, f->alpha, f->beta, fft_len, msq, k3r, k3s);
        for (int i = 0; i < n; i++) rt[i] = r[i] + dt * k3r[i];
        for (int i = 0; i < n; i++) st[i] = s[i] + dt * k3s[i];
        kerr_deriv(rt, st, n, gamma, f->omega, f->alpha, f->beta, fft_len, msq, k4r, k4s);
        for (int i = 0; i < n; i++) {
            r[i] += dt * (w[0] * k1r[i] + w[1] * k2r[i] + w[2] * k3r[i] + w[3] * k4r[i]);
            s[i] += dt * (w[0] * k1s[i] + w[1] * k2s[i] + w[2] * k3s[i] + w[3] * k4s[i]);
        }
    }
    for (int k = 0; k < n; k++) {
        out[2 * k] = r[k];
        out[2 * k + 1] = s[k];
    }
    free(buf);
}

/* src/common/out_proj.rs:24-40 forward: dense = linear; block-diagonal =
 * per group, the sum started at the bias. */
static void out_proj(const wo_ffn *f, const float *x, float *y) {
    const int E = f->n_embd;
    if (f->out_groups <= 1) {
        linear(f->op_w, f->op_b, E, E, x, y);
        return;
    }
    const int gs = E / f->out_groups;
    const float *p = f->op_w;  /* groups packed: w [gs][gs] then b [gs] */
    for (int g = 0; g < f->out_groups; g++) {
        const float *gw = p, *gb = p + (size_t)gs * gs;
        for (int i = 0; i < gs; i++) {
            float sum = gb[i];
            for (int j = 0; j < gs; j++) sum += gw[(size_t)i * gs + j] * x[g * gs + j];
            y[g * gs + i] = sum;
        }
        p += (size_t)gs * gs + gs;
    }
}

/* ffn.rs:39-230 ffn_forward_via_backend as the serve tier calls it
 * (freeze_ode, stencil, no memory): x [t][E] -> y [t][E]; agc updated. */
int wo_ffn_forward(const wo_ffn *f, wo_agc *agc, const float *x, int t, float *y) {
    const int E = f->n_embd, M = f->maestro_dim, n = E / 2;
    float *pre = (float *)malloc(sizeof(float) * (size_t)t * E);
    float *sq = (float *)malloc(sizeof(float) * (size_t)M + 4);
    float *tmp = (float *)malloc(sizeof(float) * (size_t)E * 3);
    float *ko = tmp + E, *reg = ko + E;
    if (!pre || !sq || !tmp) return -1;
    for (int p = 0; p < t; p++) {  /* maestro_in and the residual precond = x + mae_in_out */
        linear(f->mi_sq_w, f->mi_sq_b, M, E, x + (size_t)p * E, sq);
        for (int i = 0; i < M; i++) sq[i] = gelu(sq[i]);
        linear(f->mi_pr_w, f->mi_pr_b, E, M, sq, tmp);
        for (int i = 0; i < E; i++) pre[(size_t)p * E + i] = x[(size_t)p * E + i] + tmp[i];
    }
    agc_process(agc, pre, t, n);
    for (int p = 0; p < t; p++) {
        kerr_ode(f, pre + (size_t)p * E, ko);
        if (f->use_corrector)  /* ffn.rs:162-181 corrector plate */
            for (int k = 0; k < n; k++) {
                const float sc = sinf(f->phase_correction[k]), cc = cosf(f->phase_correction[k]);
                const float r = ko[2 * k], s = ko[2 * k + 1];
                ko[2 * k] = r * cc - s * sc;
                ko[2 * k + 1] = r * sc + s * cc;
            }
        linear(f->mo_sq_w, f->mo_sq_b, M, E, ko, sq);
        for (int i = 0; i < M; i++) sq[i] = gelu(sq[i]);
        linear(f->mo_pr_w, f->mo_pr_b, E, M, sq, tmp);
        for (int i = 0; i < E; i++) reg[i] = ko[i] + tmp[i];
        out_proj(f, reg, y + (size_t)p * E);
    }
    free(pre);
    free(sq);
    free(tmp);
    return 0;
}

/* kv_cache.rs:18-33 phase_native_decode: rotate each band by the output
 * corrector, then one dot product per vocabulary row of wte. */
void wo_phase_native_decode(const float *hidden, const float *corrector, const float *wte, int vocab, int n_bands,
                            float *logits) {
    const int E = 2 * n_bands;
    float *c = (float *)malloc(sizeof(float) * (size_t)E);
    for (int k = 0; k < n_bands; k++) {
        const float sc = sinf(corrector[k]), cc = cosf(corrector[k]);
        const float r = hidden[2 * k], s = hidden[2 * k + 1];
        c[2 * k] = r * cc - s * sc;
        c[2 * k + 1] = r * sc + s * cc;
    }
    for (int v = 0; v < vocab; v++) {
        float score = 0.0f;
        const float *e = wte + (size_t)v * E;
        for (int j = 0; j < E; j++) score += c[j] * e[j];
        logits[v] = score;
    }
    free(c);
}

/* kv_cache.rs:365-378: logits = lm_head . final_normed (no bias). */
void wo_lm_head(const float *hidden, const float *lm_head, int vocab, int E, float *logits) {
    for (int v = 0; v < vocab; v++) {
        float sum = 0.0f;
        for (int j = 0; j < E; j++) sum += lm_head[(size_t)v * E + j] * hidden[j];
        logits[v] = sum;
    }
}

/* kv_cache.rs:106-113 / :252-256: hidden = wte[tok] + wpe[pos] (wpe only
 * while pos < n_pos). */
void wo_embed(const int32_t *tokens, const int32_t *pos, int t, const float *wte, const float *wpe, int n_pos, int E,
              float *hidden) {
    for (int p = 0; p < t; p++) {
        const float *e = wte + (size_t)tokens[p] * E;
        float *h = hidden + (size_t)p * E;
        for (int j = 0; j < E; j++) h[j] = e[j];
        if (wpe && pos[p] < n_pos)
            for (int j = 0; j < E; j++) h[j] += wpe[(size_t)pos[p] * E + j];
    }
}
