/*
 * wave_oracle.c -- CPU restatement of wave-engine's causal multi-head wave
 * attention forward, used ONLY as test infrastructure (the parity checker
 * and the timed CPU baseline).  Nothing in the product path links or calls
 * this file.
 *
 * PARITY STATUS: parity unpinned.  The reference is Rust (crate
 * `wave-engine` 0.1.0) and cannot be compiled in this environment (no
 * rustc/cargo, missing path dependency `../kerr-memory`, no network), and
 * the reference ships no golden vectors or forward-pass tests for this path.
 * The restatement is pinned instead by hand-derived known-answer cases
 * (tests/golden/make_golden.py) that follow from the reference's semantics.
 *
 * Every function names the reference lines it restates.  Arithmetic follows
 * the reference statement by statement: fp32 throughout, products rounded
 * before the add (rustc never contracts to FMA; build with
 * -ffp-contract=off), sums in the reference's sequential order, glibc
 * atan2f/cosf/expf/logf/fmodf (Rust's f32 methods call the platform libm on
 * Linux).
 *
 * Layouts (all row-major, fp32):
 *   harmonic_raw [H]          phase_w [H][2][E]     phase_b [H][2]
 *   v_w [H][d][d]             v_b [H][d]
 *   content_w [H][C][E]       content_b [H][C]      (C = 0 or 16)
 *   out_w [E][E]              out_b [E]
 *   x [T][E]  ->  y [T][E];   att_w [H][T][T] (optional)
 * and, for the legacy dot-product attention (wo_dot_attn_forward, end of
 * file): c_attn_w [3E][E], c_attn_b [3E], c_proj_w [E][E], c_proj_b [E].
 *
 * The attention backward at the end of the file (attn_backward.rs, composed
 * as attn.rs:346-430) is pinned by the reference's own known-answer tests
 * (attn_backward.rs:336-430) and by finite differences of the forward.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define WO_N_BUCKETS 8
/* std::f32::consts::TAU rounded to f32. */
#define WO_TAU 6.28318548202514648438f

typedef struct {
    int n_embd, n_head, content_dim;
    const float *harmonic_raw, *phase_w, *phase_b, *v_w, *v_b;
    const float *content_w, *content_b, *out_w, *out_b;
} wo_weights;

/* src/common/math/core.rs:5 -- softplus(x) = x > 20 ? x : ln(1 + e^x). */
float wo_softplus(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

/* src/common/kv_cache.rs:66-70 and src/common/attn.rs:168-174. */
int wo_phase_to_bucket(float phase) {
    const float bucket_width = WO_TAU / (float)WO_N_BUCKETS;
    float normalized = fmodf(fmodf(phase, WO_TAU) + WO_TAU, WO_TAU);
    float q = normalized / bucket_width;
    /* Rust `as usize` saturates: NaN and negatives become 0. */
    size_t b = (q != q || q <= 0.0f) ? 0 : (size_t)q;
    return (int)(b < WO_N_BUCKETS - 1 ? b : WO_N_BUCKETS - 1);
}

/* src/common/attn.rs:74-83 (project_phase); same order at attn.rs:124-127. */
static float project_phase(const float *x, int n, const float *w2, const float *b2,
                           float *r_out, float *s_out) {
    float r = b2[0], s = b2[1];
    for (int j = 0; j < n; j++) {
        r += w2[j] * x[j];
        s += w2[n + j] * x[j];
    }
    if (r_out) *r_out = r;
    if (s_out) *s_out = s;
    return atan2f(s, r);
}

/* src/common/attn.rs:155-165 -- block-diagonal value projection of the
 * head's slice: v[d] = (sum_j Wv[d][j] * x[off+j]) + b[d]. */
static void value_project(const float *xh, int hd, const float *vw, const float *vb, float *v) {
    for (int d = 0; d < hd; d++) {
        float sum = 0.0f;
        for (int j = 0; j < hd; j++) sum += vw[d * hd + j] * xh[j];
        v[d] = sum + vb[d];
    }
}

static inline int bucket_adjacent(int qb, int kb) {
    return kb == (qb + WO_N_BUCKETS - 1) % WO_N_BUCKETS || kb == qb ||
           kb == (qb + 1) % WO_N_BUCKETS;
}

/* ---------------------------------------------------------------------------
 * One head of wave_attention_forward: src/common/attn.rs:116-256.
 * head_out [T][d]; att_w_head [T][T] or NULL; phase_override [T] or NULL
 * (mask-conditioned parity: use these phases instead of projecting);
 * phases_out [T] or NULL.
 * ------------------------------------------------------------------------- */
static void attn_one_head(const wo_weights *w, const float *x, int t, int head,
                          float *head_out, float *att_w_head,
                          const float *phase_override, float *phases_out) {
    const int E = w->n_embd, H = w->n_head, hd = E / H, C = w->content_dim;
    const float harmonic_n = wo_softplus(w->harmonic_raw[head]);
    const int offset = head * hd;

    float *phases = (float *)malloc(sizeof(float) * (size_t)(t > 0 ? t : 1));
    float *content = C ? (float *)malloc(sizeof(float) * (size_t)t * C) : NULL;
    float *v_all = (float *)malloc(sizeof(float) * (size_t)t * hd + 4);
    int *buckets = (int *)malloc(sizeof(int) * (size_t)(t > 0 ? t : 1));
    int *bpos = (int *)malloc(sizeof(int) * (size_t)(t > 0 ? t : 1) * WO_N_BUCKETS);
    int bcount[WO_N_BUCKETS] = {0};
    float *scores = (float *)malloc(sizeof(float) * (size_t)(t > 0 ? t : 1));

    /* attn.rs:121-130 phase projection */
    const float *pw = w->phase_w + (size_t)head * 2 * E, *pb = w->phase_b + head * 2;
    for (int pos = 0; pos < t; pos++) {
        float ph = project_phase(x + (size_t)pos * E, E, pw, pb, NULL, NULL);
        phases[pos] = phase_override ? phase_override[pos] : ph;
        if (phases_out) phases_out[pos] = phases[pos];
    }
    /* attn.rs:135-152 content projection (frozen symmetry breaker) */
    if (C) {
        const float *cw = w->content_w + (size_t)head * C * E, *cb = w->content_b + head * C;
        for (int pos = 0; pos < t; pos++)
            for (int d = 0; d < C; d++) {
                float sum = cb[d];
                for (int j = 0; j < E; j++) sum += cw[(size_t)d * E + j] * x[(size_t)pos * E + j];
                content[(size_t)pos * C + d] = sum;
            }
    }
    const float content_scale = C > 0 ? 1.0f / sqrtf((float)C) : 0.0f;
    /* attn.rs:155-165 value projection */
    for (int pos = 0; pos < t; pos++)
        value_project(x + (size_t)pos * E + offset, hd, w->v_w + (size_t)head * hd * hd,
                      w->v_b + head * hd, v_all + (size_t)pos * hd);
    /* attn.rs:168-179 bucket hash and per-bucket position lists */
    for (int pos = 0; pos < t; pos++) {
        int b = wo_phase_to_bucket(phases[pos]);
        buckets[pos] = b;
        bpos[b * t + bcount[b]++] = pos;
    }
    /* attn.rs:185-249 per-query scoring, softmax and PV */
    for (int qi = 0; qi < t; qi++) {
        const int qb = buckets[qi];
        for (int k = 0; k < t; k++) scores[k] = -INFINITY;
        for (int db = 0; db <= 2; db++) {
            int tb = db == 0 ? (qb + WO_N_BUCKETS - 1) % WO_N_BUCKETS
                   : db == 1 ? qb : (qb + 1) % WO_N_BUCKETS;
            for (int n = 0; n < bcount[tb]; n++) {
                int ki = bpos[tb * t + n];
                if (ki > qi) continue;
                float delta = phases[qi] - phases[ki];
                float score = cosf(harmonic_n * delta);
                if (C) {
                    float dot = 0.0f;
                    for (int d = 0; d < C; d++)
                        dot += content[(size_t)qi * C + d] * content[(size_t)ki * C + d];
                    score += dot * content_scale;
                }
                scores[ki] = score;
            }
        }
        if (qi > 0 && scores[qi - 1] == -INFINITY) { /* attn.rs:212-221 */
            float delta = phases[qi] - phases[qi - 1];
            float score = cosf(harmonic_n * delta);
            if (C) {
                float dot = 0.0f;
                for (int d = 0; d < C; d++)
                    dot += content[(size_t)qi * C + d] * content[(size_t)(qi - 1) * C + d];
                score += dot * content_scale;
            }
            scores[qi - 1] = score;
        }
        if (scores[qi] == -INFINITY) scores[qi] = 1.0f; /* attn.rs:222-224 */

        float max_s = -INFINITY; /* attn.rs:226 fold(f32::NEG_INFINITY, f32::max) */
        for (int k = 0; k <= qi; k++) max_s = fmaxf(max_s, scores[k]);
        float exp_sum = 0.0f;
        for (int k = 0; k <= qi; k++) {
            if (scores[k] > -INFINITY) {
                scores[k] = expf(scores[k] - max_s);
                exp_sum += scores[k];
            } else {
                scores[k] = 0.0f;
            }
        }
        if (exp_sum > 0.0f)
            for (int k = 0; k <= qi; k++) scores[k] /= exp_sum;
        if (att_w_head) memcpy(att_w_head + (size_t)qi * t, scores, sizeof(float) * (size_t)t);
        for (int d = 0; d < hd; d++) { /* attn.rs:242-248 */
            float sum = 0.0f;
            for (int k = 0; k <= qi; k++)
                if (scores[k] > 0.0f) sum += scores[k] * v_all[(size_t)k * hd + d];
            head_out[(size_t)qi * hd + d] = sum;
        }
    }
    free(phases); free(content); free(v_all); free(buckets); free(bpos); free(scores);
}

/* attn.rs:276-284: y[i] = (sum_j W[i][j] * o[j]) + b[i]. */
static void out_project(const wo_weights *w, const float *merged, int t, float *y) {
    const int E = w->n_embd;
    for (int q = 0; q < t; q++)
        for (int i = 0; i < E; i++) {
            float sum = 0.0f;
            for (int j = 0; j < E; j++) sum += w->out_w[(size_t)i * E + j] * merged[(size_t)q * E + j];
            y[(size_t)q * E + i] = sum + w->out_b[i];
        }
}

typedef struct {
    const wo_weights *w;
    const float *x;
    int t, head_begin, head_end, head_step;
    float *head_out;            /* [H][T][d] */
    float *att_w;               /* [H][T][T] or NULL */
    const float *phase_override;/* [H][T] or NULL */
    float *phases_out;          /* [H][T] or NULL */
} head_job;

static void *head_worker(void *arg) {
    head_job *j = (head_job *)arg;
    const int hd = j->w->n_embd / j->w->n_head;
    for (int h = j->head_begin; h < j->head_end; h += j->head_step)
        attn_one_head(j->w, j->x, j->t, h, j->head_out + (size_t)h * j->t * hd,
                      j->att_w ? j->att_w + (size_t)h * j->t * j->t : NULL,
                      j->phase_override ? j->phase_override + (size_t)h * j->t : NULL,
                      j->phases_out ? j->phases_out + (size_t)h * j->t : NULL);
    return NULL;
}

/* ---------------------------------------------------------------------------
 * wave_attention_forward for one sequence: src/common/attn.rs:90-305 with
 * backend = None and return_pathway_cache = false.  n_threads > 1 runs heads
 * on threads like the reference's rayon into_par_iter over heads
 * (attn.rs:116); results do not depend on n_threads.
 * Returns 0, or -1 on bad arguments / allocation failure.
 * ------------------------------------------------------------------------- */
int wo_attn_forward(const wo_weights *w, const float *x, int t, float *y, float *att_w,
                    const float *phase_override, float *phases_out, int n_threads) {
    if (!w || t < 0 || w->n_head <= 0 || w->n_embd % w->n_head) return -1;
    if (t == 0) return 0;
    const int E = w->n_embd, H = w->n_head, hd = E / H;
    float *head_out = (float *)malloc(sizeof(float) * (size_t)H * t * hd);
    float *merged = (float *)malloc(sizeof(float) * (size_t)t * E);
    if (!head_out || !merged) { free(head_out); free(merged); return -1; }
    if (n_threads < 1) n_threads = 1;
    if (n_threads > H) n_threads = H;
    head_job jobs[64];
    pthread_t th[64];
    if (n_threads > 64) n_threads = 64;
    for (int i = 0; i < n_threads; i++) {
        jobs[i] = (head_job){w, x, t, i, H, n_threads, head_out, att_w, phase_override, phases_out};
        if (n_threads > 1) pthread_create(&th[i], NULL, head_worker, &jobs[i]);
    }
    if (n_threads > 1) for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    else head_worker(&jobs[0]);
    /* attn.rs:259-270 head merge */
    for (int h = 0; h < H; h++)
        for (int q = 0; q < t; q++)
            memcpy(merged + (size_t)q * E + h * hd, head_out + ((size_t)h * t + q) * hd, sizeof(float) * hd);
    out_project(w, merged, t, y);
    free(head_out); free(merged);
    return 0;
}

/* ---------------------------------------------------------------------------
 * KV-cache attention, src/common/kv_cache.rs.  One (layer) cache:
 *   phases [H][cap], buckets [H][cap], values [H][cap][d]; *n_cached.
 * ------------------------------------------------------------------------- */

/* kv_cache.rs:121-193 -- prefill attention + out_proj for one prompt of T
 * positions starting from an empty cache.  No content bias (the serve copy
 * ignores content_proj), heads serial.  Appends T entries to the cache. */
int wo_kv_prefill(const wo_weights *w, const float *x, int t, float *y,
                  float *phases, int *buckets, float *values, int cap, int *n_cached) {
    const int E = w->n_embd, H = w->n_head, hd = E / H;
    if (*n_cached != 0 || t > cap || t <= 0) return -1;
    float *attn_out = (float *)calloc((size_t)t * E, sizeof(float));
    float *scores = (float *)malloc(sizeof(float) * (size_t)t);
    int *bpos = (int *)malloc(sizeof(int) * (size_t)t * WO_N_BUCKETS);
    if (!attn_out || !scores || !bpos) { free(attn_out); free(scores); free(bpos); return -1; }
    for (int head = 0; head < H; head++) {
        const float harmonic_n = wo_softplus(w->harmonic_raw[head]);
        const int offset = head * hd;
        float *ph = phases + (size_t)head * cap;
        int *bk = buckets + (size_t)head * cap;
        float *vv = values + (size_t)head * cap * hd;
        int bcount[WO_N_BUCKETS] = {0};
        for (int pos = 0; pos < t; pos++) { /* kv_cache.rs:129-142 */
            ph[pos] = project_phase(x + (size_t)pos * E, E, w->phase_w + (size_t)head * 2 * E,
                                    w->phase_b + head * 2, NULL, NULL);
            value_project(x + (size_t)pos * E + offset, hd, w->v_w + (size_t)head * hd * hd,
                          w->v_b + head * hd, vv + (size_t)pos * hd);
            bk[pos] = wo_phase_to_bucket(ph[pos]);
            bpos[bk[pos] * t + bcount[bk[pos]]++] = pos;
        }
        for (int qi = 0; qi < t; qi++) { /* kv_cache.rs:146-181 */
            const int qb = bk[qi];
            for (int k = 0; k < t; k++) scores[k] = -INFINITY;
            for (int db = 0; db <= 2; db++) {
                int tb = db == 0 ? (qb + WO_N_BUCKETS - 1) % WO_N_BUCKETS
                       : db == 1 ? qb : (qb + 1) % WO_N_BUCKETS;
                for (int n = 0; n < bcount[tb]; n++) {
                    int ki = bpos[tb * t + n];
                    if (ki > qi) continue;
                    scores[ki] = cosf(harmonic_n * (ph[qi] - ph[ki]));
                }
            }
            if (qi > 0 && scores[qi - 1] == -INFINITY)
                scores[qi - 1] = cosf(harmonic_n * (ph[qi] - ph[qi - 1]));
            if (scores[qi] == -INFINITY) scores[qi] = 1.0f;
            float max_s = -INFINITY;
            for (int k = 0; k <= qi; k++) max_s = fmaxf(max_s, scores[k]);
            float exp_sum = 0.0f;
            for (int k = 0; k <= qi; k++) {
                if (scores[k] > -INFINITY) { scores[k] = expf(scores[k] - max_s); exp_sum += scores[k]; }
                else scores[k] = 0.0f;
            }
            if (exp_sum > 0.0f) for (int k = 0; k <= qi; k++) scores[k] /= exp_sum;
            for (int d = 0; d < hd; d++) {
                float sum = 0.0f;
                for (int k = 0; k <= qi; k++)
                    if (scores[k] > 0.0f) sum += scores[k] * vv[(size_t)k * hd + d];
                attn_out[(size_t)qi * E + offset + d] = sum;
            }
        }
    }
    out_project(w, attn_out, t, y); /* kv_cache.rs:185-193 */
    *n_cached = t;
    free(attn_out); free(scores); free(bpos);
    return 0;
}

/* kv_cache.rs:263-335 -- forward_one attention + out_proj for one new
 * position x [E] against a cache holding *n_cached entries; appends it. */
int wo_kv_decode(const wo_weights *w, const float *x, float *y,
                 float *phases, int *buckets, float *values, int cap, int *n_cached) {
    const int E = w->n_embd, H = w->n_head, hd = E / H;
    const int n = *n_cached;
    if (n >= cap || n < 0) return -1;
    float *attn_out = (float *)calloc((size_t)E, sizeof(float));
    float *scores = (float *)malloc(sizeof(float) * (size_t)(n + 1));
    float *v_new = (float *)malloc(sizeof(float) * (size_t)hd);
    if (!attn_out || !scores || !v_new) { free(attn_out); free(scores); free(v_new); return -1; }
    for (int head = 0; head < H; head++) {
        const float harmonic_n = wo_softplus(w->harmonic_raw[head]);
        const int offset = head * hd;
        float *ph = phases + (size_t)head * cap;
        int *bk = buckets + (size_t)head * cap;
        float *vv = values + (size_t)head * cap * hd;
        float phase = project_phase(x, E, w->phase_w + (size_t)head * 2 * E, w->phase_b + head * 2, NULL, NULL);
        value_project(x + offset, hd, w->v_w + (size_t)head * hd * hd, w->v_b + head * hd, v_new);
        int bucket = wo_phase_to_bucket(phase);
        for (int k = 0; k <= n; k++) scores[k] = -INFINITY;
        /* kv_cache.rs:285-292: every cached key in buckets b-1, b, b+1
         * (bucket lists are ascending positions; order does not matter). */
        for (int k = 0; k < n; k++)
            if (bucket_adjacent(bucket, bk[k])) scores[k] = cosf(harmonic_n * (phase - ph[k]));
        scores[n] = 1.0f; /* kv_cache.rs:294 self */
        if (n > 0 && scores[n - 1] == -INFINITY) /* kv_cache.rs:296-298 */
            scores[n - 1] = cosf(harmonic_n * (phase - ph[n - 1]));
        float max_s = -INFINITY;
        for (int k = 0; k <= n; k++) max_s = fmaxf(max_s, scores[k]);
        float exp_sum = 0.0f;
        for (int k = 0; k <= n; k++) {
            if (scores[k] > -INFINITY) { scores[k] = expf(scores[k] - max_s); exp_sum += scores[k]; }
            else scores[k] = 0.0f;
        }
        if (exp_sum > 0.0f) for (int k = 0; k <= n; k++) scores[k] /= exp_sum;
        for (int d = 0; d < hd; d++) { /* kv_cache.rs:312-320 */
            float sum = 0.0f;
            for (int k = 0; k < n; k++)
                if (scores[k] > 0.0f) sum += scores[k] * vv[(size_t)k * hd + d];
            sum += scores[n] * v_new[d];
            attn_out[offset + d] = sum;
        }
        ph[n] = phase; /* kv_cache.rs:323-326 append */
        bk[n] = bucket;
        memcpy(vv + (size_t)n * hd, v_new, sizeof(float) * hd);
    }
    out_project(w, attn_out, 1, y); /* kv_cache.rs:330-335 */
    *n_cached = n + 1;
    free(attn_out); free(scores); free(v_new);
    return 0;
}

/* ---------------------------------------------------------------------------
 * Seeded generators.
 * src/common/rng.rs:24-39: xorshift64 (13, 7, 17), next_f32 = (u >> 40) / 2^24,
 * uniform(limit) = (next_f32 * 2 - 1) * limit.
 * ------------------------------------------------------------------------- */
uint64_t wo_xorshift_next(uint64_t *state) {
    uint64_t s = *state;
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    *state = s;
    return s;
}
float wo_next_f32(uint64_t *state) {
    return (float)(wo_xorshift_next(state) >> 40) / (float)(1ull << 24);
}
float wo_uniform(uint64_t *state, float limit) { return (wo_next_f32(state) * 2.0f - 1.0f) * limit; }

/* Fill `out` with n draws of uniform(limit), advancing *state in order. */
void wo_fill_uniform(uint64_t *state, float limit, float *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = wo_uniform(state, limit);
}

/* src/common/wave_model.rs:39-46 (init_linear) and :57-81 (init_block_attn):
 * per head, phase_proj [2][E] ~ U(+-1/sqrt(E)), v_proj [d][d] ~ U(+-1/sqrt(d)),
 * content_proj [C][E] ~ U(+-1/sqrt(E)) when C > 0, biases zero, harmonic_raw =
 * ln((h+1) * 0.5); then out_proj [E][E] ~ U(+-1/sqrt(E)).  Draw order is the
 * reference's.  Buffers use the layouts in the header comment. */
void wo_init_block_attn(uint64_t *state, int n_head, int n_embd, int content_dim,
                        float *harmonic_raw, float *phase_w, float *phase_b, float *v_w, float *v_b,
                        float *content_w, float *content_b, float *out_w, float *out_b) {
    const int hd = n_embd / n_head;
    const float lim_e = 1.0f / sqrtf((float)n_embd), lim_d = 1.0f / sqrtf((float)hd);
    for (int h = 0; h < n_head; h++) {
        wo_fill_uniform(state, lim_e, phase_w + (size_t)h * 2 * n_embd, (size_t)2 * n_embd);
        phase_b[2 * h] = phase_b[2 * h + 1] = 0.0f;
        wo_fill_uniform(state, lim_d, v_w + (size_t)h * hd * hd, (size_t)hd * hd);
        memset(v_b + (size_t)h * hd, 0, sizeof(float) * hd);
        if (content_dim > 0) {
            wo_fill_uniform(state, lim_e, content_w + (size_t)h * content_dim * n_embd,
                            (size_t)content_dim * n_embd);
            memset(content_b + (size_t)h * content_dim, 0, sizeof(float) * content_dim);
        }
        harmonic_raw[h] = logf((float)(h + 1) * 0.5f);
    }
    wo_fill_uniform(state, lim_e, out_w, (size_t)n_embd * n_embd);
    memset(out_b, 0, sizeof(float) * n_embd);
}

/* ---------------------------------------------------------------------------
 * Batched CPU baseline: B sequences x H heads on n_threads threads, the
 * reference's thread-per-batch-element (src/cpu/train_loop.rs:320) times
 * rayon-over-heads (attn.rs:116) flattened into one (sequence, head) pool.
 * ------------------------------------------------------------------------- */
typedef struct {
    const wo_weights *w;
    const float *x;
    int b, t;
    float *head_out; /* [B][H][T][d] */
    int next;        /* shared work counter */
    pthread_mutex_t mu;
} pool_state;

static void *pool_worker(void *arg) {
    pool_state *p = (pool_state *)arg;
    const int H = p->w->n_head, E = p->w->n_embd, hd = E / H;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        int item = p->next++;
        pthread_mutex_unlock(&p->mu);
        if (item >= p->b * H) break;
        int bi = item / H, h = item % H;
        attn_one_head(p->w, p->x + (size_t)bi * p->t * E, p->t, h,
                      p->head_out + ((size_t)bi * H + h) * p->t * hd, NULL, NULL, NULL);
    }
    return NULL;
}

typedef struct {
    const wo_weights *w;
    const float *merged;
    float *y;
    int rows, next;
    pthread_mutex_t mu;
} proj_state;

static void *proj_worker(void *arg) {
    proj_state *p = (proj_state *)arg;
    const int E = p->w->n_embd;
    for (;;) {
        pthread_mutex_lock(&p->mu);
        int r0 = p->next;
        p->next += 16;
        pthread_mutex_unlock(&p->mu);
        if (r0 >= p->rows) break;
        int r1 = r0 + 16 < p->rows ? r0 + 16 : p->rows;
        out_project(p->w, p->merged + (size_t)r0 * E, r1 - r0, p->y + (size_t)r0 * E);
    }
    return NULL;
}

int wo_attn_forward_batch(const wo_weights *w, const float *x, int b, int t, float *y, int n_threads) {
    const int E = w->n_embd, H = w->n_head, hd = E / H;
    if (b <= 0 || t <= 0) return 0;
    float *head_out = (float *)malloc(sizeof(float) * (size_t)b * H * t * hd);
    float *merged = (float *)malloc(sizeof(float) * (size_t)b * t * E);
    if (!head_out || !merged) { free(head_out); free(merged); return -1; }
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    pool_state ps = {w, x, b, t, head_out, 0, PTHREAD_MUTEX_INITIALIZER};
    for (int i = 0; i < n_threads; i++) pthread_create(&th[i], NULL, pool_worker, &ps);
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    for (int bi = 0; bi < b; bi++)
        for (int h = 0; h < H; h++)
            for (int q = 0; q < t; q++)
                memcpy(merged + ((size_t)bi * t + q) * E + h * hd,
                       head_out + (((size_t)bi * H + h) * t + q) * hd, sizeof(float) * hd);
    proj_state pj = {w, merged, y, b * t, 0, PTHREAD_MUTEX_INITIALIZER};
    for (int i = 0; i < n_threads; i++) pthread_create(&th[i], NULL, proj_worker, &pj);
    for (int i = 0; i < n_threads; i++) pthread_join(th[i], NULL);
    free(head_out); free(merged);
    return 0;
}

/* ---------------------------------------------------------------------------
 * Legacy dot-product attention: src/common/compute.rs:357-414 (attention_cpu,
 * the CPU ComputeBackend::attention of compute.rs:43).  linear_fn is
 * model.rs:144-150: y[i] = b[i] + (sum_j W[i][j] * x[j]), the sum sequential.
 * c_attn_w [3E][E], c_attn_b [3E], c_proj_w [E][E], c_proj_b [E]; x, y [T][E].
 * ------------------------------------------------------------------------- */
static void dot_linear(const float *w, const float *b, int n_out, int n_in, const float *x, float *y) {
    for (int i = 0; i < n_out; i++) {
        float sum = 0.0f;
        for (int j = 0; j < n_in; j++) sum += w[(size_t)i * n_in + j] * x[j];
        y[i] = b[i] + sum;
    }
}

int wo_dot_attn_forward(int n_head, int n_embd, const float *c_attn_w, const float *c_attn_b,
                        const float *c_proj_w, const float *c_proj_b, const float *x, int t, float *y) {
    const int E = n_embd, hd = E / n_head;
    if (n_head <= 0 || E % n_head || t <= 0) return -1;
    const float scale = 1.0f / sqrtf((float)hd); /* compute.rs:362 */
    float *qkv = (float *)malloc(sizeof(float) * (size_t)t * 3 * E);
    float *out = (float *)calloc((size_t)t * E, sizeof(float));
    float *att = (float *)malloc(sizeof(float) * (size_t)t);
    if (!qkv || !out || !att) {
        free(qkv);
        free(out);
        free(att);
        return -1;
    }
    for (int pos = 0; pos < t; pos++) /* compute.rs:368-375 */
        dot_linear(c_attn_w, c_attn_b, 3 * E, E, x + (size_t)pos * E, qkv + (size_t)pos * 3 * E);
    for (int head = 0; head < n_head; head++) { /* compute.rs:379-407 */
        const int off = head * hd;
        for (int qi = 0; qi < t; qi++) {
            const float *q = qkv + (size_t)qi * 3 * E + off;
            for (int ki = 0; ki <= qi; ki++) {
                const float *k = qkv + (size_t)ki * 3 * E + E + off;
                float dot = 0.0f;
                for (int d = 0; d < hd; d++) dot += q[d] * k[d];
                att[ki] = dot * scale;
            }
            float max_att = -INFINITY;
            for (int ki = 0; ki <= qi; ki++) max_att = fmaxf(max_att, att[ki]);
            float exp_sum = 0.0f;
            for (int ki = 0; ki <= qi; ki++) {
                att[ki] = expf(att[ki] - max_att);
                exp_sum += att[ki];
            }
            for (int ki = 0; ki <= qi; ki++) att[ki] /= exp_sum;
            for (int d = 0; d < hd; d++) {
                float sum = 0.0f;
                for (int ki = 0; ki <= qi; ki++) sum += att[ki] * qkv[(size_t)ki * 3 * E + 2 * E + off + d];
                out[(size_t)qi * E + off + d] = sum;
            }
        }
    }
    for (int pos = 0; pos < t; pos++) /* compute.rs:410-412 */
        dot_linear(c_proj_w, c_proj_b, E, E, out + (size_t)pos * E, y + (size_t)pos * E);
    free(qkv);
    free(out);
    free(att);
    return 0;
}

/* ---------------------------------------------------------------------------
 * Attention backward (the next row of the path, not yet on the GPU):
 * src/common/math/attn_backward.rs:17-328 (the primitives) composed as
 * src/common/attn.rs:346-430 (wave_attention_backward_full).  Flat row-major
 * arrays; every sum in the reference's loop order.  Outputs are overwritten.
 * ------------------------------------------------------------------------- */

/* attn_backward.rs:17-53: d_out = W^T d_y, d_w += d_y (x) merged, d_b += d_y. */
void wo_bwd_out_proj(const float *d_y, const float *merged, const float *w, int n, int t, float *d_out,
                     float *d_w, float *d_b) {
    for (int pos = 0; pos < t; pos++)
        for (int j = 0; j < n; j++) {
            float sum = 0.0f;
            for (int i = 0; i < n; i++) sum += w[(size_t)i * n + j] * d_y[(size_t)pos * n + i];
            d_out[(size_t)pos * n + j] = sum;
        }
    memset(d_w, 0, sizeof(float) * (size_t)n * n);
    for (int pos = 0; pos < t; pos++)
        for (int i = 0; i < n; i++) {
            const float dai = d_y[(size_t)pos * n + i];
            if (fabsf(dai) < 1e-12f) continue;
            for (int j = 0; j < n; j++) d_w[(size_t)i * n + j] += dai * merged[(size_t)pos * n + j];
        }
    memset(d_b, 0, sizeof(float) * (size_t)n);
    for (int pos = 0; pos < t; pos++)
        for (int i = 0; i < n; i++) d_b[i] += d_y[(size_t)pos * n + i];
}

/* attn_backward.rs:72-105: d_att_w[qi][ki] = d_head[qi] . v[ki] and
 * d_v[ki] += att_w[qi][ki] d_head[qi], over kept pairs (att_w > 0). */
void wo_bwd_value_aggregation(const float *d_head, const float *att_w, const float *v, int t, int hd,
                              float *d_att_w, float *d_v) {
    memset(d_att_w, 0, sizeof(float) * (size_t)t * t);
    for (int qi = 0; qi < t; qi++)
        for (int ki = 0; ki <= qi; ki++)
            if (att_w[(size_t)qi * t + ki] > 0.0f) {
                float dw = 0.0f;
                for (int d = 0; d < hd; d++) dw += d_head[(size_t)qi * hd + d] * v[(size_t)ki * hd + d];
                d_att_w[(size_t)qi * t + ki] = dw;
            }
    memset(d_v, 0, sizeof(float) * (size_t)t * hd);
    for (int qi = 0; qi < t; qi++)
        for (int ki = 0; ki <= qi; ki++)
            if (att_w[(size_t)qi * t + ki] > 0.0f)
                for (int d = 0; d < hd; d++)
                    d_v[(size_t)ki * hd + d] += att_w[(size_t)qi * t + ki] * d_head[(size_t)qi * hd + d];
}

/* attn_backward.rs:109-122: d_score = a (d_a - sum_k a_k d_a_k). */
void wo_bwd_softmax(const float *d_att_w, const float *att_w, int t, float *d_scores) {
    memset(d_scores, 0, sizeof(float) * (size_t)t * t);
    for (int qi = 0; qi < t; qi++) {
        float ws = 0.0f;
        for (int ki = 0; ki <= qi; ki++) ws += att_w[(size_t)qi * t + ki] * d_att_w[(size_t)qi * t + ki];
        for (int ki = 0; ki <= qi; ki++)
            d_scores[(size_t)qi * t + ki] = att_w[(size_t)qi * t + ki] * (d_att_w[(size_t)qi * t + ki] - ws);
    }
}

/* attn_backward.rs:128-163: through cos(n (th_q - th_k)) + scale c_q . c_k. */
static void bwd_score(const float *d_scores, const float *phases, float hn, const float *att_w,
                      const float *content, int C, float content_scale, int t, float *d_delta,
                      float *d_content, float *d_hn) {
    memset(d_delta, 0, sizeof(float) * (size_t)t * t);
    if (content) memset(d_content, 0, sizeof(float) * (size_t)t * C);
    float dh = 0.0f;
    for (int qi = 0; qi < t; qi++)
        for (int ki = 0; ki <= qi; ki++)
            if (att_w[(size_t)qi * t + ki] > 0.0f) {
                const float ds = d_scores[(size_t)qi * t + ki];
                const float delta = phases[qi] - phases[ki];
                const float sin_nd = sinf(hn * delta);
                d_delta[(size_t)qi * t + ki] = -sin_nd * hn * ds;
                dh += -sin_nd * delta * ds;
                if (content)
                    for (int cd = 0; cd < C; cd++) {
                        d_content[(size_t)qi * C + cd] += ds * content_scale * content[(size_t)ki * C + cd];
                        d_content[(size_t)ki * C + cd] += ds * content_scale * content[(size_t)qi * C + cd];
                    }
            }
    *d_hn = dh;
}

/* attn_backward.rs:169-184: delta = th_q - th_k. */
static void bwd_phase_subtraction(const float *d_delta, const float *att_w, int t, float *d_phases) {
    memset(d_phases, 0, sizeof(float) * (size_t)t);
    for (int qi = 0; qi < t; qi++)
        for (int ki = 0; ki <= qi; ki++)
            if (att_w[(size_t)qi * t + ki] > 0.0f) {
                d_phases[qi] += d_delta[(size_t)qi * t + ki];
                d_phases[ki] -= d_delta[(size_t)qi * t + ki];
            }
}

/* attn_backward.rs:190-231: through atan2(s, r), [r, s] = W x + b. */
void wo_bwd_phase_projection(const float *d_phases, const float *x, const float *pw, const float *pb, int n, int t,
                             float *d_x, float *d_w, float *d_b) {
    memset(d_x, 0, sizeof(float) * (size_t)t * n);
    memset(d_w, 0, sizeof(float) * (size_t)2 * n);
    d_b[0] = d_b[1] = 0.0f;
    for (int pos = 0; pos < t; pos++) {
        const float dp = d_phases[pos];
        if (fabsf(dp) < 1e-12f) continue;
        float r = pb[0], s = pb[1];
        for (int j = 0; j < n; j++) {
            r += pw[j] * x[(size_t)pos * n + j];
            s += pw[n + j] * x[(size_t)pos * n + j];
        }
        const float mag_sq = r * r + s * s;
        if (mag_sq < 1e-8f) continue;
        const float mag = fmaxf(mag_sq, 1e-12f);
        const float d_r = dp * (-s / mag), d_s = dp * (r / mag);
        for (int j = 0; j < n; j++) {
            d_x[(size_t)pos * n + j] += pw[j] * d_r + pw[n + j] * d_s;
            d_w[j] += d_r * x[(size_t)pos * n + j];
            d_w[n + j] += d_s * x[(size_t)pos * n + j];
        }
        d_b[0] += d_r;
        d_b[1] += d_s;
    }
}

/* attn_backward.rs:237-263: through v = Wv x[off .. off+hd] + b. */
void wo_bwd_value_projection(const float *d_v, const float *x, int off, int hd, int n, int t, const float *vw,
                             float *d_x, float *d_w, float *d_b) {
    memset(d_x, 0, sizeof(float) * (size_t)t * n);
    memset(d_w, 0, sizeof(float) * (size_t)hd * hd);
    memset(d_b, 0, sizeof(float) * (size_t)hd);
    for (int pos = 0; pos < t; pos++)
        for (int dd = 0; dd < hd; dd++) {
            const float dv = d_v[(size_t)pos * hd + dd];
            if (fabsf(dv) < 1e-12f) continue;
            for (int j = 0; j < hd; j++) {
                d_x[(size_t)pos * n + off + j] += vw[(size_t)dd * hd + j] * dv;
                d_w[(size_t)dd * hd + j] += dv * x[(size_t)pos * n + off + j];
            }
            d_b[dd] += dv;
        }
}

/* attn_backward.rs:269-293: through c = Wc x + b. */
static void bwd_content_projection(const float *d_c, const float *x, const float *cw, int C, int n, int t,
                                   float *d_x, float *d_w, float *d_b) {
    memset(d_x, 0, sizeof(float) * (size_t)t * n);
    memset(d_w, 0, sizeof(float) * (size_t)C * n);
    memset(d_b, 0, sizeof(float) * (size_t)C);
    for (int pos = 0; pos < t; pos++)
        for (int cd = 0; cd < C; cd++) {
            const float dc = d_c[(size_t)pos * C + cd];
            if (fabsf(dc) < 1e-12f) continue;
            for (int j = 0; j < n; j++) {
                d_x[(size_t)pos * n + j] += cw[(size_t)cd * n + j] * dc;
                d_w[(size_t)cd * n + j] += dc * x[(size_t)pos * n + j];
            }
            d_b[cd] += dc;
        }
}

/* attn_backward.rs:299-326: d_normed = sum over heads of the three input
 * gradients (phase + value first, then content where present). */
void wo_bwd_combine(const float *dxp, const float *dxv, const float *dxc, int n_head, int t, int n, float *d_normed) {
    memset(d_normed, 0, sizeof(float) * (size_t)t * n);
    for (int h = 0; h < n_head; h++)
        for (int pos = 0; pos < t; pos++) {
            const size_t o = ((size_t)h * t + pos) * n;
            for (int j = 0; j < n; j++) d_normed[(size_t)pos * n + j] += dxp[o + j] + dxv[o + j];
            if (dxc)
                for (int j = 0; j < n; j++) d_normed[(size_t)pos * n + j] += dxc[o + j];
        }
}

/* attn.rs:346-430 wave_attention_backward_full for one sequence x [t][E] and
 * the output gradient d_y [t][E]; the forward cache (WaveAttnCache,
 * attn.rs:51-70) is recomputed with the forward's own arithmetic.  Weight
 * gradients in the layouts of the weights (d_content_w / d_content_b may be
 * NULL when content_dim = 0).  Returns 0, or -1 on bad arguments /
 * allocation failure. */
int wo_attn_backward_full(const wo_weights *w, const float *x, int t, const float *d_y, float *d_x, float *d_out_w,
                          float *d_out_b, float *d_phase_w, float *d_phase_b, float *d_v_w, float *d_v_b,
                          float *d_content_w, float *d_content_b, float *d_harmonic_raw) {
    if (!w || t <= 0 || w->n_head <= 0 || w->n_embd % w->n_head) return -1;
    const int E = w->n_embd, H = w->n_head, hd = E / H, C = w->content_dim;
    const size_t tt = (size_t)t * t;
    float *merged = (float *)calloc((size_t)t * E, sizeof(float));
    float *head_out = (float *)malloc(sizeof(float) * (size_t)t * hd);
    float *att_w = (float *)malloc(sizeof(float) * tt);
    float *phases = (float *)malloc(sizeof(float) * (size_t)t);
    float *v_all = (float *)malloc(sizeof(float) * (size_t)t * hd);
    float *content = C ? (float *)malloc(sizeof(float) * (size_t)t * C) : NULL;
    float *d_out = (float *)malloc(sizeof(float) * (size_t)t * E);
    float *d_head = (float *)malloc(sizeof(float) * (size_t)t * hd);
    float *d_att = (float *)malloc(sizeof(float) * tt);
    float *d_v = (float *)malloc(sizeof(float) * (size_t)t * hd);
    float *d_sc = (float *)malloc(sizeof(float) * tt);
    float *d_delta = (float *)malloc(sizeof(float) * tt);
    float *d_c = C ? (float *)malloc(sizeof(float) * (size_t)t * C) : NULL;
    float *d_ph = (float *)malloc(sizeof(float) * (size_t)t);
    float *dxp = (float *)malloc(sizeof(float) * (size_t)H * t * E);
    float *dxv = (float *)malloc(sizeof(float) * (size_t)H * t * E);
    float *dxc = C ? (float *)malloc(sizeof(float) * (size_t)H * t * E) : NULL;
    int rc = 0;
    if (!merged || !head_out || !att_w || !phases || !v_all || (C && (!content || !d_c || !dxc)) || !d_out ||
        !d_head || !d_att || !d_v || !d_sc || !d_delta || !d_ph || !dxp || !dxv) {
        rc = -1;
        goto done;
    }
    /* the forward's merged head outputs (attn.rs:259-268) */
    for (int h = 0; h < H; h++) {
        attn_one_head(w, x, t, h, head_out, NULL, NULL, NULL);
        for (int pos = 0; pos < t; pos++)
            memcpy(merged + (size_t)pos * E + (size_t)h * hd, head_out + (size_t)pos * hd, sizeof(float) * hd);
    }
    wo_bwd_out_proj(d_y, merged, w->out_w, E, t, d_out, d_out_w, d_out_b);
    for (int h = 0; h < H; h++) {
        const float raw = w->harmonic_raw[h];
        const float hn = wo_softplus(raw);
        const float sig = 1.0f / (1.0f + expf(-raw));
        const int off = h * hd;
        /* cache of head h: phases, att_w, values, content (attn.rs:121-165) */
        attn_one_head(w, x, t, h, head_out, att_w, NULL, phases);
        for (int pos = 0; pos < t; pos++)
            value_project(x + (size_t)pos * E + off, hd, w->v_w + (size_t)h * hd * hd, w->v_b + h * hd,
                          v_all + (size_t)pos * hd);
        if (C) {
            const float *cw = w->content_w + (size_t)h * C * E, *cb = w->content_b + h * C;
            for (int pos = 0; pos < t; pos++)
                for (int d = 0; d < C; d++) {
                    float sum = cb[d];
                    for (int j = 0; j < E; j++) sum += cw[(size_t)d * E + j] * x[(size_t)pos * E + j];
                    content[(size_t)pos * C + d] = sum;
                }
        }
        const float cscale = C > 0 ? 1.0f / sqrtf((float)C) : 0.0f;
        for (int pos = 0; pos < t; pos++) /* split_heads, attn_backward.rs:56-66 */
            memcpy(d_head + (size_t)pos * hd, d_out + (size_t)pos * E + off, sizeof(float) * hd);
        wo_bwd_value_aggregation(d_head, att_w, v_all, t, hd, d_att, d_v);
        wo_bwd_softmax(d_att, att_w, t, d_sc);
        float d_hn = 0.0f;
        bwd_score(d_sc, phases, hn, att_w, content, C, cscale, t, d_delta, d_c, &d_hn);
        bwd_phase_subtraction(d_delta, att_w, t, d_ph);
        wo_bwd_phase_projection(d_ph, x, w->phase_w + (size_t)h * 2 * E, w->phase_b + h * 2, E, t,
                                dxp + (size_t)h * t * E, d_phase_w + (size_t)h * 2 * E, d_phase_b + h * 2);
        wo_bwd_value_projection(d_v, x, off, hd, E, t, w->v_w + (size_t)h * hd * hd, dxv + (size_t)h * t * E,
                                d_v_w + (size_t)h * hd * hd, d_v_b + h * hd);
        if (C)
            bwd_content_projection(d_c, x, w->content_w + (size_t)h * C * E, C, E, t, dxc + (size_t)h * t * E,
                                   d_content_w + (size_t)h * C * E, d_content_b + h * C);
        d_harmonic_raw[h] = d_hn * sig;
    }
    wo_bwd_combine(dxp, dxv, dxc, H, t, E, d_x);
done:
    free(merged); free(head_out); free(att_w); free(phases); free(v_all); free(content); free(d_out);
    free(d_head); free(d_att); free(d_v); free(d_sc); free(d_delta); free(d_c); free(d_ph); free(dxp); free(dxv);
    free(dxc);
    return rc;
}
