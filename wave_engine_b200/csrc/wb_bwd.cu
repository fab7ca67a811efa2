// wb_bwd.cu -- wave attention backward on the GPU (fp32 SIMT).
//
// wave_attention_backward_full (src/common/attn.rs:346-430) composed of the
// primitives of src/common/math/attn_backward.rs:17-328, for a batch of
// sequences, from the forward cache (WaveAttnCache, attn.rs:51-70: phases,
// (r, s), values, content, softmax weights, merged head outputs) and the
// normed input x:
//   d_out   = d_y W_out                      (out_proj_backward, :17-53)
//   per (sequence, head), with dH the head's slice of d_out:
//     dA[q][k] = dH[q] . V[k]                (value_aggregation_backward, :72-105)
//     dS[q][k] = A[q][k] (dA[q][k] - sum_k' A dA)            (softmax, :109-122)
//     d_phase[q] += -n sin(n d) dS,  d_phase[k] -= -n sin(n d) dS   (score,
//     d_n += -d sin(n d) dS,  d_c[q] += s dS c[k],  d_c[k] += s dS c[q]  :128-184)
//     dV[k]    = sum_q A[q][k] dH[q]
//   (d_r, d_s) through atan2 (:190-231), d_x and the weight gradients of the
//   phase, value and content projections (:237-293), summed over heads
//   (:299-326); d_harmonic_raw = d_n * sigmoid(raw).
// Every sum runs in fp32; only kept pairs (A > 0, k <= q) contribute, as in
// the reference.  Weight gradients are summed over the batch, each output by
// one thread in position order (deterministic).
#include "wb_bwd.h"

#include <algorithm>
#include <cmath>

namespace wb {

// ---- pass 1, one warp per query q of (b, h): dA over the query's kept keys,
// the row sum ws = sum A dA, then dS = A (dA - ws) (into dS) and the query's
// own terms: d_phase[q], d_c[q], the harmonic partial.
struct BwdRowsArgs {
    const float *att_w;   // [BH][T][T]
    const float *v;       // [BH][T][hd]
    const float *phases;  // [BH][T]
    const float *content; // [BH][T][C] or nullptr
    const float *d_out;   // [B*T][E]
    const float *hn;      // [H]
    int B, H, T, hd, C, E;
    float cscale;
    float *dS;            // [BH][T][T]
    float *d_ph;          // [BH][T] query-side phase gradient
    float *d_c;           // [BH][T][C] query-side content gradient
    float *dhn;           // [BH][T] harmonic partial per query
};

static constexpr int BWD_WARPS = 4;

__global__ void __launch_bounds__(BWD_WARPS * 32) bwd_rows_kernel(BwdRowsArgs a) {
    extern __shared__ float bsm[];  // per warp: dH row [hd]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * BWD_WARPS + warp, h = blockIdx.y, b = blockIdx.z;
    if (q >= a.T) return;
    const long long bh = (long long)b * a.H + h;
    const int T = a.T, hd = a.hd, C = a.content ? a.C : 0;
    float *dh = bsm + warp * hd;
    const float *dq = a.d_out + ((long long)b * T + q) * a.E + (long long)h * hd;
    for (int d = lane; d < hd; d += 32) dh[d] = dq[d];
    __syncwarp();
    const float *A = a.att_w + (bh * T + q) * T;
    float *dSq = a.dS + (bh * T + q) * T;
    const float *V = a.v + bh * T * hd;
    // dA and the row sum
    float ws = 0.0f;
    for (int k = lane; k <= q; k += 32) {
        const float ak = A[k];
        float da = 0.0f;
        if (ak > 0.0f) {
            const float *vk = V + (long long)k * hd;
            for (int d = 0; d < hd; d++) da = fmaf(dh[d], vk[d], da);
            ws = fmaf(ak, da, ws);
        }
        dSq[k] = da;
    }
    ws = warp_sum(ws);
    // dS and the query's own terms
    const float n = a.hn[h];
    const float thq = a.phases[bh * T + q];
    const float *cb = C ? a.content + bh * T * C : nullptr;
    float dph = 0.0f, dhn = 0.0f;
    float dcq[16];
#pragma unroll
    for (int cd = 0; cd < 16; cd++) dcq[cd] = 0.0f;
    for (int k = lane; k <= q; k += 32) {
        const float ak = A[k];
        float ds = 0.0f;
        if (ak > 0.0f) {
            ds = ak * (dSq[k] - ws);
            const float delta = thq - a.phases[bh * T + k];
            const float sn = sinf(n * delta);
            dph = fmaf(-sn * n, ds, dph);
            dhn = fmaf(-sn * delta, ds, dhn);
#pragma unroll
            for (int cd = 0; cd < 16; cd++)
                if (cd < C) dcq[cd] = fmaf(ds * a.cscale, cb[(long long)k * C + cd], dcq[cd]);
        }
        dSq[k] = ds;
    }
    dph = warp_sum(dph);
    dhn = warp_sum(dhn);
#pragma unroll
    for (int cd = 0; cd < 16; cd++)
        if (cd < C) dcq[cd] = warp_sum(dcq[cd]);
    if (lane == 0) {
        a.d_ph[bh * T + q] = dph;
        a.dhn[bh * T + q] = dhn;
        for (int cd = 0; cd < C; cd++) a.d_c[(bh * T + q) * C + cd] = dcq[cd];
    }
}

// ---- pass 2, one warp per key p of (b, h): dV[p] = sum_{q >= p} A[q][p] dH[q]
// (lanes along the head dims), and the key-side phase and content terms
// added to pass 1's query-side values.
struct BwdColsArgs {
    const float *att_w, *dS, *phases, *content, *d_out, *hn;
    int B, H, T, hd, C, E;
    float cscale;
    float *d_v;   // [BH][T][hd]
    float *d_ph;  // [BH][T] in: query side, out: total
    float *d_c;   // [BH][T][C] in: query side, out: total
};

__global__ void __launch_bounds__(BWD_WARPS * 32) bwd_cols_kernel(BwdColsArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int p = blockIdx.x * BWD_WARPS + warp, h = blockIdx.y, b = blockIdx.z;
    if (p >= a.T) return;
    const long long bh = (long long)b * a.H + h;
    const int T = a.T, hd = a.hd, C = a.content ? a.C : 0;
    const float n = a.hn[h];
    const float thp = a.phases[bh * T + p];
    const float *cb = C ? a.content + bh * T * C : nullptr;
    float dv[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // dims lane, lane + 32, lane + 64, lane + 96
    float dph = 0.0f, dc = 0.0f;
    for (int q = p; q < T; q++) {
        const float aq = a.att_w[(bh * T + q) * T + p];
        if (!(aq > 0.0f)) continue;
        const float ds = a.dS[(bh * T + q) * T + p];
        const float *dq = a.d_out + ((long long)b * T + q) * a.E + (long long)h * hd;
#pragma unroll
        for (int u = 0; u < 4; u++)
            if (lane + 32 * u < hd) dv[u] = fmaf(aq, dq[lane + 32 * u], dv[u]);
        const float delta = a.phases[bh * T + q] - thp;
        dph = fmaf(sinf(n * delta) * n, ds, dph);  // d_phase[k] -= -n sin(n d) dS
        if (lane < C) dc = fmaf(ds * a.cscale, cb[(long long)q * C + lane], dc);
    }
#pragma unroll
    for (int u = 0; u < 4; u++)
        if (lane + 32 * u < hd) a.d_v[(bh * T + p) * hd + lane + 32 * u] = dv[u];
    if (lane == 0) a.d_ph[bh * T + p] += dph;
    if (lane < C) a.d_c[(bh * T + p) * C + lane] += dc;
}

// ---- (d_r, d_s) through theta = atan2(s, r): attn_backward.rs:190-231.
__global__ void bwd_atan2_kernel(const float *d_ph, const float *rs, long long n, float *coef) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float dp = d_ph[i];
    const float r = rs[2 * i], s = rs[2 * i + 1];
    const float mag_sq = r * r + s * s;
    float dr = 0.0f, dsv = 0.0f;
    if (!(fabsf(dp) < 1e-12f) && !(mag_sq < 1e-8f)) {
        const float mag = fmaxf(mag_sq, 1e-12f);
        dr = dp * (-s / mag);
        dsv = dp * (r / mag);
    }
    coef[2 * i] = dr;
    coef[2 * i + 1] = dsv;
}

// ---- d_x[b][t][j] = sum over heads of the phase, value and content input
// gradients (attn_backward.rs:299-326).
struct BwdDxArgs {
    const float *coef;   // [BH][T][2]
    const float *d_v;    // [BH][T][hd]
    const float *d_c;    // [BH][T][C] or nullptr
    const float *wrs_t;  // [E][H][2]
    const float *wv_t;   // [H][hd(in)][hd(out)]
    const float *wc_t;   // [E][H*C]
    int B, H, T, hd, C, E;
    float *d_x;          // [B*T][E]
};

__global__ void bwd_dx_kernel(BwdDxArgs a) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long R = (long long)a.B * a.T;
    if (i >= R * a.E) return;
    const long long r = i / a.E;
    const int j = (int)(i - r * a.E);
    const int b = (int)(r / a.T), t = (int)(r - (long long)b * a.T);
    const int hj = j / a.hd, jj = j - hj * a.hd;
    float acc = 0.0f;
    for (int h = 0; h < a.H; h++) {
        const long long bht = ((long long)b * a.H + h) * a.T + t;
        float g = a.wrs_t[((long long)j * a.H + h) * 2] * a.coef[2 * bht] +
                  a.wrs_t[((long long)j * a.H + h) * 2 + 1] * a.coef[2 * bht + 1];
        if (h == hj) {
            const float *wv = a.wv_t + ((long long)h * a.hd + jj) * a.hd;
            const float *dv = a.d_v + bht * a.hd;
            float sv = 0.0f;
            for (int dd = 0; dd < a.hd; dd++) sv = fmaf(wv[dd], dv[dd], sv);
            g += sv;
        }
        if (a.d_c) {
            const float *wc = a.wc_t + (long long)j * a.H * a.C + (long long)h * a.C;
            const float *dc = a.d_c + bht * a.C;
            float sc = 0.0f;
            for (int cd = 0; cd < a.C; cd++) sc = fmaf(wc[cd], dc[cd], sc);
            g += sc;
        }
        acc += g;
    }
    a.d_x[i] = acc;
}

// ---- weight gradients: out[o][j] = sum over positions r of
// G(r, o) * X[r][xoff(o) + j], bias[o] = sum_r G(r, o).  G(r, o) is read at
// g[gofs(b, o) + t * gts] with o = (h, k): offsets below per kind.
enum { WG_OUTPROJ = 0, WG_PHASE = 1, WG_VALUE = 2, WG_CONTENT = 3 };
struct BwdWgArgs {
    int kind;
    const float *g;   // gradient source
    const float *X;   // [B*T][ldx]
    int B, H, T, hd, C, E;
    int n_out, n_in;  // output rows, inputs per row
    float *dw;        // [n_out][n_in]
    float *db;        // [n_out] or nullptr
};

__device__ __forceinline__ float wg_g(const BwdWgArgs &a, int b, int t, int o) {
    switch (a.kind) {
    case WG_OUTPROJ:  // d_y [B*T][E], o = output column
        return a.g[((long long)b * a.T + t) * a.E + o];
    case WG_PHASE: {  // coef [BH][T][2], o = h*2 + k
        const int h = o >> 1, k = o & 1;
        return a.g[(((long long)b * a.H + h) * a.T + t) * 2 + k];
    }
    case WG_VALUE: {  // d_v [BH][T][hd], o = h*hd + dd
        const int h = o / a.hd, dd = o - h * a.hd;
        return a.g[(((long long)b * a.H + h) * a.T + t) * a.hd + dd];
    }
    default: {        // d_c [BH][T][C], o = h*C + cd
        const int h = o / a.C, cd = o - h * a.C;
        return a.g[(((long long)b * a.H + h) * a.T + t) * a.C + cd];
    }
    }
}

__global__ void bwd_wgrad_kernel(BwdWgArgs a) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)a.n_out * a.n_in) return;
    const int o = (int)(i / a.n_in), j = (int)(i - (long long)o * a.n_in);
    // input column: the value projection reads its head's slice of x
    const int xcol = a.kind == WG_VALUE ? (o / a.hd) * a.hd + j : j;
    float acc = 0.0f, accb = 0.0f;
    for (int b = 0; b < a.B; b++)
        for (int t = 0; t < a.T; t++) {
            const float gv = wg_g(a, b, t, o);
            acc = fmaf(gv, a.X[((long long)b * a.T + t) * a.E + xcol], acc);
            accb += gv;
        }
    a.dw[i] = acc;
    if (a.db && j == 0) a.db[o] = accb;
}

// ---- d_harmonic_raw[h] = (sum over sequences and queries of the harmonic
// partials) * sigmoid(harmonic_raw[h]).
__global__ void bwd_harmonic_kernel(const float *dhn, const float *raw, int B, int H, int T, float *out) {
    const int h = blockIdx.x;
    float acc = 0.0f;
    for (int b = 0; b < B; b++) {
        const float *p = dhn + ((long long)b * H + h) * T;
        float s = 0.0f;
        for (int t = threadIdx.x; t < T; t += 32) s += p[t];
        acc += warp_sum(s);
    }
    if (threadIdx.x == 0) out[h] = acc * (1.0f / (1.0f + expf(-raw[h])));
}

static int bwd_launch_err(std::string *msg) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("backward launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

size_t attn_backward_scratch_bytes(int B, int H, int T, int hd, int C, int E) {
    Carve c;
    const long long BH = (long long)B * H;
    c.take<float>((size_t)B * T * E);         // d_out
    c.take<float>((size_t)BH * T * T);        // dS
    c.take<float>((size_t)BH * T);            // d_ph
    c.take<float>((size_t)BH * T * (C ? C : 1));  // d_c
    c.take<float>((size_t)BH * T);            // dhn
    c.take<float>((size_t)BH * T * hd);       // d_v
    c.take<float>((size_t)BH * T * 2);        // coef
    return c.off;
}

int attn_backward(const BwdLayer &w, const BwdCache &cache, const float *x, const float *d_y, int B, int T,
                  float *d_x, const BwdGrads &g, void *scratch, cudaStream_t st, std::string *msg) {
    const int H = w.H, hd = w.hd, E = w.E, C = cache.content ? w.C : 0;
    if (hd > 128) {
        *msg = "the backward supports head_dim <= 128";
        return WB_ENOTSUP;
    }
    const long long BH = (long long)B * H, R = (long long)B * T;
    Carve c;
    char *s = (char *)scratch;
    float *d_out = (float *)(s + c.take<float>((size_t)R * E));
    float *dS = (float *)(s + c.take<float>((size_t)BH * T * T));
    float *d_ph = (float *)(s + c.take<float>((size_t)BH * T));
    float *d_c = (float *)(s + c.take<float>((size_t)BH * T * (C ? C : 1)));
    float *dhn = (float *)(s + c.take<float>((size_t)BH * T));
    float *d_v = (float *)(s + c.take<float>((size_t)BH * T * hd));
    float *coef = (float *)(s + c.take<float>((size_t)BH * T * 2));
    const float cscale = C ? 1.0f / std::sqrt((float)C) : 0.0f;
    ProfScope ps("attn_bwd", st);
    // d_out = d_y W_out (out_proj_backward): Wt = W_out [out][in] row-major
    OutMap om{OUT_DENSE, d_out, E, WbSeqView{}, 0, T};
    launch_seqdot(d_y, (int)R, E, E, w.w_out, E, nullptr, 0, om, st);
    dim3 grid((T + BWD_WARPS - 1) / BWD_WARPS, H, B);
    BwdRowsArgs ra{cache.att_w, cache.v_all, cache.phases, C ? cache.content : nullptr, d_out, w.hn,
                   B, H, T, hd, C, E, cscale, dS, d_ph, d_c, dhn};
    bwd_rows_kernel<<<grid, BWD_WARPS * 32, BWD_WARPS * hd * sizeof(float), st>>>(ra);
    BwdColsArgs ca{cache.att_w, dS, cache.phases, C ? cache.content : nullptr, d_out, w.hn,
                   B, H, T, hd, C, E, cscale, d_v, d_ph, d_c};
    bwd_cols_kernel<<<grid, BWD_WARPS * 32, 0, st>>>(ca);
    const long long nrs = BH * T;
    bwd_atan2_kernel<<<(unsigned)((nrs + 255) / 256), 256, 0, st>>>(d_ph, cache.phase_rs, nrs, coef);
    BwdDxArgs xa{coef, d_v, C ? d_c : nullptr, w.wrs_t, w.wv_t, w.wc_t, B, H, T, hd, C, E, d_x};
    bwd_dx_kernel<<<(unsigned)((R * E + 255) / 256), 256, 0, st>>>(xa);
    auto wgrad = [&](int kind, const float *gsrc, const float *X, int n_out, int n_in, float *dw, float *db) {
        if (!dw) return;
        BwdWgArgs wa{kind, gsrc, X, B, H, T, hd, C, E, n_out, n_in, dw, db};
        const long long n = (long long)n_out * n_in;
        bwd_wgrad_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(wa);
    };
    wgrad(WG_OUTPROJ, d_y, cache.out_merged, E, E, g.out_proj_w, g.out_proj_b);
    wgrad(WG_PHASE, coef, x, 2 * H, E, g.phase_proj_w, g.phase_proj_b);
    wgrad(WG_VALUE, d_v, x, H * hd, hd, g.v_proj_w, g.v_proj_b);
    if (C) wgrad(WG_CONTENT, d_c, x, H * C, E, g.content_proj_w, g.content_proj_b);
    if (g.harmonic_raw) bwd_harmonic_kernel<<<H, 32, 0, st>>>(dhn, w.raw, B, H, T, g.harmonic_raw);
    return bwd_launch_err(msg);
}

}  // namespace wb

namespace wb {

__global__ void rows_to_heads_kernel(const float *src, int B, int T, int H, int K, float *dst) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    const long long n = (long long)B * T * H * K;
    if (i >= n) return;
    const int k = (int)(i % K);
    long long r = i / K;
    const int h = (int)(r % H);
    r /= H;
    const int t = (int)(r % T);
    const int b = (int)(r / T);
    dst[(((long long)b * H + h) * T + t) * K + k] = src[i];
}

void launch_rows_to_heads(const float *src, int B, int T, int H, int K, float *dst, cudaStream_t st) {
    const long long n = (long long)B * T * H * K;
    if (n <= 0) return;
    rows_to_heads_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(src, B, T, H, K, dst);
}

}  // namespace wb
