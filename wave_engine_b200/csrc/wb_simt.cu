// wb_simt.cu -- all-fp32 SIMT kernels (WB_PATH_EXACT).
//
// These follow the reference's operation order statement by statement:
// products rounded before the add (__fmul_rn/__fadd_rn, no FMA contraction),
// dot products summed sequentially over the input index, biases added where
// the reference adds them.  They are the correctness variant of the path and
// also produce the phases/buckets/values the KV cache stores.
#include "wb_internal.h"

#include <algorithm>

namespace wb {

// ---------------------------------------------------------------------------
// Sequential-dot linear layer over a tile of rows:
//   Y[r][n] = bias_first ? ((b[n] + W[n][0]x0) + W[n][1]x1) + ...
//                        : (((0 + W[n][0]x0) + ...) + b[n])
// with Wt = W transposed ([K][N]) so that consecutive threads read
// consecutive outputs.  The first form is the reference's phase/content
// projection (attn.rs:124-126, :141-144), the second its value projection
// (attn.rs:157-162) and out_proj (attn.rs:279-281).
// ---------------------------------------------------------------------------
template <int TOK>
__global__ void __launch_bounds__(256) seqdot_kernel(const float *__restrict__ X, int R, int K,
                                                     long long ldx, const float *__restrict__ Wt,
                                                     int N, const float *__restrict__ bias,
                                                     int bias_first, OutMap om) {
    extern __shared__ float xs[];  // [TOK][K]
    const int r0 = blockIdx.x * TOK;
    const int nrow = min(TOK, R - r0);
    for (int i = threadIdx.x; i < TOK * K; i += blockDim.x) {
        int t = i / K, j = i - t * K;
        xs[i] = t < nrow ? X[(long long)(r0 + t) * ldx + j] : 0.0f;
    }
    __syncthreads();
    for (int n = threadIdx.x; n < N; n += blockDim.x) {
        float acc[TOK];
        const float b0 = bias ? bias[n] : 0.0f;
#pragma unroll
        for (int t = 0; t < TOK; t++) acc[t] = bias_first ? b0 : 0.0f;
        for (int j = 0; j < K; j++) {
            const float w = __ldg(Wt + (long long)j * N + n);
#pragma unroll
            for (int t = 0; t < TOK; t++) acc[t] = __fadd_rn(acc[t], __fmul_rn(w, xs[t * K + j]));
        }
#pragma unroll
        for (int t = 0; t < TOK; t++) {
            if (t >= nrow) break;
            float v = bias_first ? acc[t] : __fadd_rn(acc[t], b0);
            const int r = r0 + t;
            if (om.mode == OUT_DENSE) {
                om.y[(long long)r * om.ldy + n] = v;
            } else {  // OUT_SEQ_V: value row of head om.h into the sequence view
                const int b = r / om.T, tt = r - b * om.T;
                const long long pos = wb_pos(om.sv, b, om.h, tt);
                if (pos >= 0) om.sv.v[pos * N + n] = v;
            }
        }
    }
}

void launch_seqdot(const float *X, int R, int K, long long ldx, const float *Wt, int N,
                   const float *bias, int bias_first, const OutMap &om, cudaStream_t st) {
    if (R <= 0 || N <= 0) return;
    ProfScope ps("proj_seqdot", st);
    const size_t smem32 = (size_t)32 * K * sizeof(float);
    if (smem32 <= 160 * 1024 && R >= 64) {
        cudaFuncSetAttribute(seqdot_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem32);
        seqdot_kernel<32><<<(R + 31) / 32, 256, smem32, st>>>(X, R, K, ldx, Wt, N, bias, bias_first, om);
    } else {
        const size_t smem4 = (size_t)4 * K * sizeof(float);
        cudaFuncSetAttribute(seqdot_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem4);
        seqdot_kernel<4><<<(R + 3) / 4, 256, smem4, st>>>(X, R, K, ldx, Wt, N, bias, bias_first, om);
    }
}

// ---------------------------------------------------------------------------
// (r, s) -> theta = atan2f(s, r) and bucket (attn.rs:127, :171-174).
// rs is [R][H][2]; row r = b*T + t.
// ---------------------------------------------------------------------------
__global__ void phase_kernel(const float *__restrict__ rs, int R, int H, int T, WbSeqView sv) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= R * H) return;
    const int r = i / H, h = i - r * H;
    const float rr = rs[(long long)i * 2], ss = rs[(long long)i * 2 + 1];
    const float th = atan2f(ss, rr);
    const int b = r / T, t = r - b * T;
    const long long pos = wb_pos(sv, b, h, t);
    if (pos < 0) return;
    sv.theta[pos] = th;
    sv.bucket[pos] = (uint8_t)phase_to_bucket(th);
}

void launch_phase(const float *rs, int R, int H, int T, const WbSeqView &sv, cudaStream_t st) {
    const int n = R * H;
    if (n <= 0) return;
    ProfScope ps("phase", st);
    phase_kernel<<<(n + 255) / 256, 256, 0, st>>>(rs, R, H, T, sv);
}

// ---------------------------------------------------------------------------
// Literal prefill attention, one warp per (batch, head, query):
// src/common/attn.rs:185-249 (and kv_cache.rs:146-181 with use_content = 0).
// Three passes over the causal keys: max, exp-sum, normalised PV.
// ---------------------------------------------------------------------------
struct AttnSimtArgs {
    WbSeqView sv;
    const float *content;  // [B*T][H*C] or nullptr
    int C;
    float content_scale;
    const float *harmonic_n;  // [H]
    int B, H, T, hd;
    void *o;         // [B*T][H*hd] merged heads (float or bf16)
    float *att_w;    // [B][H][T][T] or nullptr
    const int *tile_list;   // [0] = n, [1..n] = flagged query tiles b*Hg*n_qt + (h-h0)*n_qt + qt (nullptr = all)
    int h0, Hg;             // tile mode: heads h0 .. h0 + Hg - 1 (rows bh = b * Hg + h - h0)
};

__device__ __forceinline__ void store_out(float *p, float v) { *p = v; }
__device__ __forceinline__ void store_out(__nv_bfloat16 *p, float v) { *p = __float2bfloat16_rn(v); }

template <int DPL, class OutT>  // head dims per lane (hd <= 32*DPL)
__device__ void attn_simt_query(const AttnSimtArgs &a, int b, int h, int q);

// One warp per query (8 queries per CTA).
template <int DPL, class OutT>
__global__ void __launch_bounds__(256) attn_simt_kernel(AttnSimtArgs a) {
    const int warp = threadIdx.x >> 5;
    const int q = blockIdx.x * 8 + warp;
    if (q >= a.T) return;
    attn_simt_query<DPL, OutT>(a, blockIdx.z, blockIdx.y, q);
}

// Fallback over the flagged 128-query tiles listed by the tensor-core
// kernel: a small fixed grid walks the list (CTA i takes entries i,
// i + gridDim.x, ...), its 8 warps looping over a tile's queries.  With no
// flagged tile every CTA reads the count and exits.
template <int DPL, class OutT>
__global__ void __launch_bounds__(256) attn_simt_tiles_kernel(AttnSimtArgs a) {
    const int n_qt = (a.T + 127) / 128;
    const int n = a.tile_list[0];
    const int warp = threadIdx.x >> 5;
    for (int e = blockIdx.x; e < n; e += gridDim.x) {
        const int t = a.tile_list[1 + e];
        const int tile = t % n_qt, bh = t / n_qt;
        const int b = bh / a.Hg, h = a.h0 + (bh - b * a.Hg);
        for (int q = tile * 128 + warp; q < min(a.T, tile * 128 + 128); q += 8) attn_simt_query<DPL, OutT>(a, b, h, q);
    }
}

template <int DPL, class OutT>
__device__ void attn_simt_query(const AttnSimtArgs &a, int b, int h, int q) {
    const int lane = threadIdx.x & 31;
    // key k of (b, h) at index at(k): contiguous, or through the page table
    const bool paged = a.sv.pages != nullptr;
    const long long base = paged ? 0 : wb_slot_base(a.sv, b, h);
    auto at = [&](int k) -> long long { return paged ? wb_pos(a.sv, b, h, k) : base + k; };
    const float *theta = a.sv.theta;
    const uint8_t *bucket = a.sv.bucket;
    const float *V = a.sv.v;
    const float hn = a.harmonic_n[h];
    const long long iq = at(q);
    if (iq < 0) return;  // unmapped page: nothing to attend from
    const float thq = theta[iq];
    const uint32_t amask = allowed_bucket_mask(bucket[iq]);
    const int C = a.C;
    const long long HC = (long long)a.H * C;
    const float *cq_ptr = C ? a.content + ((long long)b * a.T + q) * HC + (long long)h * C : nullptr;
    float cq[16];
#pragma unroll
    for (int d = 0; d < 16; d++) cq[d] = (d < C) ? cq_ptr[d] : 0.0f;

    auto score = [&](int k) -> float {
        if (k > q) return -INFINITY;
        const long long ik = at(k);
        if (ik < 0) return -INFINITY;
        const bool ok = ((amask >> bucket[ik]) & 1u) || k == q - 1;
        if (!ok) return -INFINITY;
        float s = cosf(__fmul_rn(hn, __fsub_rn(thq, theta[ik])));
        if (C) {
            const float *ck = a.content + ((long long)b * a.T + k) * HC + (long long)h * C;
            float dot = 0.0f;
#pragma unroll
            for (int d = 0; d < 16; d++)
                if (d < C) dot = __fadd_rn(dot, __fmul_rn(cq[d], ck[d]));
            s = __fadd_rn(s, __fmul_rn(dot, a.content_scale));
        }
        return s;
    };

    float m = -INFINITY;
    for (int k = lane; k <= q; k += 32) m = fmaxf(m, score(k));
    m = warp_max(m);
    float es = 0.0f;
    for (int k = lane; k <= q; k += 32) {
        float s = score(k);
        if (s > -INFINITY) es = __fadd_rn(es, expf(__fsub_rn(s, m)));
    }
    es = warp_sum(es);

    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; i++) acc[i] = 0.0f;
    float *aw = a.att_w ? a.att_w + (((long long)b * a.H + h) * a.T + q) * a.T : nullptr;
    for (int k0 = 0; k0 <= q; k0 += 32) {
        const int k = k0 + lane;
        float p = 0.0f;
        if (k <= q) {
            float s = score(k);
            if (s > -INFINITY) {
                p = expf(__fsub_rn(s, m));
                if (es > 0.0f) p = __fdiv_rn(p, es);
            }
            if (aw) aw[k] = p;
        }
        const int nk = min(32, q - k0 + 1);
        for (int j = 0; j < nk; j++) {
            const float pj = __shfl_sync(0xffffffffu, p, j);
            if (pj > 0.0f) {  // p > 0 only for mapped keys
                const float *vr = V + at(k0 + j) * a.hd;
#pragma unroll
                for (int i = 0; i < DPL; i++) {
                    const int dd = lane + 32 * i;
                    if (dd < a.hd) acc[i] = __fadd_rn(acc[i], __fmul_rn(pj, vr[dd]));
                }
            }
        }
    }
    if (aw)
        for (int k = q + 1 + lane; k < a.T; k += 32) aw[k] = -INFINITY;
    OutT *orow = (OutT *)a.o + ((long long)b * a.T + q) * ((long long)a.H * a.hd) + (long long)h * a.hd;
#pragma unroll
    for (int i = 0; i < DPL; i++) {
        const int dd = lane + 32 * i;
        if (dd < a.hd) store_out(orow + dd, acc[i]);
    }
}

template <class OutT>
static void launch_attn_simt_t(const AttnSimtArgs &a, cudaStream_t st) {
    ProfScope ps(a.tile_list ? "attn_simt_fallback" : "attn_simt", st);
    if (a.tile_list) {
        const unsigned grid = (unsigned)std::min<long long>(256, (long long)a.B * a.Hg * ((a.T + 127) / 128));
        if (a.hd <= 32) attn_simt_tiles_kernel<1, OutT><<<grid, 256, 0, st>>>(a);
        else if (a.hd <= 64) attn_simt_tiles_kernel<2, OutT><<<grid, 256, 0, st>>>(a);
        else if (a.hd <= 128) attn_simt_tiles_kernel<4, OutT><<<grid, 256, 0, st>>>(a);
        else attn_simt_tiles_kernel<8, OutT><<<grid, 256, 0, st>>>(a);
        return;
    }
    dim3 grid((a.T + 7) / 8, a.H, a.B);
    if (a.hd <= 32) attn_simt_kernel<1, OutT><<<grid, 256, 0, st>>>(a);
    else if (a.hd <= 64) attn_simt_kernel<2, OutT><<<grid, 256, 0, st>>>(a);
    else if (a.hd <= 128) attn_simt_kernel<4, OutT><<<grid, 256, 0, st>>>(a);
    else attn_simt_kernel<8, OutT><<<grid, 256, 0, st>>>(a);
}

void launch_attn_simt(const WbSeqView &sv, const float *content, int C, float content_scale,
                      const float *harmonic_n, int B, int H, int T, int hd, float *o,
                      float *att_w, cudaStream_t st) {
    AttnSimtArgs a{sv, content, C, content_scale, harmonic_n, B, H, T, hd, o, att_w, nullptr, 0, H};
    launch_attn_simt_t<float>(a, st);
}

void launch_attn_simt_fallback_bf16(const WbSeqView &sv, const float *content, int C, float content_scale,
                                    const float *harmonic_n, int B, int H, int T, int hd, __nv_bfloat16 *o,
                                    const int *tile_list, int h0, int Hg, cudaStream_t st) {
    AttnSimtArgs a{sv, content, C, content_scale, harmonic_n, B, H, T, hd, o, nullptr, tile_list, h0, Hg};
    launch_attn_simt_t<__nv_bfloat16>(a, st);
}

void launch_attn_simt_fallback_f32(const WbSeqView &sv, const float *content, int C, float content_scale,
                                   const float *harmonic_n, int B, int H, int T, int hd, float *o,
                                   const int *tile_list, int h0, int Hg, cudaStream_t st) {
    AttnSimtArgs a{sv, content, C, content_scale, harmonic_n, B, H, T, hd, o, nullptr, tile_list, h0, Hg};
    launch_attn_simt_t<float>(a, st);
}

void launch_projections_exact(const ProjWeights &w, const float *x, int B, int T, const WbSeqView &sv, float *rs,
                              float *content, cudaStream_t st) {
    const int R = B * T, E = w.E, H = w.H, hd = w.hd;
    OutMap dense{OUT_DENSE, rs, 2LL * H, sv, 0, T};
    launch_seqdot(x, R, E, E, w.wrs_t, 2 * H, w.brs, 1, dense, st);
    launch_phase(rs, R, H, T, sv, st);
    if (content) {
        OutMap cm{OUT_DENSE, content, (long long)H * w.C, sv, 0, T};
        launch_seqdot(x, R, E, E, w.wc_t, H * w.C, w.bc, 1, cm, st);
    }
    for (int h = 0; h < H; h++) {
        OutMap vm{OUT_SEQ_V, nullptr, 0, sv, h, T};
        launch_seqdot(x + (size_t)h * hd, R, hd, E, w.wv_t + (size_t)h * hd * hd, hd, w.bv + (size_t)h * hd, 0,
                      vm, st);
    }
}

// ---------------------------------------------------------------------------
// Literal decode attention, one warp per (sequence, head):
// src/common/kv_cache.rs:280-326.  Reads the slot's n cached entries, scores
// the new position's phase against keys in buckets b-1..b+1 plus the
// previous position, self score 1.0, softmax over n+1 entries, PV in key
// order then the self value, and appends (phase, bucket, value) at index n.
// ---------------------------------------------------------------------------
struct DecodeSimtArgs {
    WbSeqView sv;            // cache view of this layer (slot = seq_ids)
    const int32_t *len;      // [slots] cached positions of this layer
    const float *theta_new;  // [n_seq][H]
    const float *v_new;      // [n_seq][H][hd]
    const float *harmonic_n;
    int n_seq, H, hd;
    float *o;                // [n_seq][H*hd]
    uint32_t *dev_err;       // WB_DERR_BOUNDS: the appended position's page is unmapped
};

template <int DPL>
__global__ void __launch_bounds__(128) decode_simt_kernel(DecodeSimtArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x * 4 + warp, i = blockIdx.y;
    if (h >= a.H) return;
    const int slot = a.sv.slot ? a.sv.slot[i] : i;
    const int n = a.len[slot];
    // key k at index at(k): contiguous, or through the page table (the
    // caller reserved pages for every cached key and the appended one)
    const bool paged = a.sv.pages != nullptr;
    const long long base = paged ? 0 : wb_slot_base(a.sv, i, h);
    auto at = [&](int k) -> long long { return paged ? wb_pos(a.sv, i, h, k) : base + k; };
    const long long inew = (n < 0 || (!paged && n >= a.sv.cap)) ? -1 : at(n);
    if (inew < 0) {
        if (lane == 0) atomicOr(a.dev_err, WB_DERR_BOUNDS);
        return;
    }
    const float *theta = a.sv.theta;
    const uint8_t *bucket = a.sv.bucket;
    const float *V = a.sv.v;
    const float hn = a.harmonic_n[h];
    const float ph = a.theta_new[(long long)i * a.H + h];
    const int qb = phase_to_bucket(ph);
    const uint32_t amask = allowed_bucket_mask(qb);
    const float *vnew = a.v_new + ((long long)i * a.H + h) * a.hd;

    auto score = [&](int k) -> float {  // k < n
        const long long ik = at(k);
        const bool ok = ((amask >> bucket[ik]) & 1u) || k == n - 1;
        return ok ? cosf(__fmul_rn(hn, __fsub_rn(ph, theta[ik]))) : -INFINITY;
    };
    float m = (lane == 0) ? 1.0f : -INFINITY;  // self score (kv_cache.rs:294)
    for (int k = lane; k < n; k += 32) m = fmaxf(m, score(k));
    m = warp_max(m);
    float es = 0.0f;
    for (int k = lane; k < n; k += 32) {
        float s = score(k);
        if (s > -INFINITY) es = __fadd_rn(es, expf(__fsub_rn(s, m)));
    }
    es = warp_sum(es);
    const float e_self = expf(__fsub_rn(1.0f, m));
    es = __fadd_rn(es, e_self);

    float acc[DPL];
#pragma unroll
    for (int j = 0; j < DPL; j++) acc[j] = 0.0f;
    for (int k0 = 0; k0 < n; k0 += 32) {
        const int k = k0 + lane;
        float p = 0.0f;
        if (k < n) {
            float s = score(k);
            if (s > -INFINITY) p = __fdiv_rn(expf(__fsub_rn(s, m)), es);
        }
        const int nk = min(32, n - k0);
        for (int j = 0; j < nk; j++) {
            const float pj = __shfl_sync(0xffffffffu, p, j);
            if (pj > 0.0f) {
                const float *vr = V + at(k0 + j) * a.hd;
#pragma unroll
                for (int u = 0; u < DPL; u++) {
                    const int dd = lane + 32 * u;
                    if (dd < a.hd) acc[u] = __fadd_rn(acc[u], __fmul_rn(pj, vr[dd]));
                }
            }
        }
    }
    const float p_self = __fdiv_rn(e_self, es);
    float *orow = a.o + (long long)i * a.H * a.hd + (long long)h * a.hd;
    float *vdst = a.sv.v + inew * a.hd;
#pragma unroll
    for (int u = 0; u < DPL; u++) {
        const int dd = lane + 32 * u;
        if (dd < a.hd) {
            orow[dd] = __fadd_rn(acc[u], __fmul_rn(p_self, vnew[dd]));
            vdst[dd] = vnew[dd];
        }
    }
    if (lane == 0) {
        a.sv.theta[inew] = ph;
        a.sv.bucket[inew] = (uint8_t)qb;
    }
}

void launch_decode_simt(const WbSeqView &sv, const int32_t *len, const float *theta_new,
                        const float *v_new, const float *harmonic_n, int n_seq, int H, int hd,
                        float *o, uint32_t *dev_err, cudaStream_t st) {
    DecodeSimtArgs a{sv, len, theta_new, v_new, harmonic_n, n_seq, H, hd, o, dev_err};
    dim3 grid((H + 3) / 4, n_seq);
    ProfScope ps("decode_simt", st);
    if (hd <= 32) decode_simt_kernel<1><<<grid, 128, 0, st>>>(a);
    else if (hd <= 64) decode_simt_kernel<2><<<grid, 128, 0, st>>>(a);
    else if (hd <= 128) decode_simt_kernel<4><<<grid, 128, 0, st>>>(a);
    else decode_simt_kernel<8><<<grid, 128, 0, st>>>(a);
}

// theta_new only (no cache write): rs [n][H][2] -> theta [n][H].
__global__ void theta_only_kernel(const float *__restrict__ rs, int n, float *theta) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) theta[i] = atan2f(rs[2LL * i + 1], rs[2LL * i]);
}
void launch_theta_only(const float *rs, int n, float *theta, cudaStream_t st) {
    if (n > 0) theta_only_kernel<<<(n + 255) / 256, 256, 0, st>>>(rs, n, theta);
}

// len[slot(i)] += delta (set = 0) or = value (set = 1) for each listed sequence.
// len[slot] = value (set) or len[slot] += value, for slots inside [0,
// n_slots); an increment stops at cap (a full cache was flagged already).
__global__ void len_update_kernel(int32_t *len, const int32_t *slots, int n_seq, int value, int set, int n_slots,
                                  int cap, const int32_t *pages, int max_pages) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_seq) return;
    const int s = slots ? slots[i] : i;
    if (s < 0 || s >= n_slots) return;
    // a paged slot never grows past its reserved pages (those writes were skipped)
    if (set) {
        if (value == 0 || wb_pos_mapped(pages, max_pages, s, value - 1)) len[s] = value;
    } else if (len[s] < cap && wb_pos_mapped(pages, max_pages, s, len[s] + value - 1)) {
        len[s] = min(cap, len[s] + value);
    }
}
void launch_len_update(int32_t *len, const int32_t *slots, int n_seq, int value, int set, int n_slots, int cap,
                       cudaStream_t st, const int32_t *pages, int max_pages) {
    if (n_seq > 0)
        len_update_kernel<<<(n_seq + 127) / 128, 128, 0, st>>>(len, slots, n_seq, value, set, n_slots, cap, pages,
                                                               max_pages);
}

// n floats from pinned host memory (its device alias) to device memory, 16
// bytes per load: one pass over the bus without a copy-engine transfer,
// whose fixed cost dominates the few KB of a decode step's inputs.
__global__ void copy_f4_kernel(const float4 *__restrict__ src, float4 *__restrict__ dst, long long n4) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x)
        dst[i] = src[i];
}
void launch_copy_f4(const float *src, float *dst, long long n, cudaStream_t st) {
    const long long n4 = n / 4;
    if (n4 <= 0) return;
    const int grid = (int)std::min<long long>(148, (n4 + 255) / 256);
    copy_f4_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const float4 *>(src), reinterpret_cast<float4 *>(dst), n4);
}

// Bucket derivation for wb_kv_cache_load: bucket[i] = phase_to_bucket(theta[i]).
__global__ void bucket_from_theta_kernel(const float *theta, uint8_t *bucket, long long n) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i < n) bucket[i] = (uint8_t)phase_to_bucket(theta[i]);
}
void launch_bucket_from_theta(const float *theta, uint8_t *bucket, long long n, cudaStream_t st) {
    if (n > 0) bucket_from_theta_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(theta, bucket, n);
}

}  // namespace wb
