// wb_tc.cu -- WB_PATH_TENSOR: tcgen05 tensor-core prefill attention.
//
// Wave attention scores are cos(n*(theta_q - theta_k)) + c_q.c_k/4 over
// keys whose phase bucket is within one of the query's (src/common/attn.rs
// :185-224).  By cos(a-b) = cos a cos b + sin a sin b the score is a dot
// product of two feature rows, so S = Qf Kf^T runs on tcgen05.  Feature
// columns (bf16):
//
//   FW = 16 (no content: the serve prefill, --freeze-ode):
//     0..5    cos/sin(n theta) as a bf16 hi/lo split:
//             Q = [cH, cL, cH, sH, sL, sH], K = [cH, cH, cL, sH, sH, sL]
//             (products hi*hi + lo*hi + hi*lo: ~2^-16 relative error)
//     6..13   bucket mask: Q = 0 for the 3 allowed buckets, -512 for the
//             other 5; K = one-hot of the key's bucket.  A masked key's
//             score is pushed to about -512 and its exp is 0.
//     14..15  zero
//   FW = 64 (content): cos/sin at 0..5, content as hi/lo triples
//     (Q = [qH, qL, qH] of c_q/4, K = [kH, kH, kL] of c_k) at 6..53, bucket
//     mask at 54..61, zero at 62..63.
//
// Values enter PV as a bf16 hi + lo pair (two MMAs into one fp32
// accumulator), the merged output is fp32 and out_proj is tf32.  Single
// bf16 features/values exceed a 2e-3 max-abs error with the reference's own
// uniform init (src/common/wave_model.rs:39-46) at every model size.
//
// Softmax needs no running max: every score is bounded by
// 1 + |c_q| max_k|c_k| / 4 and the self score 1 + |c_q|^2/4 is always
// present, so exp(s - s_self) neither overflows nor loses the row as long
// as |c_q| (max|c_k| - |c_q|) / 4 <= 64.  Query tiles where that bound fails
// are listed and recomputed by the fp32 SIMT kernel.  The reference's
// "always score the previous position" rule (attn.rs:212-221) is a single
// extra term per query, added exactly in the epilogue when the previous
// key is bucket-masked.
#include "wb_ptx.cuh"
#include "wb_tc.h"
#include "wb_decode.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>

namespace wb {

static constexpr int QT = 128;      // queries per work item (TMEM lanes)
static constexpr int KT = 128;      // keys per tile
static constexpr float MASK_BIAS = -512.0f;
// P and the values enter the PV products in fp16 (11-bit significand: P and
// a value each carry a relative rounding error of at most 2^-11, 8x finer
// than bf16), so P = exp(s - shift) must stay below fp16's 65504: a tile
// whose scores may exceed the fixed shift by more than this goes to the fp32
// fallback
static constexpr float BOUND_LIMIT = 10.0f;
// Dot-product attention: the a-priori bound only keeps the fp32 exponentials
// finite; whether a probability fits fp16 is checked per key tile at run time
// (a thread's 64 probabilities of one tile summing past DOT_P_TILE_SUM, fp16's
// largest finite value -- the only way one of them can exceed it -- sends the
// query tile to the fp32 fallback).
static constexpr float DOT_BOUND_LIMIT = 60.0f;
static constexpr float DOT_P_TILE_SUM = 65504.0f;

// ---------------------------------------------------------------------------
// Tensor maps (driver entry point fetched at run time; no libcuda link).
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
        else
            cudaGetLastError();
    }
    return fn;
}

static int make_tmap(CUtensorMap *m, const void *base, CUtensorMapDataType dt, int rank, const uint64_t *dims,
                     const uint64_t *strides, const uint32_t *box, CUtensorMapSwizzle sw, std::string *msg) {
    auto fn = encode_fn();
    if (!fn) {
        *msg = "cuTensorMapEncodeTiled unavailable";
        return WB_ECUDA;
    }
    uint32_t estr[5] = {1, 1, 1, 1, 1};
    CUresult r = fn(m, dt, rank, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *msg = "cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r);
        return WB_ECUDA;
    }
    return WB_OK;
}

// ---------------------------------------------------------------------------
// Feature pre-pass.
// ---------------------------------------------------------------------------
struct FeatArgs {
    WbSeqView sv;
    const float *content;  // [B*T][H*C] or nullptr
    int C;
    float cscale;
    const float *hn;
    int B, H, T, hd, hdp;
    int Hg, h0;                   // heads computed: h0 .. h0 + Hg - 1 (rows bh = b * Hg + (h - h0))
    __nv_bfloat16 *qf, *kf;       // [BH][T][FW]
    __half *vh;                   // [BH][T][hdp] values (fp16)
    float *m0, *sprev, *cnorm;    // [BH][T]
    unsigned int *cmax;           // [BH], float bits
};

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ float f16_round(float x) { return __half2float(__float2half_rn(x)); }

// Features of the attention core, one warp per 32 consecutive rows
// i = bh * T + t (8 warps per CTA).  Lane l owns row i0 + l for the per-row
// quantities (phase, bucket, content, self score, previous-position term);
// its Q and K feature rows (FW bf16 each) are built in a per-warp shared
// buffer (rows padded by one word: conflict-free) and leave as one
// contiguous block of 32 rows (lanes along the words).  Value rows are
// converted with the lanes along the row (8 rows of loads in flight).  The
// previous position's phase, bucket and content come from the neighbouring
// lane (lane 0 loads them).
static constexpr int FEAT_WARPS = 8;

template <int FW>
__global__ void __launch_bounds__(FEAT_WARPS * 32) feat_kernel(FeatArgs a) {
    static_assert(FW == 16 || FW == 64, "feature width 16 (no content) or 64 (content)");
    constexpr int BB = FW == 64 ? 54 : 6;     // first bucket column
    constexpr int FWW = FW / 2;               // 32-bit words per feature row
    constexpr int RS = FWW + 1;               // padded row stride (words)
    constexpr int NC = FW == 64 ? 16 : 0;     // content dims carried
    __shared__ uint32_t fbuf[FEAT_WARPS][32 * RS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long BH = (long long)a.B * a.Hg, total = BH * a.T;
    const long long i0 = ((long long)blockIdx.x * FEAT_WARPS + warp) * 32;
    if (i0 >= total) return;
    const long long i = i0 + lane;
    const bool live = i < total;
    const long long ii = live ? i : total - 1;
    const int bh = (int)(ii / a.T), t = (int)(ii - (long long)bh * a.T);
    const int b = bh / a.Hg, h = a.h0 + (bh - b * a.Hg);
    // cache index of this row (an unmapped page -- never reserved by the
    // caller -- reads index 0 instead of faulting)
    const long long it = max(0LL, wb_pos(a.sv, b, h, t));
    const float th = a.sv.theta[it];
    const int bk = a.sv.bucket[it];
    const float n = a.hn[h];
    const int C = (NC && a.content) ? a.C : 0;
    float c[NC > 0 ? NC : 1];
    {
        const float *cr = C ? a.content + ((long long)b * a.T + t) * ((long long)a.H * C) + (long long)h * C : nullptr;
#pragma unroll
        for (int d = 0; d < NC; d++) c[d] = (d < C) ? cr[d] : 0.0f;
    }
    float c2 = 0.0f;
#pragma unroll
    for (int d = 0; d < NC; d++) c2 = fmaf(c[d], c[d], c2);
    float sn, cs;
    sincosf(n * th, &sn, &cs);
    const float csh = bf16_round(cs), snh = bf16_round(sn);
    const float csl = cs - csh, snl = sn - snh;
    const uint32_t allow = allowed_bucket_mask(bk);

    // ---- Q and K feature rows through the warp's buffer
    uint32_t *fb = fbuf[warp];
    auto emit = [&](__nv_bfloat16 *dst) {
        __syncwarp();
        const long long words = min(32LL, total - i0) * FWW;
        uint32_t *g = reinterpret_cast<uint32_t *>(dst + i0 * FW);
        for (int w = lane; w < words; w += 32) g[w] = fb[(w / FWW) * RS + (w % FWW)];
        __syncwarp();
    };
    {
        uint32_t *row = fb + lane * RS;
        float q[FW];
#pragma unroll
        for (int u = 0; u < FW; u++) q[u] = 0.0f;
        q[0] = csh; q[1] = csl; q[2] = csh; q[3] = snh; q[4] = snl; q[5] = snh;
#pragma unroll
        for (int d = 0; d < NC; d++) {
            const float cq = c[d] * a.cscale;
            const float qh = bf16_round(cq);
            q[6 + 3 * d] = qh; q[7 + 3 * d] = cq - qh; q[8 + 3 * d] = qh;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) q[BB + u] = ((allow >> u) & 1u) ? 0.0f : MASK_BIAS;
#pragma unroll
        for (int w = 0; w < FWW; w++) row[w] = pack_bf16(q[2 * w], q[2 * w + 1]);
        emit(a.qf);
#pragma unroll
        for (int u = 0; u < FW; u++) q[u] = 0.0f;
        q[0] = csh; q[1] = csh; q[2] = csl; q[3] = snh; q[4] = snh; q[5] = snl;
#pragma unroll
        for (int d = 0; d < NC; d++) {
            const float kh = bf16_round(c[d]);
            q[6 + 3 * d] = kh; q[7 + 3 * d] = kh; q[8 + 3 * d] = c[d] - kh;
        }
#pragma unroll
        for (int u = 0; u < 8; u++) q[BB + u] = (bk == u) ? 1.0f : 0.0f;
#pragma unroll
        for (int w = 0; w < FWW; w++) row[w] = pack_bf16(q[2 * w], q[2 * w + 1]);
        emit(a.kf);
    }

    // ---- values in fp16, zero padded to hdp; lanes along the row
    {
        const int hd = a.hd, hdp = a.hdp;
        const int nrows = (int)min(32LL, total - i0);
        const long long vrow0 = it;  // this lane's value row (cache view)
        for (int j0 = 0; j0 < nrows; j0 += 8) {
            float2 v[8][2];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int j = j0 + u;
                const long long vr = __shfl_sync(0xffffffffu, vrow0, j & 31);
                const float *src = a.sv.v + vr * hd;
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const int col = (q * 32 + lane) * 2;  // columns col, col + 1
                    float2 x2 = make_float2(0.f, 0.f);
                    if (j < nrows && col < hdp) {
                        if (col + 1 < hd) x2 = *reinterpret_cast<const float2 *>(src + col);
                        else if (col < hd) x2.x = src[col];
                    }
                    v[u][q] = x2;
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int j = j0 + u;
                if (j >= nrows) break;
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const int col = (q * 32 + lane) * 2;
                    if (col >= hdp) continue;
                    const float2 x2 = v[u][q];
                    const long long o = (i0 + j) * hdp + col;
                    *reinterpret_cast<uint32_t *>(a.vh + o) = pack_f16(x2.x, x2.y);
                }
            }
        }
    }

    // ---- self score, content norm, previous-position term
    const float self = 1.0f + c2 * a.cscale;
    const float cn = sqrtf(c2);
    // previous position: the lane below (same bh), lane 0 loads it
    float thp = __shfl_up_sync(0xffffffffu, th, 1);
    int bkp = __shfl_up_sync(0xffffffffu, bk, 1);
    float cp[NC > 0 ? NC : 1];
#pragma unroll
    for (int d = 0; d < NC; d++) cp[d] = __shfl_up_sync(0xffffffffu, c[d], 1);
    const int bh_below = __shfl_up_sync(0xffffffffu, bh, 1);
    if (t > 0 && (lane == 0 || bh_below != bh)) {
        const long long ip = max(0LL, wb_pos(a.sv, b, h, t - 1));
        thp = a.sv.theta[ip];
        bkp = a.sv.bucket[ip];
        const float *cr =
            C ? a.content + ((long long)b * a.T + t - 1) * ((long long)a.H * C) + (long long)h * C : nullptr;
#pragma unroll
        for (int d = 0; d < NC; d++) cp[d] = (d < C) ? cr[d] : 0.0f;
    }
    float sp = -INFINITY;
    if (t > 0 && !((allow >> bkp) & 1u)) {
        sp = cosf(n * (th - thp));
        if (C) {
            float dot = 0.0f;
#pragma unroll
            for (int d = 0; d < NC; d++)
                if (d < C) dot = fmaf(c[d], cp[d], dot);
            sp += dot * a.cscale;
        }
    }
    if (live) {
        a.m0[i] = self;
        a.cnorm[i] = cn;
        a.sprev[i] = sp;
    }
    // per-(b, h) maximum content norm: one atomic per run of equal bh
    if (NC) {
        float mx = live ? cn : 0.0f;
        const unsigned same = __match_any_sync(0xffffffffu, bh);
        const int leader = __ffs(same) - 1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float other = __shfl_xor_sync(0xffffffffu, mx, o);
            const int obh = __shfl_xor_sync(0xffffffffu, bh, o);
            if (obh == bh) mx = fmaxf(mx, other);
        }
        if (lane == leader && live) atomicMax(a.cmax + bh, __float_as_uint(mx));
    }
}

// ---------------------------------------------------------------------------
// Attention core: a persistent, warp-specialised kernel.  One CTA per SM
// walks work items -- 128 queries of one (sequence, head) -- handed out by
// an atomic counter, in groups of ATT_GROUP (sequence, head) rows, the
// longest query tiles of a group first (a group's key/value tiles stay in
// L2 while its items read them).  Per key tile j of an item (keys
// 128j..128j+127): S = Qf Kf_j^T (TMEM, fp32) -> P = exp(S - s_self) (fp16,
// written back into the first half of each thread's own S columns) ->
// O += P V_j (A from TMEM, the fp16 value tile from shared memory).
// ---------------------------------------------------------------------------
struct AttnTcArgs {
    int BH, H, T, hd, n_qt;     // BH = B * Hg rows
    int Hg, h0;                 // heads computed: h0 .. h0 + Hg - 1
    int n_items;                // BH * n_qt
    const float *m0, *sprev, *cnorm;
    const unsigned int *cmax;
    WbSeqView sv;               // fp32 values for the previous-position term
    float *o;                   // [B*T][E] merged head outputs
    int E;
    int *sched;                 // [0] work counter, [1] fallback count, [2..] fallback tiles bh * n_qt + qt
    uint32_t *dev_err;
    int dot;                    // dot-product features: bound |q| max|k| - shift instead of the content bound
    float bound;                // a score may exceed the row's shift by at most this (else the tile falls back)
    int o_tma;                  // o tiles leave by TMA stores through tm_o (head_dim a multiple of 32)
    int *tflag;                 // dot: per-tile flags [BH * n_qt], zero at launch (tiles listed at run time)
};

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

static constexpr int ATT_SOFTMAX_WARPS = 16;  // four per TMEM lane group
static constexpr int ATT_EPI_WARPS = 4;       // one per TMEM lane group
static constexpr int ATT_W_PROD = ATT_SOFTMAX_WARPS + ATT_EPI_WARPS;  // TMA + work items
static constexpr int ATT_W_MMA = ATT_W_PROD + 1;                      // PV issuer (and TMEM owner)
static constexpr int ATT_W_QK = ATT_W_MMA + 1;                        // QK issuer
static constexpr int ATT_THREADS = (ATT_W_QK + 1) * 32;               // 736
static constexpr int ATT_GROUP = 16;          // (sequence, head) rows per item group
static constexpr int ATT_SLOTS = 4;           // work-item descriptor ring

// A published work item: its (sequence, head) row and query tile (bh < 0:
// no more work) and the per-row fixed shift m0 and previous-position score.
struct AttnItem {
    int bh, qt, pad0, pad1;
    float m0[QT];
    float sp[QT];
};

template <int HDP, int FW>
struct AttnSmem {
    // feature rows of FW = 128 (dot-product attention at head_dim 65-128)
    // sit in two 64-column swizzle atoms, one 16 KB block per atom
    static_assert(FW == 16 || FW == 64 || FW == 128, "feature width 16, 64 or 128");
    static constexpr int FCH = FW > 64 ? FW / 64 : 1;  // TMA boxes per Q / K tile
    static constexpr int Q_BYTES = QT * FW * 2;      // 4 / 16 / 32 KB
    static constexpr int K_BYTES = KT * FW * 2;      // 4 / 16 / 32 KB
    static constexpr int V_BYTES = KT * HDP * 2;     // one fp16 value tile: 16 / 32 KB
    // epilogue staging per warp, 1024-byte aligned: a 32 x 32 fp32 tile in
    // the 128-byte swizzle for the TMA store (4 KB), or 32 x 33 floats
    static constexpr int EPI_WARP = 5120;
    static constexpr int FIXED = 2 * Q_BYTES + ATT_EPI_WARPS * EPI_WARP + ATT_SLOTS * (int)sizeof(AttnItem) +
                                 2 * 4 * QT * 4 + 512 + 16 + 1024;
    // K/V ring stages: as many as shared memory holds, at most 6
    static constexpr int ST_FIT = (232448 - FIXED) / (K_BYTES + V_BYTES);
    static constexpr int ST = ST_FIT < 6 ? ST_FIT : 6;
    static constexpr int OFF_Q = 0;                  // two Q buffers (items alternate)
    static constexpr int OFF_K = OFF_Q + 2 * Q_BYTES;
    static constexpr int OFF_V = OFF_K + ST * K_BYTES;
    static constexpr int OFF_EPI = OFF_V + ST * V_BYTES;                 // epilogue staging
    static constexpr int OFF_SLOT = OFF_EPI + ATT_EPI_WARPS * EPI_WARP;
    static constexpr int OFF_LSUM = OFF_SLOT + ATT_SLOTS * (int)sizeof(AttnItem);  // [2][4][QT] row-sum partials
    static constexpr int OFF_BAR = OFF_LSUM + 2 * 4 * QT * 4;
    // TMEM columns: NS score buffers of 128 columns (P(g) is written over the
    // first half of each thread's S(g) columns), then OBUF O buffers of HDP
    // columns: three S buffers let QK run two tiles ahead of the PV that
    // frees a buffer
    static constexpr int NS = 3;
    static constexpr int O_COL = NS * 128;
    static constexpr int OBUF = (512 - O_COL) / HDP >= 2 ? 2 : 1;
    // barriers: qfull[2], qfree[2], kvfull[ST], kvfree[ST], sfull[NS], pready[NS],
    // ofull[2], ofree[2], lready[2], itemfull[SLOTS], itemfree[SLOTS], mmadone,
    // sfree[NS], qkdone
    static constexpr int NBAR = 4 + 2 * ST + 2 * NS + 6 + 2 * ATT_SLOTS + 1 + NS + 1;
    static constexpr int BYTES = OFF_BAR + NBAR * 8 + 16 + 1024;  // + TMEM slot, alignment slack
    static_assert(ST >= 2, "attention K/V ring below two stages");
    static_assert(OFF_EPI % 1024 == 0 && EPI_WARP % 1024 == 0, "swizzled epilogue tiles need 1024-byte alignment");
    static_assert(EPI_WARP >= 32 * 33 * 4, "epilogue staging");
    static_assert(NBAR * 8 <= 512, "barrier space");
    static_assert(BYTES <= 232448, "attention shared memory above the 227 KB limit");
    static_assert(O_COL + OBUF * HDP <= 512, "TMEM: NS S and OBUF O buffers");
};

// Bounded mbarrier wait that also gives up once another role has raised the
// CTA's abort flag (so one timeout does not chain into one per barrier).
__device__ __forceinline__ bool att_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (ptx::mbar_try_wait_sleep(bar, parity, 20000)) return true;
        if (*abort_flag) return false;
        if (clock64() - t0 > 4000000000LL) {
            *abort_flag = 1;
            return false;
        }
    }
}

// Roles (704 threads):
//   warps 0-15 (softmax): four per TMEM lane group (warps w, w+4, w+8, w+12
//     own query rows 32(w&3)..+31, key columns 0-31, 32-63, 64-95, 96-127 of
//     each S tile): P = exp2 of the fixed shift, causal mask on the diagonal
//     tile, P (fp16) stored over the first 16 of the thread's own 32 S
//     columns; the row-sum partials go to shared memory per item.
//   warps 16-19 (epilogue): one per lane group: O / l, stored through
//     per-warp staging -- item k's
//     epilogue runs while the softmax warps work on item k+1 (O is double
//     buffered in TMEM).
//   warp 20 (producer): takes work items from the counter, tests the
//     bounded-score condition (content only; failing tiles go to the
//     fallback list), publishes the item (row, tile, m0 and previous-position
//     scores of its 128 rows), then loads Q and the K/V tiles by TMA.
//   warp 21 (PV): lane 0 issues O += P V per tile once P is ready; it owns
//     TMEM.
//   warp 22 (QK): lane 0 issues S_g = Qf Kf^T up to three tiles ahead of the
//     PV (three S buffers in TMEM).
// Roles 21 and 22 sit on their own schedulers' queues (warp % 4 = 1 and 2)
// beside four softmax warps each.
// TMEM columns: S0 [0,128), S1 [128,256), S2 [256,384), then the O buffers.
template <int HDP, int FW>
__global__ void __launch_bounds__(ATT_THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                   const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                   AttnTcArgs a) {
    using L = AttnSmem<HDP, FW>;
    constexpr int ST = L::ST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + L::OFF_BAR);
    uint64_t *qfull = bars, *qfree = bars + 2;
    uint64_t *kvfull = bars + 4, *kvfree = kvfull + ST;
    constexpr int NS = L::NS;
    uint64_t *sfull = kvfree + ST, *pready = sfull + NS, *ofull = pready + NS, *ofree = ofull + 2;
    uint64_t *lready = ofree + 2, *itemfull = lready + 2, *itemfree = itemfull + ATT_SLOTS;
    uint64_t *mmadone = itemfree + ATT_SLOTS;
    uint64_t *sfree = mmadone + 1, *qkdone = sfree + NS;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(qkdone + 1);
    AttnItem *slots = reinterpret_cast<AttnItem *>(sm + L::OFF_SLOT);
    float *lsum = reinterpret_cast<float *>(sm + L::OFF_LSUM);
    __shared__ int s_abort;
    volatile int *abort_flag = &s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < L::NBAR; i++) {
            uint64_t *bb = bars + i;
            uint32_t cnt = 1;
            if (bb >= pready && bb < pready + NS) cnt = ATT_SOFTMAX_WARPS / 2 * 32;  // one softmax group per tile
            else if (bb == lready || bb == lready + 1) cnt = ATT_SOFTMAX_WARPS * 32;
            else if (bb == ofree || bb == ofree + 1) cnt = ATT_EPI_WARPS * 32;
            else if (bb >= itemfull && bb < itemfull + ATT_SLOTS) cnt = 32;
            else if (bb >= itemfree && bb < itemfree + ATT_SLOTS) cnt = ATT_SOFTMAX_WARPS + ATT_EPI_WARPS + 1;
            ptx::mbar_init(bb, cnt);
        }
        ptx::fence_mbar_init();
        s_abort = 0;
    }
    if (warp == ATT_W_MMA) {
        ptx::tmem_alloc(tmem_slot, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t F_SW = FW >= 64 ? ptx::UMMA_SW128 : ptx::UMMA_SW32;
    constexpr uint32_t F_SBO = FW >= 64 ? 1024 : 256;  // 8 rows of the swizzle atom

    if (warp == ATT_W_PROD) {
        // ---------------- producer: work items, Q and K/V tiles
        long long g = 0;  // global tile counter of this CTA
        int k = 0;        // items published
        const int per_grp = ATT_GROUP * a.n_qt;
        if (lane == 0) {
            ptx::prefetch_tmap(&tm_q);
            ptx::prefetch_tmap(&tm_k);
            ptx::prefetch_tmap(&tm_v);
        }
        // Work items are fetched one ahead of the one whose tiles are being
        // issued: the counter's atomic for item k + 1 goes out when item k is
        // taken, and item k + 1's row data (fixed shifts, previous-position
        // scores) are loaded into registers before item k's K/V loop, so
        // neither round trip stands between two items (items of one or two
        // key tiles are common: a sequence's first query tiles).
        // take(): the first item at or after `item` that the tensor path runs
        // (content: tiles failing the bounded-score test go to the fallback
        // list), bh = -1 past the end; its rows' data into m0v / spv.
        auto take = [&](int item, int &bh, int &qt, float (&m0v)[4], float (&spv)[4]) {
            for (;;) {
                if (item >= a.n_items) {
                    bh = -1;
                    qt = 0;
                    return;
                }
                const int grp = item / per_grp, rr = item - grp * per_grp;
                const int gsz = min(ATT_GROUP, a.BH - grp * ATT_GROUP);
                bh = grp * ATT_GROUP + rr % gsz;
                qt = a.n_qt - 1 - rr / gsz;
                bool violate = false;
                if (FW >= 64) {
                    // bounded-score test of the tile's rows (content and
                    // dot-product features)
                    const float cm = __uint_as_float(__ldg(a.cmax + bh));
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int q = qt * QT + u * 32 + lane;
                        if (q < a.T) {
                            const long long rq = (long long)bh * a.T + q;
                            const float cn = __ldg(a.cnorm + rq);
                            violate |= a.dot ? cn * cm - __ldg(a.m0 + rq) > a.bound
                                             : 0.25f * cn * (cm - cn) > a.bound;
                        }
                    }
                }
                if (!__any_sync(0xffffffffu, violate)) break;
                int nx = 0;
                if (lane == 0) {
                    const int e = atomicAdd(a.sched + 1, 1);
                    a.sched[2 + e] = bh * a.n_qt + qt;
                    nx = atomicAdd(a.sched, 1);
                }
                item = __shfl_sync(0xffffffffu, nx, 0);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int q = qt * QT + u * 32 + lane;
                const long long rq = (long long)bh * a.T + q;
                m0v[u] = q < a.T ? __ldg(a.m0 + rq) : 0.0f;
                spv[u] = q < a.T ? __ldg(a.sprev + rq) : -INFINITY;
            }
        };
        int nitem = 0;  // lane 0: the counter value for the item after the current one
        if (lane == 0) nitem = atomicAdd(a.sched, 1);
        int cbh, cqt;
        float cm0[4], csp[4];
        take(__shfl_sync(0xffffffffu, nitem, 0), cbh, cqt, cm0, csp);
        if (lane == 0 && cbh >= 0) nitem = atomicAdd(a.sched, 1);
        for (;;) {
            const int s = k % ATT_SLOTS;
            if (k >= ATT_SLOTS && !att_wait(itemfree + s, ((k / ATT_SLOTS) - 1) & 1, abort_flag)) {
                if (lane == 0) atomicOr(a.dev_err, WB_DERR_TIMEOUT_TMA);
                break;
            }
            AttnItem *it = slots + s;
            const int bh = cbh, qt = cqt;
            if (lane == 0) {
                it->bh = bh;
                it->qt = qt;
            }
            if (bh >= 0) {
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    it->m0[u * 32 + lane] = cm0[u];
                    it->sp[u * 32 + lane] = csp[u];
                }
            }
            ptx::mbar_arrive(itemfull + s);  // every lane: its writes are released
            k++;
            if (bh < 0) break;
            // the next item (its counter value came back during this item's
            // predecessor) and the counter for the one after it
            take(__shfl_sync(0xffffffffu, nitem, 0), cbh, cqt, cm0, csp);
            if (lane == 0 && cbh >= 0) nitem = atomicAdd(a.sched, 1);
            if (lane == 0) {
                bool ok = true;
                // Q of item i = k - 1 into buffer i & 1, free once item i - 2's QKs completed
                const int i = k - 1, qb = i & 1;
                if (i >= 2 && !att_wait(qfree + qb, ((i - 2) >> 1) & 1, abort_flag)) ok = false;
                if (ok) {
                    ptx::mbar_arrive_expect_tx(qfull + qb, L::Q_BYTES);
#pragma unroll
                    for (int c = 0; c < L::FCH; c++)
                        ptx::tma_load_3d(sm + L::OFF_Q + qb * L::Q_BYTES + c * (QT * 128), &tm_q, qfull + qb, c * 64,
                                         qt * QT, bh);
                }
                for (int j = 0; ok && j <= qt; j++, g++) {
                    const int st = (int)(g % ST);
                    const long long f = g / ST;
                    if (f >= 1 && !att_wait(kvfree + st, (uint32_t)((f - 1) & 1), abort_flag)) {
                        ok = false;
                        break;
                    }
                    ptx::mbar_arrive_expect_tx(kvfull + st, L::K_BYTES + L::V_BYTES);
#pragma unroll
                    for (int c = 0; c < L::FCH; c++)
                        ptx::tma_load_3d(sm + L::OFF_K + st * L::K_BYTES + c * (KT * 128), &tm_k, kvfull + st, c * 64,
                                         j * KT, bh);
                    uint8_t *vst = sm + L::OFF_V + st * L::V_BYTES;
#pragma unroll
                    for (int c = 0; c < HDP / 64; c++)
                        ptx::tma_load_3d(vst + c * (KT * 128), &tm_v, kvfull + st, c * 64, j * KT, bh);
                }
                if (!ok) atomicOr(a.dev_err, WB_DERR_TIMEOUT_TMA);
            }
            g = __shfl_sync(0xffffffffu, g, 0);
            if (*abort_flag) break;
        }
        // copies still in flight (only after an abort) land before the CTA
        // leaves: wait for the last fill of every stage and the last Q
        if (lane == 0 && *abort_flag) {
            for (long long gg = g - 1; gg >= 0 && gg >= g - ST; gg--)
                ptx::mbar_wait(kvfull + (gg % ST), (uint32_t)((gg / ST) & 1), 200000000LL);
            for (int i = k - 2; i >= 0 && i >= k - 3; i--) ptx::mbar_wait(qfull + (i & 1), (i >> 1) & 1, 200000000LL);
        }
    } else if (warp == ATT_W_MMA) {
        // ---------------- PV issuer: per tile g in order, O += P(g) V(g)
        // once P(g) is ready (and, on an item's first tile, its O buffer has
        // been read); the commits free the K/V stage and, once the MMAs have
        // read P(g), the S buffer g % NS for QK(g + NS).  QK and PV come
        // from two threads that sleep in their own barrier waits: one thread
        // polling for both fell ~1000 cycles behind a ready P on a scheduler
        // it shares with four softmax warps, and one thread issuing both in a
        // fixed order stalls PV behind a K/V tile still in flight.
        if (lane == 0) {
            // fp16 P (TMEM) x the fp16 value tile (HDP/64 adjacent 64-column
            // atoms of the stage, MN-major), N = HDP
            constexpr uint32_t IDESC_PV = ptx::idesc_f16(128, HDP, 0, 1);
            long long gp = 0;
            int kp = 0, jp = 0;
            bool ok = true;
            for (;;) {
                const int sl = kp % ATT_SLOTS;
                const int ob = kp % L::OBUF;
                if (jp == 0) {
                    if (!att_wait(itemfull + sl, (kp / ATT_SLOTS) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    if (slots[sl].bh < 0) break;  // the end marker's slot is never returned
                    if (kp >= L::OBUF && !att_wait(ofree + ob, ((kp - L::OBUF) / L::OBUF) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                }
                if (!att_wait(pready + (int)(gp % NS), (uint32_t)((gp / NS) & 1), abort_flag)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t O_t = tmem + L::O_COL + (uint32_t)(ob * HDP);
                const uint32_t P_t = tmem + (uint32_t)((gp % NS) * 128);
                const uint64_t vd0 = ptx::smem_desc(ptx::smem_u32(sm + L::OFF_V + (int)(gp % ST) * L::V_BYTES),
                                                    KT * 128, 1024, ptx::UMMA_SW128);
#pragma unroll
                for (int kk = 0; kk < KT / 16; kk++) {
                    // keys 16kk..16kk+15: half kk/4 of the tile (its S columns 64h..), packed two per column
                    const uint32_t a_t = P_t + (uint32_t)(64 * (kk >> 2) + 8 * (kk & 3));
                    ptx::mma_bf16_ta(O_t, a_t, vd0 + (uint64_t)(kk * 2048 >> 4), IDESC_PV, (jp > 0 || kk > 0));
                }
                ptx::mma_commit(kvfree + (int)(gp % ST));
                ptx::mma_commit(sfree + (int)(gp % NS));
                gp++;
                if (++jp == slots[sl].qt + 1) {
                    ptx::mma_commit(ofull + ob);
                    ptx::mbar_arrive(itemfree + sl);
                    kp++;
                    jp = 0;
                }
            }
            if (!ok) atomicOr(a.dev_err, WB_DERR_TIMEOUT_MMA);
            // every MMA of this thread has completed before TMEM is released
            ptx::mma_commit(mmadone);
            ptx::mbar_wait(mmadone, 0, 200000000LL);
        }
        __syncwarp();
    } else if (warp == ATT_W_QK) {
        // ---------------- QK issuer: S(g) = Qf Kf_g^T into S buffer g % NS,
        // once PV(g - NS) has read that buffer and K/V tile g has landed
        if (lane == 0) {
            constexpr uint32_t IDESC_QK = ptx::idesc_bf16(128, 128, 0, 0);
            const uint32_t sQ0 = ptx::smem_u32(sm + L::OFF_Q);
            long long gq = 0;
            int kq = 0, jq = 0, qtk = 0;  // qtk: the item's last key tile, read while its slot is held
            bool ok = true;
            for (;;) {
                const int sl = kq % ATT_SLOTS;
                if (jq == 0) {
                    if (!att_wait(itemfull + sl, (kq / ATT_SLOTS) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    if (slots[sl].bh < 0) break;
                    qtk = slots[sl].qt;
                    if (!att_wait(qfull + (kq & 1), (kq >> 1) & 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                }
                if ((gq >= NS && !att_wait(sfree + (int)(gq % NS), (uint32_t)(((gq / NS) - 1) & 1), abort_flag)) ||
                    !att_wait(kvfull + (int)(gq % ST), (uint32_t)((gq / ST) & 1), abort_flag)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const int st = (int)(gq % ST);
                const uint32_t sK = ptx::smem_u32(sm + L::OFF_K + st * L::K_BYTES);
                const uint32_t S_t = tmem + (uint32_t)((gq % NS) * 128);
                const uint32_t sQ = sQ0 + (uint32_t)((kq & 1) * L::Q_BYTES);
                const uint64_t ad0 = ptx::smem_desc(sQ, 16, F_SBO, F_SW), bd0 = ptx::smem_desc(sK, 16, F_SBO, F_SW);
                // K = 16 per MMA: 32 bytes along a 128-byte swizzle row; past
                // 64 columns the next atom block (QT / KT rows x 128 B)
#pragma unroll
                for (int kk = 0; kk < FW / 16; kk++)
                    ptx::mma_bf16(S_t, ad0 + (uint64_t)((kk >> 2) * (QT * 8) + (kk & 3) * 2),
                                  bd0 + (uint64_t)((kk >> 2) * (KT * 8) + (kk & 3) * 2), IDESC_QK, kk > 0);
                ptx::mma_commit(sfull + (int)(gq % NS));
                gq++;
                if (++jq == qtk + 1) {
                    ptx::mma_commit(qfree + (kq & 1));  // Q of item kq no longer read
                    kq++;
                    jq = 0;
                }
            }
            if (!ok) atomicOr(a.dev_err, WB_DERR_TIMEOUT_MMA);
            ptx::mma_commit(qkdone);
            ptx::mbar_wait(qkdone, 0, 200000000LL);
        }
        __syncwarp();
    } else if (warp < ATT_SOFTMAX_WARPS) {
        // ---------------- softmax: two groups of 8 warps take the key tiles
        // in turn (group G the tiles g with g % 2 == G of the CTA's tile
        // sequence; tile g sits in S buffer g % NS), so one group's
        // exponentials overlap the other's waits; within a group two warps
        // per TMEM lane group each own 64 key columns, processed as two
        // 32-column chunks
        const float LOG2E = 1.4426950408889634f;
        const int row = tid & (QT - 1);
        const int grp = warp >> 3, half = (warp >> 2) & 1;
        const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
        long long g = 0;
        for (int k = 0;; k++) {
            const int sl = k % ATT_SLOTS;
            if (!att_wait(itemfull + sl, (k / ATT_SLOTS) & 1, abort_flag)) {
                atomicOr(a.dev_err, WB_DERR_TIMEOUT_SOFTMAX);
                break;
            }
            const AttnItem *it = slots + sl;
            const int bh = it->bh, qt = it->qt;
            const float nm0 = -it->m0[row] * LOG2E;
            const float sp = it->sp[row];
            __syncwarp();
            if (bh < 0) break;
            if (lane == 0) ptx::mbar_arrive(itemfree + sl);
            // the previous position's weight when its bucket is masked
            // (attn.rs:212-221): it replaces the ~0 of key q-1's column, in
            // the diagonal tile or, for the tile's first row, in column 127
            // of the tile before
            const float ep = sp > -INFINITY ? fast_exp2(fmaf(sp, LOG2E, nm0)) : 0.0f;
            const uint64_t l2e2 = ptx::f2_pack(LOG2E, LOG2E), nm2 = ptx::f2_pack(nm0, nm0);
            uint64_t l2 = ptx::f2_pack(0.0f, 0.0f);  // row-sum partials of even and odd columns
            bool ok = true, ovf = false;
            for (int j = 0; j <= qt; j++, g++) {
                if ((int)(g & 1) != grp) continue;
                const int sb = (int)(g % NS);
                if (!att_wait(sfull + sb, (uint32_t)((g / NS) & 1), abort_flag)) {
                    atomicOr(a.dev_err, WB_DERR_TIMEOUT_SOFTMAX);
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const bool diag = (j == qt);
                const uint32_t S_t = tmem + (uint32_t)(sb * 128 + half * 64) + lane_base;
                uint32_t pk0[16], pk1[16];
                // exp2((s - shift) log2 e) of columns 2i, 2i+1 (the scaling as
                // one packed fp32x2 FMA)
                auto exp_pair = [&](const uint32_t (&r)[32], int i, float &e0, float &e1) {
                    const uint64_t xv =
                        ptx::f2_fma(ptx::f2_pack(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), l2e2, nm2);
                    float x0, x1;
                    ptx::f2_unpack(xv, x0, x1);
                    e0 = fast_exp2(x0);
                    e1 = fast_exp2(x1);
                };
                auto exps = [&](const uint32_t (&r)[32], uint32_t (&pk)[16], int kbase) {
                    int pcol = -1;
                    if (ep > 0.0f) {
                        if (diag && row >= 1 && ((row - 1) >> 5) == (kbase >> 5)) pcol = (row - 1) & 31;
                        else if (j + 1 == qt && row == 0 && kbase == 96) pcol = 31;
                    }
                    if (__any_sync(0xffffffffu, diag || pcol >= 0)) {
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            float e0, e1;
                            exp_pair(r, i, e0, e1);
                            if (diag) {
                                if (kbase + 2 * i > row) e0 = 0.0f;
                                if (kbase + 2 * i + 1 > row) e1 = 0.0f;
                            }
                            if (2 * i == pcol) e0 = ep;
                            if (2 * i + 1 == pcol) e1 = ep;
                            l2 = ptx::f2_add(l2, ptx::f2_pack(e0, e1));
                            pk[i] = pack_f16(e0, e1);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 16; i++) {
                            float e0, e1;
                            exp_pair(r, i, e0, e1);
                            l2 = ptx::f2_add(l2, ptx::f2_pack(e0, e1));
                            pk[i] = pack_f16(e0, e1);
                        }
                    }
                };
                {
                    const uint64_t l2_before = l2;
                    uint32_t r[32];
                    ptx::tmem_ld32(S_t, r);
                    ptx::tmem_ld_wait();
                    exps(r, pk0, half * 64);
                    ptx::tmem_ld32(S_t + 32, r);
                    ptx::tmem_ld_wait();
                    exps(r, pk1, half * 64 + 32);
                    if (a.dot) {
                        // this tile's 64 probabilities of the row (the running
                        // sums' increase): past the limit one may not fit fp16
                        float b0, b1, a0, a1;
                        ptx::f2_unpack(l2_before, b0, b1);
                        ptx::f2_unpack(l2, a0, a1);
                        ovf |= !((a0 - b0) + (a1 - b1) <= DOT_P_TILE_SUM);
                    }
                }
                // P over the first half of this thread's (already read) S columns
                ptx::tmem_st16(S_t, pk0);
                ptx::tmem_st16(S_t + 16, pk1);
                ptx::tmem_st_wait();
                ptx::tc_fence_before();
                ptx::mbar_arrive(pready + sb);
            }
            if (!ok) break;
            // the item's row-sum partials; the buffer of item k-2 must have
            // been read by its epilogue.  A parity wait names one phase of
            // ofree and must not fall two phases behind: with two O buffers
            // ofree[k % 2] has completed at most the phase of item k-2 (item
            // k's epilogue needs these row sums); with one, item k-1's
            // epilogue may already be done too, so wait for that one (it
            // follows item k-2's and needs nothing from this item)
            constexpr int LAG = L::OBUF == 1 ? 1 : 2;
            if (k >= LAG && !att_wait(ofree + (k - LAG) % L::OBUF, ((k - LAG) / L::OBUF) & 1, abort_flag)) {
                atomicOr(a.dev_err, WB_DERR_TIMEOUT_SOFTMAX);
                break;
            }
            if (ovf) {
                // dot-product features: the query tile goes to the fp32
                // fallback list once (its O from this kernel is overwritten)
                const int tile = bh * a.n_qt + qt;
                if (atomicExch(a.tflag + tile, 1) == 0) a.sched[2 + atomicAdd(a.sched + 1, 1)] = tile;
            }
            float l0, l1;
            ptx::f2_unpack(l2, l0, l1);
            lsum[((k & 1) * 4 + grp * 2 + half) * QT + row] = l0 + l1;
            ptx::mbar_arrive(lready + (k & 1));
        }
    } else {
        // ---------------- epilogue (warps 16-19): O / l
        const int ew = warp - ATT_SOFTMAX_WARPS;  // lane group
        const int row = ew * 32 + lane;
        const uint32_t lane_base = (uint32_t)(ew * 32) << 16;
        uint8_t *tbuf = sm + L::OFF_EPI + ew * L::EPI_WARP;
        float *buf = reinterpret_cast<float *>(tbuf);
        if (a.o_tma && lane == 0) ptx::prefetch_tmap(&tm_o);
        for (int k = 0;; k++) {
            const int sl = k % ATT_SLOTS;
            if (!att_wait(itemfull + sl, (k / ATT_SLOTS) & 1, abort_flag)) {
                atomicOr(a.dev_err, WB_DERR_TIMEOUT_SOFTMAX);
                break;
            }
            const AttnItem *it = slots + sl;
            const int bh = it->bh, qt = it->qt;
            __syncwarp();
            if (bh < 0) break;
            if (lane == 0) ptx::mbar_arrive(itemfree + sl);
            const int b = bh / a.Hg, h = a.h0 + (bh - b * a.Hg);
            const int q0 = qt * QT + ew * 32;  // this warp's first row
            if (!att_wait(ofull + k % L::OBUF, (k / L::OBUF) & 1, abort_flag) ||
                !att_wait(lready + (k & 1), (k >> 1) & 1, abort_flag)) {
                atomicOr(a.dev_err, WB_DERR_TIMEOUT_MMA);
                break;
            }
            ptx::tc_fence_after();
            const float *ls = lsum + (k & 1) * 4 * QT + row;
            const float inv = 1.0f / ((ls[0] + ls[QT]) + (ls[2 * QT] + ls[3 * QT]));
            const uint32_t O_t = tmem + L::O_COL + (uint32_t)((k % L::OBUF) * HDP) + lane_base;
            float *orow0 = a.o + ((long long)b * a.T + q0) * a.E + (long long)h * a.hd;
            const int nrow = min(32, a.T - q0);
#pragma unroll 1
            for (int c = 0; c < HDP / 32; c++) {
                // 32 output columns
                uint32_t r[32];
                ptx::tmem_ld32(O_t + c * 32, r);
                ptx::tmem_ld_wait();
                if (c == HDP / 32 - 1) {
                    // O buffer and row sums read: the MMA and softmax may reuse them
                    ptx::tc_fence_before();
                    ptx::mbar_arrive(ofree + k % L::OBUF);
                }
#pragma unroll
                for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) * inv);
                if (a.o_tma) {
                    // the 32 x 32 tile through shared memory and one TMA store
                    // (rows past T are clipped by the map): row `lane`, its
                    // 16-byte chunk cc at chunk cc ^ (lane & 7) -- the 128-byte
                    // swizzle, conflict-free for these row-per-lane writes.
                    // The buffer's previous store must have read it first.
                    if (lane == 0) ptx::bulk_wait_read<0>();
                    __syncwarp();
#pragma unroll
                    for (int cc = 0; cc < 8; cc++) {
                        float4 v4 = make_float4(__uint_as_float(r[4 * cc]), __uint_as_float(r[4 * cc + 1]),
                                                __uint_as_float(r[4 * cc + 2]), __uint_as_float(r[4 * cc + 3]));
                        *reinterpret_cast<float4 *>(tbuf + lane * 128 + ((cc ^ (lane & 7)) << 4)) = v4;
                    }
                    ptx::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && q0 < a.T && c * 32 < a.hd) {
                        ptx::tma_store_3d(&tm_o, tbuf, h * a.hd + c * 32, q0, b);
                        ptx::bulk_commit();
                    }
                } else {
                    warp_stage32(buf, r, lane);
                    const int d = c * 32 + lane;
                    if (d < a.hd)
#pragma unroll 4
                        for (int jr = 0; jr < nrow; jr++) orow0[(long long)jr * a.E + d] = buf[jr * 33 + lane];
                }
            }
        }
        // every TMA store of this warp has written global memory
        if (lane == 0) ptx::bulk_wait<0>();
    }
    __syncwarp();
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == ATT_W_MMA) ptx::tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// bf16 GEMM with fp32 output and bias: C[m][n] = sum_k A[m][k] B[n][k] + bias[n]
// (A, B K-major).  128x128 tile per CTA, 64-wide K blocks in a 3-stage TMA
// ring; warp 0 lane 0 loads, warp 1 lane 0 issues tcgen05.mma; all four
// warps run the epilogue from TMEM.
// ---------------------------------------------------------------------------
// TF32 = true: A and B are fp32 in memory and the MMA is kind::tf32 (K = 8
// per instruction); the 128-byte K block then holds 32 elements instead of 64.
static constexpr int GBM = 128, GBN = 128, GST = 3;
// narrow tiles for GEMMs whose 128 x 128 grid would leave most SMs idle
// (the decode out_proj of 64-1000 rows): 4x the CTAs, a deeper TMA ring
static constexpr int GBN_NARROW = 32, GST_NARROW = 6;
template <int BN, int NST>
struct GemmSmem {
    static constexpr int STAGE = (GBM + BN) * 128;  // A and B rows of one 128-byte K block
    static constexpr int BYTES = NST * STAGE + 128 + 1024;
    static_assert(STAGE % 1024 == 0, "128-byte-swizzled operands need 1024-byte alignment");
    static_assert(NST * STAGE >= 4 * 32 * 33 * 4, "epilogue staging reuses the ring");
};
static constexpr int G_ROW = 128;                       // bytes of one K block row

template <bool TF32, int BN = GBN, int NST = GST>
__global__ void __launch_bounds__(128, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const float *__restrict__ bias, float *__restrict__ C, int M, int N, int K, long long ldc,
                   uint32_t *dev_err, int accumulate) {
    constexpr int GBK = TF32 ? 32 : 64;  // elements per K block
    constexpr int STAGE = GemmSmem<BN, NST>::STAGE;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + NST * STAGE);
    uint64_t *full = bars, *empty = bars + NST, *done = bars + 2 * NST;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * NST + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    // column tiles vary fastest: the CTAs of one row tile run together and
    // read its A rows from L2 after the first
    const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * BN;
    const int nk = (K + GBK - 1) / GBK;
    if (tid == 0) {
        for (int i = 0; i < 2 * NST + 1; i++) ptx::mbar_init(bars + i, 1);
        ptx::fence_mbar_init();
    }
    if (warp == 0) {
        ptx::tmem_alloc(tmem_slot, BN);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    if (tid == 0) {
        ptx::prefetch_tmap(&tm_a);
        ptx::prefetch_tmap(&tm_b);
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % NST;
            if (kb >= NST && !ptx::mbar_wait(empty + s, ((kb / NST) - 1) & 1)) {
                atomicOr(dev_err, WB_DERR_TIMEOUT_MMA);
                ok = false;
                break;
            }
            uint8_t *st = sm + s * STAGE;
            ptx::mbar_arrive_expect_tx(full + s, STAGE);
            ptx::tma_load_2d(st, &tm_a, full + s, kb * GBK, m0);
            ptx::tma_load_2d(st + GBM * G_ROW, &tm_b, full + s, kb * GBK, n0);
        }
    } else if (tid == 32) {
        constexpr uint32_t IDESC = TF32 ? ptx::idesc_tf32(GBM, BN) : ptx::idesc_bf16(GBM, BN, 0, 0);
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % NST;
            if (!ptx::mbar_wait(full + s, (kb / NST) & 1)) {
                atomicOr(dev_err, WB_DERR_TIMEOUT_TMA);
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            const uint32_t sa = ptx::smem_u32(sm + s * STAGE), sb = sa + GBM * G_ROW;
#pragma unroll
            for (int k = 0; k < 4; k++) {  // 32 bytes of K per instruction
                const uint64_t ad = ptx::smem_desc(sa + k * 32, 16, 1024, ptx::UMMA_SW128);
                const uint64_t bd = ptx::smem_desc(sb + k * 32, 16, 1024, ptx::UMMA_SW128);
                if (TF32)
                    ptx::mma_tf32(tmem, ad, bd, IDESC, (kb > 0 || k > 0));
                else
                    ptx::mma_bf16(tmem, ad, bd, IDESC, (kb > 0 || k > 0));
            }
            ptx::mma_commit(empty + s);
        }
        ptx::mma_commit(done);
    }
    const bool fin = ptx::mbar_wait(done, 0);
    if (!fin && tid == 0) atomicOr(dev_err, WB_DERR_TIMEOUT_MMA);
    ptx::tc_fence_after();
    if (fin) {
        // the pipeline stages are free (every MMA has completed): each warp
        // stages its 32 rows chunk by chunk and stores them row by row
        float *buf = reinterpret_cast<float *>(sm) + warp * 32 * 33;
        const int lane = tid & 31;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c++) {
            uint32_t r[32];
            ptx::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c * 32, r);
            ptx::tmem_ld_wait();
            warp_stage32(buf, r, lane);
            const int n = n0 + c * 32 + lane;
            const float bv = (bias && n < N) ? bias[n] : 0.0f;
#pragma unroll 4
            for (int j = 0; j < 32; j++) {
                const int m = m0 + warp * 32 + j;
                if (m < M && n < N) {
                    float *c = C + (long long)m * ldc + n;
                    *c = accumulate ? *c + (buf[j * 33 + lane] + bv) : buf[j * 33 + lane] + bv;
                }
            }
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) ptx::tmem_dealloc(tmem, BN);
    (void)ok;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int tc_layer_upload(TcLayerWeights *t, const wb_attn_weights_desc *w, std::string *msg) {
    t->E = w->n_embd;
    t->H = w->n_head;
    t->hd = w->n_embd / w->n_head;
    t->C = w->content_dim;
    {
        int rc = proj_weights_upload(&t->proj, w, msg);
        if (rc) return rc;
    }
    const size_t n = (size_t)t->E * t->E;
    if (cudaMalloc(&t->w_o32, n * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        *msg = "cudaMalloc for fp32 out_proj failed";
        return WB_ENOMEM;
    }
    if (cudaMemcpy(t->w_o32, w->out_proj_w, n * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
        *msg = "upload of out_proj failed";
        return WB_ECUDA;
    }
    return WB_OK;
}

void tc_layer_free(TcLayerWeights *t) {
    proj_weights_free(&t->proj);
    if (t->w_o32) cudaFree(t->w_o32);
    t->w_o32 = nullptr;
}

// Workspace pieces of the attention core, carved after `off`.
struct CoreLayout {
    size_t qf, kf, vh, m0, sp, cn, cm, sched, tflag, o, end;
};
static int core_fw(bool content) { return content ? 64 : 16; }
// fw_dot: feature width of the dot-product core (64 or 128), 0 for wave attention
static CoreLayout core_layout(const TcLayerWeights &t, int B, int T, size_t off, int Hg, bool content,
                              int fw_dot = 0) {
    const int hdp = t.hd <= 64 ? 64 : 128;
    const int fw = fw_dot ? fw_dot : core_fw(content);
    const long long BH = (long long)B * Hg, R = (long long)B * T;
    const int n_qt = (T + QT - 1) / QT;
    Carve cv;
    cv.off = off;
    CoreLayout c;
    c.qf = cv.take<__nv_bfloat16>(BH * T * fw);
    c.kf = cv.take<__nv_bfloat16>(BH * T * fw);
    c.vh = cv.take<__half>(BH * T * hdp);
    c.m0 = cv.take<float>(BH * T);
    c.sp = cv.take<float>(BH * T);
    c.cn = cv.take<float>(BH * T);
    c.cm = cv.take<unsigned int>(BH);
    c.sched = cv.take<int>(2 + BH * n_qt);
    c.tflag = fw_dot ? cv.take<int>(BH * n_qt) : 0;
    c.o = cv.take<float>(R * t.E);
    c.end = cv.off;
    return c;
}

// y = A W^T + bias on the tcgen05 GEMM: A [M][K] and W [N][K] bf16 (tf32 =
// false) or fp32 (tf32 = true), K-major with row strides lda / ldw elements
// (0 = K); C [M][ldc] fp32; bias may be null.
static int launch_gemm(bool tf32, const void *A, const void *W, const float *bias, float *C, int M, int N, int K,
                       long long ldc, uint32_t *dev_err, cudaStream_t st, std::string *msg, long long lda = 0,
                       long long ldw = 0, int accumulate = 0) {
    const int esz = tf32 ? 4 : 2;
    if (!lda) lda = K;
    if (!ldw) ldw = K;
    if (M <= 0 || N <= 0 || K <= 0 || ((long long)K * esz) % 16 || (lda * esz) % 16 || (ldw * esz) % 16 ||
        (reinterpret_cast<uintptr_t>(A) % 16) || (reinterpret_cast<uintptr_t>(W) % 16)) {
        *msg = "bad GEMM shape (rows and bases of A and W must be 16-byte aligned)";
        return WB_EINVAL;
    }
    const CUtensorMapDataType dt = tf32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const uint32_t bk = G_ROW / esz;
    CUtensorMap ta, tb;
    int rc;
    const uint64_t adims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t astr[1] = {(uint64_t)lda * esz};
    const uint32_t abox[2] = {bk, GBM};
    if ((rc = make_tmap(&ta, A, dt, 2, adims, astr, abox, CU_TENSOR_MAP_SWIZZLE_128B, msg))) return rc;
    const uint64_t bdims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t bstr[1] = {(uint64_t)ldw * esz};
    // 128 x 128 tiles, or 128 x 32 when the wide grid would be smaller than
    // one CTA per SM of a B200 (148)
    const long long wide_tiles = (long long)((N + GBN - 1) / GBN) * ((M + GBM - 1) / GBM);
    const bool narrow = wide_tiles < 148;
    const int bn = narrow ? GBN_NARROW : GBN;
    const uint32_t bbox[2] = {bk, (uint32_t)bn};
    if ((rc = make_tmap(&tb, W, dt, 2, bdims, bstr, bbox, CU_TENSOR_MAP_SWIZZLE_128B, msg))) return rc;
    if ((M + GBM - 1) / GBM > 65535) {
        *msg = "GEMM with more than 65535 row tiles";
        return WB_EINVAL;
    }
    dim3 gg((unsigned)((N + bn - 1) / bn), (unsigned)((M + GBM - 1) / GBM));
    ProfScope ps(tf32 ? "gemm_tf32" : "gemm_bf16", st);
    auto go = [&](auto kernel, int smem) {
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        kernel<<<gg, 128, smem, st>>>(ta, tb, bias, C, M, N, K, ldc, dev_err, accumulate);
    };
    using Wide = GemmSmem<GBN, GST>;
    using Narrow = GemmSmem<GBN_NARROW, GST_NARROW>;
    if (tf32) {
        if (narrow) go(gemm_tc_kernel<true, GBN_NARROW, GST_NARROW>, Narrow::BYTES);
        else go(gemm_tc_kernel<true, GBN, GST>, Wide::BYTES);
    } else {
        if (narrow) go(gemm_tc_kernel<false, GBN_NARROW, GST_NARROW>, Narrow::BYTES);
        else go(gemm_tc_kernel<false, GBN, GST>, Wide::BYTES);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("gemm launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

template <int HDP, int FW>
static int launch_attn_tc(const CUtensorMap &tq, const CUtensorMap &tk, const CUtensorMap &tv, const AttnTcArgs &aa,
                          int sm_count, cudaStream_t st, std::string *msg) {
    using L = AttnSmem<HDP, FW>;
    const int grid = std::max(1, std::min(aa.n_items, sm_count));
    // o [B][T][E] fp32 as 32 x 32 tiles for TMA stores, when a tile's
    // columns start 16-byte aligned and stay inside one head (head_dim a
    // multiple of 32); other head dims store rows from registers
    AttnTcArgs a2 = aa;
    CUtensorMap to;
    memset(&to, 0, sizeof(to));
    a2.o_tma = 0;
    if (aa.hd % 32 == 0 && ((uintptr_t)aa.o & 15) == 0 && (aa.E * 4) % 16 == 0) {
        const int B = aa.BH / aa.Hg;
        const uint64_t dims[3] = {(uint64_t)aa.E, (uint64_t)aa.T, (uint64_t)B};
        const uint64_t strides[2] = {(uint64_t)aa.E * 4, (uint64_t)aa.T * aa.E * 4};
        const uint32_t box[3] = {32, 32, 1};
        int rc = make_tmap(&to, aa.o, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B, msg);
        if (rc) return rc;
        a2.o_tma = 1;
    }
    ProfScope ps("attn_tc", st);
    cudaFuncSetAttribute(attn_tc_kernel<HDP, FW>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
    attn_tc_kernel<HDP, FW><<<grid, ATT_THREADS, L::BYTES, st>>>(tq, tk, tv, to, a2);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("attention launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

// Runs features -> tcgen05 attention -> SIMT fallback for listed tiles ->
// tcgen05 out_proj, given phases/buckets/values already in `sv` and (when
// content is non-null) content vectors.  The workspace must already hold
// core_layout(...).end bytes.
static int tc_attention_core(const TcLayerWeights &t, const WbSeqView &sv, const float *content, int B, int T,
                             int h0, int Hg, bool add_bias, float *y, Workspace *ws, const CoreLayout &lay,
                             uint32_t *dev_err, int sm_count, cudaStream_t st, std::string *msg) {
    const int H = t.H, hd = t.hd, E = t.E;
    const int hdp = hd <= 64 ? 64 : 128;
    const int fw = core_fw(content != nullptr);
    const long long BH = (long long)B * Hg, R = (long long)B * T;
    const int n_qt = (T + QT - 1) / QT;
    if (BH * n_qt > 0x7fffffffLL) {
        *msg = "too many attention work items";
        return WB_EINVAL;
    }
    int rc;
    char *w = (char *)ws->p;
    __nv_bfloat16 *qf = (__nv_bfloat16 *)(w + lay.qf), *kf = (__nv_bfloat16 *)(w + lay.kf);
    __half *vh = (__half *)(w + lay.vh);
    float *ob = (float *)(w + lay.o);
    float *m0 = (float *)(w + lay.m0), *sp = (float *)(w + lay.sp), *cn = (float *)(w + lay.cn);
    unsigned int *cm = (unsigned int *)(w + lay.cm);
    int *sched = (int *)(w + lay.sched);
    if ((content && cudaMemsetAsync(cm, 0, BH * sizeof(unsigned int), st) != cudaSuccess) ||
        cudaMemsetAsync(sched, 0, 2 * sizeof(int), st) != cudaSuccess) {
        *msg = "cudaMemsetAsync failed";
        return WB_ECUDA;
    }
    const float cscale = content ? 1.0f / std::sqrt((float)t.C) : 0.0f;
    FeatArgs fa{sv, content, content ? t.C : 0, cscale, t.harmonic_n, B, H, T, hd, hdp, Hg, h0,
                qf, kf, vh, m0, sp, cn, cm};
    const unsigned fgrid = (unsigned)((BH * T + FEAT_WARPS * 32 - 1) / (FEAT_WARPS * 32));
    {
        ProfScope ps("feat", st);
        if (fw == 64) feat_kernel<64><<<fgrid, FEAT_WARPS * 32, 0, st>>>(fa);
        else feat_kernel<16><<<fgrid, FEAT_WARPS * 32, 0, st>>>(fa);
    }

    CUtensorMap tq, tk, tv;
    {
        const uint64_t dims[3] = {(uint64_t)fw, (uint64_t)T, (uint64_t)BH};
        const uint64_t strides[2] = {(uint64_t)fw * 2, (uint64_t)T * fw * 2};
        const uint32_t box[3] = {(uint32_t)fw, 128, 1};
        const CUtensorMapSwizzle fsw = fw == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B;
        if ((rc = make_tmap(&tq, qf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box, fsw, msg))) return rc;
        if ((rc = make_tmap(&tk, kf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box, fsw, msg))) return rc;
        const uint64_t vdims[3] = {(uint64_t)hdp, (uint64_t)T, (uint64_t)BH};
        const uint64_t vstr[2] = {(uint64_t)hdp * 2, (uint64_t)T * hdp * 2};
        const uint32_t vbox[3] = {64, 128, 1};
        if ((rc = make_tmap(&tv, vh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, vdims, vstr, vbox,
                            CU_TENSOR_MAP_SWIZZLE_128B, msg)))
            return rc;
    }
    AttnTcArgs aa{(int)BH, H, T, hd, n_qt, Hg, h0, (int)(BH * n_qt), m0, sp, cn, cm, sv, ob, E, sched, dev_err, 0,
                  BOUND_LIMIT};
    if (hdp == 64)
        rc = fw == 64 ? launch_attn_tc<64, 64>(tq, tk, tv, aa, sm_count, st, msg)
                      : launch_attn_tc<64, 16>(tq, tk, tv, aa, sm_count, st, msg);
    else
        rc = fw == 64 ? launch_attn_tc<128, 64>(tq, tk, tv, aa, sm_count, st, msg)
                      : launch_attn_tc<128, 16>(tq, tk, tv, aa, sm_count, st, msg);
    if (rc) return rc;
    // query tiles whose scores may exceed the fixed-shift bound (content
    // only): recomputed in fp32 from the list the attention kernel built
    if (content)
        launch_attn_simt_fallback_f32(sv, content, t.C, cscale, t.harmonic_n, B, H, T, hd, ob, sched + 1, h0, Hg,
                                      st);
    // out_proj: y = o W_o^T (+ b_o), over the computed heads' columns of o
    // and W_o (K = Hg * hd): the partial output of a head range
    if (Hg == H)
        return launch_gemm(true, ob, t.w_o32, add_bias ? t.b_o : nullptr, y, (int)R, E, E, E, dev_err, st, msg);
    return launch_gemm(true, ob + (size_t)h0 * hd, t.w_o32 + (size_t)h0 * hd, add_bias ? t.b_o : nullptr, y, (int)R,
                       E, Hg * hd, E, dev_err, st, msg, E, E);
}

// ---------------------------------------------------------------------------
// Dot-product attention on the same core (compute.rs:357-414): per row
// i = (b * H + h) * T + t, Qf = bf16(q / sqrt(d)) and Kf = bf16(k) padded
// with zeros to 64 columns (no bucket columns: nothing is masked but the
// causal triangle), values in fp16, and the fixed shift = the fp32
// self score q.k_t / sqrt(d), which every row contains.  A score exceeds
// the shift by at most |q| max_k|k| / sqrt(d) - s_self; query tiles where
// that passes the bound go to the fp32 core through the fallback list.
// ---------------------------------------------------------------------------
struct DotFeatArgs {
    const float *qkv;  // [B*T][3E]
    int B, H, T, hd, E;
    float scale;
    __nv_bfloat16 *qf, *kf;  // [BH][T][FW]
    __half *vh;              // [BH][T][FW] values (fp16)
    float *m0, *sprev, *cnorm;         // [BH][T]
    unsigned int *cmax;                // [BH], float bits of max |k|
};

static constexpr int DOT_FEAT_WARPS = 8;

// DOT_FEAT_ROWS consecutive input rows (b, t..t+R-1) per CTA; warp w takes
// heads w, w + 8, ... of those rows.  A warp loads the q, k and v slices of
// all R rows of a head straight from global memory (3R loads per lane in
// flight: 16- or 8-byte loads when the slice is a full, aligned FW-wide
// run, else predicated 4-byte loads), then forms each row's features and
// raises max |k| of the head once for the R rows (per-row atomics on one
// address per head serialised in L2).
// The row's fixed softmax shift m0 is the largest of the scores of four keys
// it certainly sees (causal): its own, the previous one, key t0/2 and key 0
// (t0 the row group's first row).  So the
// row's largest probability is at least ~1 (no underflow); a shift far below
// the row's true maximum shows at run time (DOT_P_TILE_SUM).
static constexpr int DOT_FEAT_ROWS = 4;

// FW = 64 (head_dim <= 64) or 128: each lane forms FW / 32 adjacent columns
// of a row's features and values (zero past head_dim).  vec: hd == FW and
// every slice start aligned to FW / 32 floats.
template <int FW>
__global__ void __launch_bounds__(DOT_FEAT_WARPS * 32) dot_feat_kernel(DotFeatArgs a, int vec) {
    static_assert(FW == 64 || FW == 128, "dot-product feature width");
    constexpr int EPL = FW / 32;  // columns per lane
    constexpr int R = DOT_FEAT_ROWS;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int n_tb = (a.T + R - 1) / R;  // row groups per sequence (a group stays within one)
    const int b = blockIdx.x / n_tb, t0 = (blockIdx.x - b * n_tb) * R;
    const int nr = min(R, a.T - t0);
    const long long rs = 3LL * a.E;  // qkv row stride
    const float *rows0 = a.qkv + ((long long)b * a.T + t0) * rs;
    const float *seq0 = a.qkv + (long long)b * a.T * rs;
    // EPL columns of a head slice starting at p (zero past head_dim or when !ok)
    auto load_slice = [&](const float *p, bool ok, float (&dst)[EPL]) {
        if (vec) {
            if constexpr (EPL == 4) {
                float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
                if (ok) f = __ldg(reinterpret_cast<const float4 *>(p) + lane);
                dst[0] = f.x, dst[1] = f.y, dst[2] = f.z, dst[3] = f.w;
            } else {
                float2 f = make_float2(0.f, 0.f);
                if (ok) f = __ldg(reinterpret_cast<const float2 *>(p) + lane);
                dst[0] = f.x, dst[1] = f.y;
            }
        } else {
#pragma unroll
            for (int u = 0; u < EPL; u++) {
                const int d = EPL * lane + u;
                dst[u] = ok && d < a.hd ? __ldg(p + d) : 0.0f;
            }
        }
    };
    // lane-partial dot product in the order of the self score below
    auto part_dot = [&](const float (&x)[EPL], const float (&y)[EPL]) {
        float d = fmaf(x[0], y[0], x[1] * y[1]);
        if constexpr (EPL == 4) d += fmaf(x[2], y[2], x[3] * y[3]);
        return d;
    };
    for (int h = warp; h < a.H; h += DOT_FEAT_WARPS) {
        const long long bh = (long long)b * a.H + h;
        float q[R][EPL], k[R][EPL], v[R][EPL], k0[EPL], kh[EPL], kp[EPL];
        // keys 0, t0 / 2 and t0 - 1 of the sequence (visible to every row of the group)
        load_slice(seq0 + a.E + h * a.hd, true, k0);
        load_slice(seq0 + (long long)(t0 >> 1) * rs + a.E + h * a.hd, true, kh);
        load_slice(rows0 - rs + a.E + h * a.hd, t0 > 0, kp);
#pragma unroll
        for (int r = 0; r < R; r++) {
            const float *row = rows0 + r * rs + h * a.hd;
            const bool rok = r < nr;
            if (vec) {
                if constexpr (EPL == 4) {
                    float4 z = make_float4(0.f, 0.f, 0.f, 0.f), fq = z, fk = z, fv = z;
                    if (rok) {
                        fq = __ldg(reinterpret_cast<const float4 *>(row) + lane);
                        fk = __ldg(reinterpret_cast<const float4 *>(row + a.E) + lane);
                        fv = __ldg(reinterpret_cast<const float4 *>(row + 2 * a.E) + lane);
                    }
                    q[r][0] = fq.x, q[r][1] = fq.y, q[r][2] = fq.z, q[r][3] = fq.w;
                    k[r][0] = fk.x, k[r][1] = fk.y, k[r][2] = fk.z, k[r][3] = fk.w;
                    v[r][0] = fv.x, v[r][1] = fv.y, v[r][2] = fv.z, v[r][3] = fv.w;
                } else {
                    float2 z = make_float2(0.f, 0.f), fq = z, fk = z, fv = z;
                    if (rok) {
                        fq = __ldg(reinterpret_cast<const float2 *>(row) + lane);
                        fk = __ldg(reinterpret_cast<const float2 *>(row + a.E) + lane);
                        fv = __ldg(reinterpret_cast<const float2 *>(row + 2 * a.E) + lane);
                    }
                    q[r][0] = fq.x, q[r][1] = fq.y;
                    k[r][0] = fk.x, k[r][1] = fk.y;
                    v[r][0] = fv.x, v[r][1] = fv.y;
                }
            } else {
#pragma unroll
                for (int u = 0; u < EPL; u++) {
                    const int d = EPL * lane + u;
                    const bool ok = rok && d < a.hd;
                    q[r][u] = ok ? __ldg(row + d) : 0.0f;
                    k[r][u] = ok ? __ldg(row + a.E + d) : 0.0f;
                    v[r][u] = ok ? __ldg(row + 2 * a.E + d) : 0.0f;
                }
            }
        }
        float kmax = 0.0f;
#pragma unroll
        for (int r = 0; r < R; r++) {
            if (r >= nr) break;
            const long long i = bh * a.T + t0 + r;  // feature row
#pragma unroll
            for (int u = 0; u < EPL; u++) q[r][u] *= a.scale;
            // scores against keys 0, t0 / 2 and the previous one (row t0 + r - 1)
            float s0 = part_dot(q[r], k0), s1 = part_dot(q[r], kh);
            float sq = r == 0 ? part_dot(q[r], kp) : part_dot(q[r], k[r > 0 ? r - 1 : 0]);
            float s, qq, kk;
            if constexpr (EPL == 2) {
                reinterpret_cast<uint32_t *>(a.qf + i * FW)[lane] = pack_bf16(q[r][0], q[r][1]);
                reinterpret_cast<uint32_t *>(a.kf + i * FW)[lane] = pack_bf16(k[r][0], k[r][1]);
                reinterpret_cast<uint32_t *>(a.vh + i * FW)[lane] = pack_f16(v[r][0], v[r][1]);
                s = fmaf(q[r][0], k[r][0], q[r][1] * k[r][1]);
                qq = fmaf(q[r][0], q[r][0], q[r][1] * q[r][1]);
                kk = fmaf(k[r][0], k[r][0], k[r][1] * k[r][1]);
            } else {
                reinterpret_cast<uint2 *>(a.qf + i * FW)[lane] =
                    make_uint2(pack_bf16(q[r][0], q[r][1]), pack_bf16(q[r][2], q[r][3]));
                reinterpret_cast<uint2 *>(a.kf + i * FW)[lane] =
                    make_uint2(pack_bf16(k[r][0], k[r][1]), pack_bf16(k[r][2], k[r][3]));
                reinterpret_cast<uint2 *>(a.vh + i * FW)[lane] =
                    make_uint2(pack_f16(v[r][0], v[r][1]), pack_f16(v[r][2], v[r][3]));
                s = fmaf(q[r][0], k[r][0], q[r][1] * k[r][1]) + fmaf(q[r][2], k[r][2], q[r][3] * k[r][3]);
                qq = fmaf(q[r][0], q[r][0], q[r][1] * q[r][1]) + fmaf(q[r][2], q[r][2], q[r][3] * q[r][3]);
                kk = fmaf(k[r][0], k[r][0], k[r][1] * k[r][1]) + fmaf(k[r][2], k[r][2], k[r][3] * k[r][3]);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                s += __shfl_xor_sync(0xffffffffu, s, o);
                qq += __shfl_xor_sync(0xffffffffu, qq, o);
                kk += __shfl_xor_sync(0xffffffffu, kk, o);
                s0 += __shfl_xor_sync(0xffffffffu, s0, o);
                s1 += __shfl_xor_sync(0xffffffffu, s1, o);
                sq += __shfl_xor_sync(0xffffffffu, sq, o);
            }
            kmax = fmaxf(kmax, sqrtf(kk));
            if (lane == 0) {
                // every sampled key is at or before the row (row 0 sees only itself)
                a.m0[i] = t0 + r > 0 ? fmaxf(fmaxf(s, sq), fmaxf(s0, s1)) : s;
                a.sprev[i] = -INFINITY;  // no previous-position rule
                a.cnorm[i] = sqrtf(qq);
            }
        }
        if (lane == 0) atomicMax(a.cmax + bh, __float_as_uint(kmax));  // non-negative floats order as their bits
    }
}

// features and values padded to 64 columns up to head_dim 64, else 128
static int dot_fw(int hd) { return hd <= 64 ? 64 : 128; }

size_t tc_dot_core_bytes(int B, int T, int E, int H) {
    const int fw = dot_fw(E / H);
    TcLayerWeights t{};
    t.E = fw * H;
    t.H = H;
    t.hd = fw;
    // the core layout without its merged-output rows (the caller owns o)
    const CoreLayout c = core_layout(t, B, T, 0, H, true, fw);
    return c.o;
}

int tc_dot_attention(const float *qkv, int B, int T, int E, int H, float *o, void *ws, int force_fallback,
                     uint32_t *dev_err, int sm_count, cudaStream_t st, std::string *msg) {
    const int hd = E / H;
    if (hd > 128) {
        *msg = "the tensor-core dot-product core supports head_dim <= 128";
        return WB_ENOTSUP;
    }
    const int fw = dot_fw(hd);
    const long long BH = (long long)B * H;
    const int n_qt = (T + QT - 1) / QT;
    if (BH * n_qt > 0x7fffffffLL) {
        *msg = "too many attention work items";
        return WB_EINVAL;
    }
    TcLayerWeights t{};
    t.E = fw * H;
    t.H = H;
    t.hd = fw;
    const CoreLayout lay = core_layout(t, B, T, 0, H, true, fw);
    char *w = (char *)ws;
    __nv_bfloat16 *qf = (__nv_bfloat16 *)(w + lay.qf), *kf = (__nv_bfloat16 *)(w + lay.kf);
    __half *vh = (__half *)(w + lay.vh);
    float *m0 = (float *)(w + lay.m0), *sp = (float *)(w + lay.sp), *cn = (float *)(w + lay.cn);
    unsigned int *cm = (unsigned int *)(w + lay.cm);
    int *sched = (int *)(w + lay.sched), *tflag = (int *)(w + lay.tflag);
    if (cudaMemsetAsync(cm, 0, BH * sizeof(unsigned int), st) != cudaSuccess ||
        cudaMemsetAsync(sched, 0, 2 * sizeof(int), st) != cudaSuccess ||
        cudaMemsetAsync(tflag, 0, BH * n_qt * sizeof(int), st) != cudaSuccess) {
        *msg = "cudaMemsetAsync failed";
        return WB_ECUDA;
    }
    DotFeatArgs fa{qkv, B, H, T, hd, E, 1.0f / std::sqrt((float)hd), qf, kf, vh, m0, sp, cn, cm};
    {
        ProfScope ps("dot_feat", st);
        const unsigned grid = (unsigned)((long long)B * ((T + DOT_FEAT_ROWS - 1) / DOT_FEAT_ROWS));
        // full-width slices whose starts (row stride 3E, head offsets hd, the
        // base) are aligned to the lane's FW / 32 floats load as vectors
        const int vec = hd == fw && E % (fw / 32) == 0 && ((uintptr_t)qkv % (fw / 8)) == 0;
        if (fw == 64) dot_feat_kernel<64><<<grid, DOT_FEAT_WARPS * 32, 0, st>>>(fa, vec);
        else dot_feat_kernel<128><<<grid, DOT_FEAT_WARPS * 32, 0, st>>>(fa, vec);
    }
    if (force_fallback) {
        // testing: every tile fails the bound (|q| max|k| - s_self > limit)
        if (cudaMemsetAsync(cm, 0x7f, BH * sizeof(unsigned int), st) != cudaSuccess) {
            *msg = "cudaMemsetAsync failed";
            return WB_ECUDA;
        }
    }
    int rc;
    CUtensorMap tq, tk, tv;
    {
        // rows of fw bf16 / fp16; boxes of 64 columns (one 128-byte swizzle
        // atom), two per tile at fw = 128
        const uint64_t dims[3] = {(uint64_t)fw, (uint64_t)T, (uint64_t)BH};
        const uint64_t strides[2] = {(uint64_t)fw * 2, (uint64_t)T * fw * 2};
        const uint32_t box[3] = {64, 128, 1};
        if ((rc = make_tmap(&tq, qf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B, msg)) ||
            (rc = make_tmap(&tk, kf, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B, msg)) ||
            (rc = make_tmap(&tv, vh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_128B, msg)))
            return rc;
    }
    WbSeqView none{};
    AttnTcArgs aa{(int)BH, H, T, hd, n_qt, H, 0, (int)(BH * n_qt), m0, sp, cn, cm, none, o, E, sched, dev_err, 1,
                  DOT_BOUND_LIMIT, 0, tflag};
    if ((rc = fw == 64 ? launch_attn_tc<64, 64>(tq, tk, tv, aa, sm_count, st, msg)
                       : launch_attn_tc<128, 128>(tq, tk, tv, aa, sm_count, st, msg)))
        return rc;
    return launch_dot_attn_tiles(qkv, B, T, E, H, o, sched + 1, (int)(BH * n_qt), st, msg);
}

int tc_gemm_bf16(const __nv_bfloat16 *A, const __nv_bfloat16 *B, const float *bias, float *C, int M, int N, int K,
                 uint32_t *dev_err, cudaStream_t st, std::string *msg) {
    return launch_gemm(false, A, B, bias, C, M, N, K, N, dev_err, st, msg);
}

int tc_gemm_tf32(const float *A, const float *B, const float *bias, float *C, int M, int N, int K, uint32_t *dev_err,
                 cudaStream_t st, std::string *msg) {
    return launch_gemm(true, A, B, bias, C, M, N, K, N, dev_err, st, msg);
}

// x -> hi = bf16(x), lo = bf16(x - hi): the two terms of a bf16 split whose
// products hi.hi + lo.hi + hi.lo carry ~16 mantissa bits
__global__ void split_bf16_kernel(const float *__restrict__ x, long long n, __nv_bfloat16 *__restrict__ hi,
                                  __nv_bfloat16 *__restrict__ lo) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[i] = h;
        lo[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

int split_bf16(const float *x, long long n, __nv_bfloat16 *hi, __nv_bfloat16 *lo, cudaStream_t st) {
    if (n <= 0) return WB_OK;
    const int grid = (int)std::min<long long>(4 * 148, (n + 255) / 256);
    split_bf16_kernel<<<grid, 256, 0, st>>>(x, n, hi, lo);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

int tc_gemm_bf16x3(const __nv_bfloat16 *A_hi, const __nv_bfloat16 *A_lo, const __nv_bfloat16 *W_hi,
                   const __nv_bfloat16 *W_lo, const float *bias, float *C, int M, int N, int K, uint32_t *dev_err,
                   cudaStream_t st, std::string *msg) {
    int rc = launch_gemm(false, A_hi, W_hi, bias, C, M, N, K, N, dev_err, st, msg);
    if (!rc) rc = launch_gemm(false, A_lo, W_hi, nullptr, C, M, N, K, N, dev_err, st, msg, 0, 0, 1);
    if (!rc) rc = launch_gemm(false, A_hi, W_lo, nullptr, C, M, N, K, N, dev_err, st, msg, 0, 0, 1);
    return rc;
}

int tc_attn_forward(const TcLayerWeights &t, const float *x, int B, int T, bool use_content, float *y,
                    float *phases_out, Workspace *ws, uint32_t *dev_err, int sm_count, cudaStream_t st,
                    std::string *msg, int h0, int h1, bool add_bias) {
    const int H = t.H, hd = t.hd;
    if (h1 < 0) h1 = H;
    if (h0 < 0 || h1 > H || h0 >= h1) {
        *msg = "bad head range";
        return WB_EINVAL;
    }
    const int Hg = h1 - h0;
    if (Hg < H && ((size_t)h0 * hd * 4) % 16) {
        *msg = "a head range must start at a multiple of 4 columns (head_begin * head_dim)";
        return WB_ENOTSUP;
    }
    const long long R = (long long)B * T;
    if ((t.E * 2) % 16) {
        *msg = "n_embd must be a multiple of 8 for the tensor path";
        return WB_ENOTSUP;
    }
    if (hd > 128) {
        *msg = "WB_PATH_TENSOR supports head_dim <= 128";
        return WB_ENOTSUP;
    }
    Carve cv;
    const size_t o_rs = cv.take<float>(R * 2 * H);
    const size_t o_ct = cv.take<float>(use_content ? R * H * t.C : 1);
    const size_t o_th = cv.take<float>(R * H);
    const size_t o_bk = cv.take<uint8_t>(R * H);
    const size_t o_v = cv.take<float>(R * H * hd);
    const CoreLayout lay = core_layout(t, B, T, cv.off, Hg, use_content);
    if (ws_ensure(ws, lay.end, msg)) return WB_ENOMEM;
    char *w = (char *)ws->p;
    WbSeqView sv;
    sv.theta = (float *)(w + o_th);
    sv.bucket = (uint8_t *)(w + o_bk);
    sv.v = (float *)(w + o_v);
    sv.seq_stride = (long long)H * T;
    sv.cap = T;
    sv.slot = nullptr;
    float *content = use_content ? (float *)(w + o_ct) : nullptr;
    (void)o_rs;
    int rc = launch_proj_tc(t.proj, t.pw.wrs_t, t.pw.brs, t.pw.wv_t, t.pw.bv, x, B, T, sv, content, h0, Hg, dev_err, st, msg);
    if (rc) return rc;
    rc = tc_attention_core(t, sv, content, B, T, h0, Hg, add_bias, y, ws, lay, dev_err, sm_count, st, msg);
    if (rc) return rc;
    if (phases_out &&
        cudaMemcpyAsync(phases_out, sv.theta, R * H * sizeof(float), cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
        *msg = "phase copy failed";
        return WB_ECUDA;
    }
    return WB_OK;
}

int tc_kv_prefill(const TcLayerWeights &t, const WbSeqView &sv, const float *x, int n_seq, int T, float *y,
                  Workspace *ws, uint32_t *dev_err, int sm_count, cudaStream_t st, std::string *msg) {
    if (t.hd > 128) {
        *msg = "WB_PATH_TENSOR supports head_dim <= 128";
        return WB_ENOTSUP;
    }
    const long long R = (long long)n_seq * T;
    Carve cv;
    const size_t o_rs = cv.take<float>(R * 2 * t.H);
    const CoreLayout lay = core_layout(t, n_seq, T, cv.off, t.H, false);
    if (ws_ensure(ws, lay.end, msg)) return WB_ENOMEM;
    (void)o_rs;
    int rc = launch_proj_tc(t.proj, t.pw.wrs_t, t.pw.brs, t.pw.wv_t, t.pw.bv, x, n_seq, T, sv, nullptr, 0, t.H, dev_err, st, msg);
    if (rc) return rc;
    return tc_attention_core(t, sv, nullptr, n_seq, T, 0, t.H, true, y, ws, lay, dev_err, sm_count, st, msg);
}

// Rows from which the decode out_proj runs on the tensor-core GEMM (below
// it the SIMT kernel, launched as a programmatic dependent, is faster: 32
// rows take 9 us of a 27 us layer step on the SIMT kernel and 21 us on the
// 128x128-tile GEMM; 256 rows take 49 us on the SIMT kernel and 33 us on
// the GEMM, B200, graph-replayed steps).
static constexpr int kDecodeGemmMinRows = 64;
static int decode_gemm_min_rows() { return kDecodeGemmMinRows; }
int tc_decode_plain_store_rows() { return kDecodeGemmMinRows; }

int tc_kv_decode(const TcLayerWeights &t, const WbSeqView &sv, int32_t *len, int cap, int n_slots, const float *x,
                 int n_seq, float *y, void *scratch, size_t scratch_bytes, uint32_t *dev_err, int sm_count,
                 cudaStream_t st, std::string *msg, bool chain, bool *ends_with_out) {
    if (ends_with_out) *ends_with_out = false;
    if (t.hd > 128) {
        *msg = "fast decode supports head_dim <= 128";
        return WB_ENOTSUP;
    }
    DecodeLaunch L{sv, len, cap, n_slots, x, t.wrs_h, t.pw.brs, t.pw.wv_t, t.pw.bv, t.wo_t, t.b_o, t.harmonic_n,
                   n_seq, t.H, t.hd, t.E, sm_count, dev_err, chain};
    float *o = nullptr;
    int rc = launch_decode_attn(L, scratch, scratch_bytes, &o, st, msg);
    if (rc) return rc;
    if (n_seq >= decode_gemm_min_rows()) {
        // many rows: out_proj on the tcgen05 TF32 GEMM, then lengths += 1
        launch_len_update(len, sv.slot, n_seq, 1, 0, n_slots, cap, st, sv.pages, sv.max_pages);
        return launch_gemm(true, o, t.w_o32, t.b_o, y, n_seq, t.E, t.E, t.E, dev_err, st, msg);
    }
    // few rows: the SIMT out_proj kernel (programmatic dependent of the
    // attention grid), which also advances the lengths
    rc = launch_decode_out(o, t.wo_t, t.b_o, y, n_seq, t.E, cap, len, sv.slot, n_slots, st, msg, sv.pages,
                          sv.max_pages);
    if (rc == WB_OK && ends_with_out) *ends_with_out = true;
    return rc;
}

}  // namespace wb
