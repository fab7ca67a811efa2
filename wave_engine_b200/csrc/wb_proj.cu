// wb_proj.cu -- tensor-core projections for WB_PATH_TENSOR.
//
// One GEMM computes, for every row x (a position's n_embd vector), all the
// per-head projections of src/common/attn.rs:121-165:
//   columns [0, H*hd)            values   v = Wv_h x_h + b   (block diagonal)
//   columns [H*hd, H*hd + H*C)   content  c = Wc_h x + b      (C = 0 or 16)
//   columns [.., + 2H)           phase    (r, s) = Wp_h x + b
// (the phase columns are kept in W but computed by phase_fma_kernel below).
// The weight matrix W [N][E] holds the block-diagonal value weights densely
// (zeros outside a head's block); a 128-column tile that only holds value
// columns reads just the K range of its heads, so the zeros are not
// multiplied.
//
// Precision: 3xTF32.  Each operand is split into a tf32 head (round to
// nearest) and its fp32 remainder; on kind::tf32 tcgen05.mma the main
// products Ah Bh accumulate in one TMEM accumulator and the corrections
// Ah Bl + Al Bh -- about 2^-11 smaller -- in a second one, so the tensor
// core's accumulation does not drop the corrections' low bits against the
// large running sum; the epilogue adds the two in fp32.  Values and content
// come out with ~1e-6 relative error.  The phase (r, s) decides a discrete
// bucket, and the tensor core's own fp32 accumulation over hundreds of K
// steps still moves it by up to ~1e-4 rad, so phases are computed by a
// separate fp32 SIMT kernel (phase_fma_kernel) with a sequential sum over
// the input index like the reference's loop.  The weight halves are
// prepared on the host; the row halves are made in shared memory by two
// converter warps.
//
// Warp roles per CTA (128 x 128 output tile, 128 threads): warp 0 lane 0
// issues TMA loads (x tile, W head/remainder tiles) into a 3-stage ring,
// warp 1 lane 0 issues the MMAs, warps 2-3 split the x tile; then all four
// warps drain TMEM.  The epilogue writes values into the sequence view
// (cache layout), content rows densely, and turns (r, s) into the phase
// atan2f(s, r) and its bucket.
#include "wb_proj.h"
#include "wb_ptx.cuh"

#include <cudaTypedefs.h>

#include <cmath>
#include <cstring>
#include <vector>

namespace wb {

static constexpr int PBM = 128, PBN = 128, PBK = 32, PST = 3;
static constexpr int P_TILE = PBM * PBK * 4;      // 16 KB (128 rows x 128 B)
static constexpr int P_STAGE = 4 * P_TILE;        // A, A_lo, B_hi, B_lo
static constexpr int P_SMEM = PST * P_STAGE + 256 + 1024;

struct ProjArgs {
    int R, E, H, hd, C, T;
    int n_v, n_c, n_rs, N;  // column counts (n_v = H*hd, n_c = H*C, n_rs = 2H)
    int v0, v1, c0, c1;     // value and content column windows of the heads computed
    const float *bias;      // [N]
    WbSeqView sv;           // values, phases, buckets (rows r = b*T + t)
    float *content;         // [R][H*C] or nullptr
    uint32_t *dev_err;
};

__device__ __forceinline__ uint32_t tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

__global__ void __launch_bounds__(128, 1)
    proj_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_wh,
                   const __grid_constant__ CUtensorMap tm_wl, ProjArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + PST * P_STAGE);
    uint64_t *full = bars, *conv = bars + PST, *empty = bars + 2 * PST, *done = bars + 3 * PST;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * PST + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    // tiles: the value window in PBN-column steps, then the content window
    // (no content tiles without a content output, e.g. the serve prefill)
    const int n_vt = (a.v1 - a.v0 + PBN - 1) / PBN;
    const int n_ct = a.content ? (a.c1 - a.c0 + PBN - 1) / PBN : 0;
    const int n_tiles = n_vt + n_ct;
    const int nt = blockIdx.x % n_tiles, mt = blockIdx.x / n_tiles;
    const bool value_tile = nt < n_vt;
    const int n0 = value_tile ? a.v0 + nt * PBN : a.c0 + (nt - n_vt) * PBN;
    const int nend = value_tile ? min(a.v1, n0 + PBN) : min(a.c1, n0 + PBN);
    const int m0 = mt * PBM;
    // K range: value tiles need the inputs of their heads only
    int k_lo = 0, k_hi = a.E;
    if (value_tile) {
        k_lo = (n0 / a.hd) * a.hd;
        k_hi = min(a.E, ((nend + a.hd - 1) / a.hd) * a.hd);
    }
    const int kb0 = k_lo / PBK, kb1 = (k_hi + PBK - 1) / PBK, nk = kb1 - kb0;

    if (tid == 0) {
        for (int i = 0; i < 3 * PST + 1; i++) ptx::mbar_init(bars + i, 1);
        ptx::fence_mbar_init();
    }
    if (warp == 0) {
        ptx::tmem_alloc(tmem_slot, 256);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;           // main products
    const uint32_t tmem_c = tmem + PBN;         // corrections

    if (tid == 0) {  // TMA producer
        ptx::prefetch_tmap(&tm_x);
        ptx::prefetch_tmap(&tm_wh);
        ptx::prefetch_tmap(&tm_wl);
        for (int i = 0; i < nk; i++) {
            const int s = i % PST;
            if (i >= PST && !ptx::mbar_wait(empty + s, ((i / PST) - 1) & 1)) {
                atomicOr(a.dev_err, WB_DERR_TIMEOUT_MMA);
                break;
            }
            uint8_t *st = sm + s * P_STAGE;
            const int kx = (kb0 + i) * PBK;
            ptx::mbar_arrive_expect_tx(full + s, 3 * P_TILE);
            ptx::tma_load_2d(st, &tm_x, full + s, kx, m0);
            ptx::tma_load_2d(st + 2 * P_TILE, &tm_wh, full + s, kx, n0);
            ptx::tma_load_2d(st + 3 * P_TILE, &tm_wl, full + s, kx, n0);
        }
    } else if (tid == 32) {  // MMA issuer
        constexpr uint32_t IDESC = ptx::idesc_tf32(PBM, PBN);
        for (int i = 0; i < nk; i++) {
            const int s = i % PST;
            if (!ptx::mbar_wait(conv + s, (i / PST) & 1)) {
                atomicOr(a.dev_err, WB_DERR_TIMEOUT_TMA);
                break;
            }
            ptx::tc_fence_after();
            const uint32_t base = ptx::smem_u32(sm + s * P_STAGE);
            const uint32_t ah = base, al = base + P_TILE, bh = base + 2 * P_TILE, bl = base + 3 * P_TILE;
#pragma unroll
            for (int k = 0; k < 4; k++) {  // 8 tf32 = 32 bytes of K per instruction
                const uint64_t dah = ptx::smem_desc(ah + k * 32, 16, 1024, ptx::UMMA_SW128);
                const uint64_t dal = ptx::smem_desc(al + k * 32, 16, 1024, ptx::UMMA_SW128);
                const uint64_t dbh = ptx::smem_desc(bh + k * 32, 16, 1024, ptx::UMMA_SW128);
                const uint64_t dbl = ptx::smem_desc(bl + k * 32, 16, 1024, ptx::UMMA_SW128);
                ptx::mma_tf32(tmem, dah, dbh, IDESC, (i > 0 || k > 0));
                ptx::mma_tf32(tmem_c, dah, dbl, IDESC, (i > 0 || k > 0));
                ptx::mma_tf32(tmem_c, dal, dbh, IDESC, 1);
            }
            ptx::mma_commit(empty + s);
        }
        ptx::mma_commit(done);
    } else if (warp >= 2) {  // converters: x -> (tf32 head in place, remainder)
        const int ct = tid - 64;
        for (int i = 0; i < nk; i++) {
            const int s = i % PST;
            if (!ptx::mbar_wait(full + s, (i / PST) & 1)) {
                if (ct == 0) atomicOr(a.dev_err, WB_DERR_TIMEOUT_TMA);
                break;
            }
            float4 *A = reinterpret_cast<float4 *>(sm + s * P_STAGE);
            float4 *Al = reinterpret_cast<float4 *>(sm + s * P_STAGE + P_TILE);
#pragma unroll 4
            for (int e = ct; e < P_TILE / 16; e += 64) {
                const float4 v = A[e];
                float4 h, l;
                h.x = __uint_as_float(tf32_rna(v.x));
                h.y = __uint_as_float(tf32_rna(v.y));
                h.z = __uint_as_float(tf32_rna(v.z));
                h.w = __uint_as_float(tf32_rna(v.w));
                l.x = v.x - h.x;
                l.y = v.y - h.y;
                l.z = v.z - h.z;
                l.w = v.w - h.w;
                A[e] = h;
                Al[e] = l;
            }
            ptx::fence_proxy_async_smem();
            asm volatile("bar.sync 1, 64;" ::: "memory");
            if (ct == 0) ptx::mbar_arrive(conv + s);
        }
    }

    // epilogue: TMEM -> registers -> destinations by column kind
    const bool fin = ptx::mbar_wait(done, 0);
    if (!fin && tid == 0) atomicOr(a.dev_err, WB_DERR_TIMEOUT_MMA);
    ptx::tc_fence_after();
    if (fin) {
        // the pipeline stages are free (every MMA has completed): each warp
        // stages its 32 rows chunk by chunk and stores them row by row, lane
        // = column (a value row segment of one head, or a content row)
        float *buf = reinterpret_cast<float *>(sm) + warp * 32 * 33;
        const int lane = tid & 31;
        // this lane's row (for the per-row cache offsets, shuffled below)
        const int mr = m0 + warp * 32 + lane;
        const int br = mr / a.T, tr = mr - br * a.T;
        const long long row_off = mr < a.R ? wb_row(a.sv, br, tr) : -1;  // + h * cap per head; -1: no cache row
#pragma unroll 1
        for (int c = 0; c < PBN / 32; c++) {
            uint32_t r[32], rc[32];
            ptx::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c * 32, r);
            ptx::tmem_ld32(tmem_c + ((uint32_t)(warp * 32) << 16) + c * 32, rc);
            ptx::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i++) r[i] = __float_as_uint(__uint_as_float(r[i]) + __uint_as_float(rc[i]));
            warp_stage32(buf, r, lane);
            const int n = n0 + c * 32 + lane;
            const bool is_v = value_tile && n < nend, is_c = !value_tile && n < nend && a.content;
            const float bv = n < nend ? a.bias[n] : 0.0f;
            const int h = is_v ? n / a.hd : 0, d = is_v ? n - h * a.hd : 0;
            const long long hoff = (long long)h * a.sv.cap;
#pragma unroll 4
            for (int j = 0; j < 32; j++) {
                const int m = m0 + warp * 32 + j;
                const long long off = __shfl_sync(0xffffffffu, row_off, j);
                if (m >= a.R) continue;
                const float v = buf[j * 33 + lane] + bv;
                if (is_v) {
                    if (off >= 0) a.sv.v[(off + hoff) * a.hd + d] = v;
                }
                else if (is_c) a.content[(long long)m * a.n_c + (n - a.n_v)] = v;
            }
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 0) ptx::tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------
// Phases: (r, s) = b + sum_j W[.][j] x[j] in fp32, j in order (attn.rs:124-127
// with fused multiply-adds), then theta = atan2f(s, r) and its bucket
// (attn.rs:127, :171-174).  Every output keeps one sequential sum in one
// thread (the phase decides a discrete bucket, so the sum is not split).
// CTA = 128 rows x all 2H outputs, 256 threads: thread (row pair p, output
// group g) owns rows p and p + 64 and outputs g*OPT .. g*OPT + OPT - 1 (OPT
// = 2H / 4 rounded up to even: whole (r, s) pairs).  x arrives in chunks of
// PH_KC columns, staged in shared memory with rows padded to PH_KC + 1
// floats (the lanes of a warp read 32 rows of one column: conflict-free);
// the next chunk's loads are in flight while the current one is used.  The
// chunk's phase weights [PH_KC][2H] sit beside it (read as broadcasts).
// ---------------------------------------------------------------------------
static constexpr int PH_ROWS = 128, PH_THREADS = 256;

template <int OPT, int KC>
__global__ void __launch_bounds__(PH_THREADS, 3) phase_fma_kernel(const float *__restrict__ x,
                                                                const float *__restrict__ wrs_t,
                                                                const float *__restrict__ brs, int R, int E, int H,
                                                                int T, WbSeqView sv, int h0, int Hg) {
    constexpr int WST = 4 * OPT;                        // weight row stride: 4 groups x OPT outputs
    constexpr int RPL = PH_THREADS / KC;                // rows covered by one load instruction
    constexpr int XLD = PH_ROWS / RPL;                  // x loads per thread per chunk
    constexpr int WLD = (KC * WST + PH_THREADS - 1) / PH_THREADS;
    __shared__ float xs[2][PH_ROWS * (KC + 1)];
    __shared__ __align__(16) float ws[2][KC * WST];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.x * PH_ROWS;
    // outputs: (r, s) of heads h0 .. h0 + Hg - 1 (columns 2*h0 .. of the
    // [E][2H] weight rows)
    const int NO = 2 * Hg, NOT = 2 * H;
    wrs_t += 2 * h0;
    brs += 2 * h0;
    const int rp = tid % (PH_ROWS / 2), g = tid / (PH_ROWS / 2);
    const int o0 = g * OPT;
    float acc[2][OPT];
#pragma unroll
    for (int q = 0; q < OPT; q++) {
        const float b = o0 + q < NO ? brs[o0 + q] : 0.0f;
        acc[0][q] = b;
        acc[1][q] = b;
    }
    // this thread's x loads: column lc of rows lr, lr + RPL, ... (one base
    // pointer, constant stride); all of a chunk's loads go out together
    const int lc = tid % KC, lr = tid / KC;
    const long long xstride = (long long)RPL * E;
    float xv[XLD];
    float wv[WLD];
    auto load_chunk = [&](int k0) {
        const bool colok = k0 + lc < E;
        const float *xp = x + (long long)(m0 + lr) * E + k0 + lc;
#pragma unroll
        for (int u = 0; u < XLD; u++)
            xv[u] = (colok && m0 + lr + u * RPL < R) ? __ldg(xp + u * xstride) : 0.0f;
#pragma unroll
        for (int u = 0; u < WLD; u++) {
            const int e = u * PH_THREADS + tid;
            const int k = e / WST, o = e % WST;
            wv[u] = (e < KC * WST && k0 + k < E && o < NO) ? __ldg(wrs_t + (long long)(k0 + k) * NOT + o) : 0.0f;
        }
    };
    auto store_chunk = [&](int buf) {
#pragma unroll
        for (int u = 0; u < XLD; u++) xs[buf][(lr + u * RPL) * (KC + 1) + lc] = xv[u];
#pragma unroll
        for (int u = 0; u < WLD; u++) {
            const int e = u * PH_THREADS + tid;
            if (e < KC * WST) ws[buf][e] = wv[u];
        }
    };
    load_chunk(0);
    store_chunk(0);
    int buf = 0;
    for (int k0 = 0; k0 < E; k0 += KC) {
        __syncthreads();  // chunk `buf` stored; chunk buf ^ 1 free
        const bool more = k0 + KC < E;
        if (more) load_chunk(k0 + KC);
        const int kn = min(KC, E - k0);
        const float *x0 = xs[buf] + rp * (KC + 1);
        const float *x1 = xs[buf] + (rp + PH_ROWS / 2) * (KC + 1);
        const float *wr = ws[buf] + o0;
        for (int k = 0; k < kn; k++) {
            const float a0 = x0[k], a1 = x1[k];
#pragma unroll
            for (int q = 0; q < OPT; q += 2) {
                const float2 w = *reinterpret_cast<const float2 *>(wr + k * WST + q);
                acc[0][q] = fmaf(w.x, a0, acc[0][q]);
                acc[0][q + 1] = fmaf(w.y, a0, acc[0][q + 1]);
                acc[1][q] = fmaf(w.x, a1, acc[1][q]);
                acc[1][q + 1] = fmaf(w.y, a1, acc[1][q + 1]);
            }
        }
        if (more) store_chunk(buf ^ 1);
        buf ^= 1;
    }
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        const int m = m0 + rp + rr * (PH_ROWS / 2);
        if (m >= R) continue;
        const int b = m / T, t = m - b * T;
#pragma unroll
        for (int q = 0; q < OPT; q += 2) {
            const int hl = (o0 + q) / 2;
            if (hl >= Hg) break;
            const int h = h0 + hl;
            const float th = atan2f(acc[rr][q + 1], acc[rr][q]);
            const long long pos = wb_pos(sv, b, h, t);
            if (pos < 0) continue;
            sv.theta[pos] = th;
            sv.bucket[pos] = (uint8_t)phase_to_bucket(th);
        }
    }
}

// ---------------------------------------------------------------------------
// Values and phases in one fp32 pass over x, for head_dim 48 or 64 and at
// most 16 heads computed -- the serve models.  The value
// projection of a head is a 64x64 block on that head's 64 inputs
// (attn.rs:155-165): too little work per row for a tensor-core tile to pay
// for its pipeline, and exact in fp32 here.  CTA = 64 rows, 256 threads; the
// x columns are walked in rounds of two heads' inputs (128 columns), x
// staged transposed ([column][row]) in shared memory, the next round's x in
// registers and its weights in flight (cp.async) while the current round is
// used:
//   values: thread (head of the pair, 4 rows, 8 outputs), one sequential
//     fmaf sum per output over the head's inputs, + b (attn.rs:160-163);
//   phases: thread (2 rows, 4 of the 2H outputs = 2 whole (r, s) pairs),
//     b + the sequential fmaf sum over all E inputs, round after round in
//     input order -- the same order as phase_fma_kernel -- then atan2f and
//     the bucket.
// ---------------------------------------------------------------------------
static constexpr int VP_ROWS = 64, VP_THREADS = 256;
static constexpr int VP_KCH = 128;  // x columns per round (two heads of <= 64)
static constexpr int VP_XS = 68;    // floats per staged x column (64 rows + pad; 16-byte aligned)
static constexpr int VP_OPT = 4;    // phase outputs per thread
static constexpr int VP_NOP = 8 * VP_OPT;
static constexpr int VP_SMEM = (2 * VP_KCH * VP_XS + 2 * 2 * 64 * 64 + 2 * VP_KCH * VP_NOP) * 4;

struct VpArgs {
    const float *x;            // [R][E]
    const float *wv_t, *bv;    // [H][hd(in)][hd(out)], [H][hd]
    const float *wrs_t, *brs;  // [E][H][2], [H][2]
    int R, E, H, T, h0, Hg;
    WbSeqView sv;
};

// HD: head_dim (48 or 64).  Thread (value role) outputs d = 4*dg + j and
// 32 + 4*dg + j (j < 4): each of its two float4 weight loads and stores
// covers 128 contiguous bytes across the 8 lanes of one row.
template <int HD>
__global__ void __launch_bounds__(VP_THREADS, 1) vproj_phase_kernel(VpArgs a) {
    static_assert(HD % 4 == 0 && HD <= 64 && HD > 32, "value tiling assumes 32 < head_dim <= 64");
    extern __shared__ __align__(16) float vsm[];
    float *xs = vsm;                          // [2][KCH][XS]
    float *wsv = xs + 2 * VP_KCH * VP_XS;     // [2][2 heads][64 in][64 out]
    float *wrs = wsv + 2 * 2 * 64 * 64;       // [2][KCH][NOP]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m0 = blockIdx.x * VP_ROWS;
    const int E = a.E, H = a.H, NO = 2 * a.Hg;
    const int n_rounds = (H + 1) / 2;
    // value role: head 2p + hl, rows rg*4 .. +3, outputs 4*dg + j and 32 + 4*dg + j
    const int hl = tid >> 7, tq = tid & 127, rg = tq >> 3, dg = tq & 7;
    const bool hi_ok = 32 + 4 * dg < HD;  // the second output quad exists
    // phase role: rows 2*rp, 2*rp + 1, outputs g*OPT .. +OPT-1
    const int rp = lane, g = warp;
    // cache row indices (wb_row: + h * cap per head, -1 = none) of this thread's rows
    long long vrow[4], prow[2];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = m0 + rg * 4 + i;
        const int b = row < a.R ? row / a.T : 0, t = row - b * a.T;
        vrow[i] = row < a.R ? wb_row(a.sv, b, t) : -1;
    }
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const int row = m0 + 2 * rp + i;
        const int b = row < a.R ? row / a.T : 0, t = row - b * a.T;
        prow[i] = row < a.R ? wb_row(a.sv, b, t) : -1;
    }
    float ph[2][VP_OPT];
#pragma unroll
    for (int q = 0; q < VP_OPT; q++) {
        const int o = g * VP_OPT + q;
        const float b = o < NO ? __ldg(a.brs + 2 * a.h0 + o) : 0.0f;
        ph[0][q] = b;
        ph[1][q] = b;
    }
    // x: warp-instruction wi covers rows (wi & 7)*8 .. +7 and column quads
    // (wi >> 3)*4 .. +3 (64 contiguous bytes per row)
    float4 xr[8];
    auto load_x = [&](int p) {
        const int c0 = 2 * p * HD, kc = min(2, H - 2 * p) * HD;
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int wi = warp + 8 * u;
            const int r = (wi & 7) * 8 + (lane >> 2), k = ((wi >> 3) * 4 + (lane & 3)) * 4;
            const int row = m0 + r;
            xr[u] = (k < kc && row < a.R) ? __ldg(reinterpret_cast<const float4 *>(a.x + (long long)row * E + c0 + k))
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store_x = [&](int buf, int p) {
        const int kc = min(2, H - 2 * p) * HD;
        float *d = xs + buf * VP_KCH * VP_XS;
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int wi = warp + 8 * u;
            const int r = (wi & 7) * 8 + (lane >> 2), k = ((wi >> 3) * 4 + (lane & 3)) * 4;
            if (k < kc) {
                d[(k + 0) * VP_XS + r] = xr[u].x;
                d[(k + 1) * VP_XS + r] = xr[u].y;
                d[(k + 2) * VP_XS + r] = xr[u].z;
                d[(k + 3) * VP_XS + r] = xr[u].w;
            }
        }
    };
    auto load_w = [&](int buf, int p) {
        constexpr int Q4 = HD / 4, PER_HEAD = HD * Q4;  // float4 per weight row / per head
        const int c0 = 2 * p * HD, nh = min(2, H - 2 * p), kc = nh * HD;
        float *wv = wsv + buf * 2 * 64 * 64;
        for (int e = tid; e < nh * PER_HEAD; e += VP_THREADS) {
            const int hh = e / PER_HEAD, rem = e - hh * PER_HEAD, k = rem / Q4, dq = rem - k * Q4;
            ptx::cp_async<16>(wv + (hh * 64 + k) * 64 + dq * 4, a.wv_t + ((long long)(2 * p + hh) * HD + k) * HD + dq * 4);
        }
        // phase weights: column o = lane (o < 2*Hg <= 32), rows k = warp, warp + 8, ...
        float *wr = wrs + buf * VP_KCH * VP_NOP;
        if (lane < NO)
            for (int k = warp; k < kc; k += VP_THREADS / 32)
                ptx::cp_async<4>(wr + k * VP_NOP + lane, a.wrs_t + (long long)(c0 + k) * 2 * H + 2 * a.h0 + lane);
        ptx::cp_async_commit();
    };
    load_x(0);
    store_x(0, 0);
    load_w(0, 0);
    for (int p = 0; p < n_rounds; p++) {
        const int buf = p & 1;
        ptx::cp_async_wait<0>();
        __syncthreads();  // round p staged; the buffers of round p - 1 are free
        const bool more = p + 1 < n_rounds;
        if (more) {
            load_x(p + 1);
            load_w(buf ^ 1, p + 1);
        }
        const float *xb = xs + buf * VP_KCH * VP_XS;
        {  // phases: this round's inputs, in order
            const int kc = min(2, H - 2 * p) * HD;
            const float *wr = wrs + buf * VP_KCH * VP_NOP + g * VP_OPT;
            if (g * VP_OPT < NO)
#pragma unroll 4
                for (int k = 0; k < kc; k++) {
                    const float2 xv = *reinterpret_cast<const float2 *>(xb + k * VP_XS + 2 * rp);
                    const float4 w = *reinterpret_cast<const float4 *>(wr + k * VP_NOP);
                    ph[0][0] = fmaf(w.x, xv.x, ph[0][0]);
                    ph[0][1] = fmaf(w.y, xv.x, ph[0][1]);
                    ph[0][2] = fmaf(w.z, xv.x, ph[0][2]);
                    ph[0][3] = fmaf(w.w, xv.x, ph[0][3]);
                    ph[1][0] = fmaf(w.x, xv.y, ph[1][0]);
                    ph[1][1] = fmaf(w.y, xv.y, ph[1][1]);
                    ph[1][2] = fmaf(w.z, xv.y, ph[1][2]);
                    ph[1][3] = fmaf(w.w, xv.y, ph[1][3]);
                }
        }
        const int h = 2 * p + hl;
        if (h < H && h >= a.h0 && h < a.h0 + a.Hg) {  // values of head h
            float acc[4][8];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;
            const float *xh = xb + hl * HD * VP_XS + rg * 4;
            const float *wh = wsv + buf * 2 * 64 * 64 + hl * 64 * 64 + 4 * dg;
#pragma unroll 4
            for (int k = 0; k < HD; k++) {
                const float4 xv = *reinterpret_cast<const float4 *>(xh + k * VP_XS);
                const float4 w0 = *reinterpret_cast<const float4 *>(wh + k * 64);
                const float4 w1 = *reinterpret_cast<const float4 *>(wh + k * 64 + 32);
                const float xi[4] = {xv.x, xv.y, xv.z, xv.w};
                const float wj[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] = fmaf(wj[j], xi[i], acc[i][j]);
            }
            const float4 b0 = __ldg(reinterpret_cast<const float4 *>(a.bv + h * HD + 4 * dg));
            const float4 b1 = hi_ok ? __ldg(reinterpret_cast<const float4 *>(a.bv + h * HD + 32 + 4 * dg))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
            const long long hoff = (long long)h * a.sv.cap;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                if (vrow[i] < 0) continue;
                float *dst = a.sv.v + (vrow[i] + hoff) * HD + 4 * dg;
                *reinterpret_cast<float4 *>(dst) =
                    make_float4(acc[i][0] + b0.x, acc[i][1] + b0.y, acc[i][2] + b0.z, acc[i][3] + b0.w);
                if (hi_ok)
                    *reinterpret_cast<float4 *>(dst + 32) =
                        make_float4(acc[i][4] + b1.x, acc[i][5] + b1.y, acc[i][6] + b1.z, acc[i][7] + b1.w);
            }
        }
        if (more) store_x(buf ^ 1, p + 1);
    }
#pragma unroll
    for (int rr = 0; rr < 2; rr++) {
        if (prow[rr] < 0) continue;
#pragma unroll
        for (int q = 0; q < VP_OPT; q += 2) {
            const int hl2 = (g * VP_OPT + q) / 2;
            if (hl2 >= a.Hg) break;
            const int h = a.h0 + hl2;
            const float th = atan2f(ph[rr][q + 1], ph[rr][q]);
            const long long pos = prow[rr] + (long long)h * a.sv.cap;
            a.sv.theta[pos] = th;
            a.sv.bucket[pos] = (uint8_t)phase_to_bucket(th);
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
// ---------------------------------------------------------------------------
// Values and phases of a head_dim-64 layer, in one pass over x (attn.rs
// :121-130, :155-165; kv_cache.rs:129-142): vphase_tc_kernel.  A CTA owns
// 128 rows and walks x one head's 64 input columns at a time (chunk h),
// TMA'd into a 2-stage ring with the weights those inputs meet: head h's 64
// value rows and the 2H phase rows (r, s of every head), as tf32 heads and
// remainders.  One 3xTF32 tcgen05 MMA sequence per chunk (N = 64 + 32:
// main = xh Wh, corr = xh Wl + xl Wh) gives head h's values and every
// head's phase partial sums over the chunk's 64 inputs; the epilogue warps
// store the values and add the phase partials to fp32 running sums in input
// order (a 64-term tensor-core sum per chunk, then a sequential fp32 sum over
// the chunks), and after the last chunk turn (r, s) into phase and bucket.
//   warp 0: TMA producer; warp 1: MMA; warps 2-9: split x into tf32 head
//   (in place) and remainder; warps 10-13: epilogue (TMEM lane groups).
// ---------------------------------------------------------------------------
static constexpr int VT_ROWS = 128;
static constexpr int VT_THREADS = 14 * 32;
static constexpr int VT_N = 96;                    // 64 value + up to 32 phase outputs
static constexpr int VT_X = 128 * 64 * 4;          // x chunk (two 32-column SW128 atoms)
static constexpr int VT_WATOM = VT_N * 128;        // one K atom of the chunk's weights (96 rows)
static constexpr int VT_W = 2 * VT_WATOM;          // chunk weights, one precision
static constexpr int VT_STAGE = 2 * VT_X + 2 * VT_W;
static constexpr int VT_SMEM = 2 * VT_STAGE + 128 + 1024;
static_assert(VT_SMEM <= 232448, "vphase shared memory above the 227 KB limit");

struct VtArgs {
    int R, T, E;
    const float *bias;  // value biases [H*64] (ProjTcWeights bias rows 0..n_v)
    const float *brs;   // [H][2]
    WbSeqView sv;
    uint32_t *dev_err;
};

template <int H>
__global__ void __launch_bounds__(VT_THREADS, 1)
    vphase_tc_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_wh,
                     const __grid_constant__ CUtensorMap tm_wl, int phase_row0, VtArgs a) {
    static_assert(H % 4 == 0 && H <= 16, "heads per layer: a multiple of 4, at most 16");
    constexpr int NP = 2 * H;  // phase outputs (r, s per head)
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + 2 * VT_STAGE);
    uint64_t *full = bars, *conv = bars + 2, *empty = bars + 4, *vfull = bars + 6, *vfree = bars + 8;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 10);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * VT_ROWS;
    if (tid == 0) {
        for (int i = 0; i < 10; i++) ptx::mbar_init(bars + i, (bars + i == vfree || bars + i == vfree + 1) ? 128 : 1);
        ptx::fence_mbar_init();
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, 512);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    auto stage = [&](int s) { return sm + s * VT_STAGE; };

    if (warp == 0) {
        // ---------------- producer: x chunk, value rows of head h, phase rows
        if (lane == 0) {
            ptx::prefetch_tmap(&tm_x);
            ptx::prefetch_tmap(&tm_wh);
            ptx::prefetch_tmap(&tm_wl);
            for (int h = 0; h < H; h++) {
                const int s = h & 1;
                if (h >= 2 && !ptx::mbar_wait(empty + s, ((h - 2) >> 1) & 1)) {
                    atomicOr(a.dev_err, WB_DERR_TIMEOUT_MMA);
                    break;
                }
                uint8_t *st = stage(s);
                ptx::mbar_arrive_expect_tx(full + s, VT_X + 2 * VT_W);
                for (int t = 0; t < 2; t++) {
                    const int k = h * 64 + t * 32;
                    ptx::tma_load_2d(st + t * (VT_X / 2), &tm_x, full + s, k, m0);
                    uint8_t *wh = st + 2 * VT_X + t * VT_WATOM, *wl = wh + VT_W;
                    // rows 0-63: head h's value outputs; rows 64-95: the phase
                    // outputs of every head (zeros past the last row of W)
                    ptx::tma_load_2d(wh, &tm_wh, full + s, k, h * 64);
                    ptx::tma_load_2d(wh + 32 * 128, &tm_wh, full + s, k, h * 64 + 32);
                    ptx::tma_load_2d(wh + 64 * 128, &tm_wh, full + s, k, phase_row0);
                    ptx::tma_load_2d(wl, &tm_wl, full + s, k, h * 64);
                    ptx::tma_load_2d(wl + 32 * 128, &tm_wl, full + s, k, h * 64 + 32);
                    ptx::tma_load_2d(wl + 64 * 128, &tm_wl, full + s, k, phase_row0);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA: 3xTF32, N = 96 (values of head h | phase partials)
        if (lane == 0) {
            constexpr uint32_t IDESC = ptx::idesc_tf32(128, VT_N);
            for (int h = 0; h < H; h++) {
                const int s = h & 1, b = h & 1;
                if (!ptx::mbar_wait(conv + s, (h >> 1) & 1) ||
                    (h >= 2 && !ptx::mbar_wait(vfree + b, ((h - 2) >> 1) & 1))) {
                    atomicOr(a.dev_err, WB_DERR_TIMEOUT_TMA);
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t xh = ptx::smem_u32(stage(s)), xl = xh + VT_X;
                const uint32_t wh = xh + 2 * VT_X, wl = wh + VT_W;
                const uint32_t Dm = tmem + (uint32_t)(b * 256), Dc = Dm + 128;
                const uint64_t dah0 = ptx::smem_desc(xh, 16, 1024, ptx::UMMA_SW128);
                const uint64_t dal0 = ptx::smem_desc(xl, 16, 1024, ptx::UMMA_SW128);
                const uint64_t dbh0 = ptx::smem_desc(wh, 16, 1024, ptx::UMMA_SW128);
                const uint64_t dbl0 = ptx::smem_desc(wl, 16, 1024, ptx::UMMA_SW128);
#pragma unroll
                for (int t = 0; t < 2; t++)
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint64_t ao = (uint64_t)((t * (VT_X / 2) + k * 32) >> 4);
                        const uint64_t bo = (uint64_t)((t * VT_WATOM + k * 32) >> 4);
                        ptx::mma_tf32(Dm, dah0 + ao, dbh0 + bo, IDESC, (t > 0 || k > 0));
                        ptx::mma_tf32(Dc, dah0 + ao, dbl0 + bo, IDESC, (t > 0 || k > 0));
                        ptx::mma_tf32(Dc, dal0 + ao, dbh0 + bo, IDESC, 1);
                    }
                ptx::mma_commit(empty + s);
                ptx::mma_commit(vfull + b);
            }
        }
        __syncwarp();
    } else if (warp < 10) {
        // ---------------- workers: x -> tf32 head (in place) and remainder
        const int wt = tid - 64;  // 0..255
        for (int h = 0; h < H; h++) {
            const int s = h & 1;
            if (!ptx::mbar_wait(full + s, (h >> 1) & 1)) {
                if (wt == 0) atomicOr(a.dev_err, WB_DERR_TIMEOUT_TMA);
                break;
            }
            float4 *X = reinterpret_cast<float4 *>(stage(s));
            float4 *XL = reinterpret_cast<float4 *>(stage(s) + VT_X);
#pragma unroll 4
            for (int e = wt; e < VT_X / 16; e += 256) {
                const float4 v = X[e];
                float4 hi, lo;
                hi.x = __uint_as_float(tf32_rna(v.x));
                hi.y = __uint_as_float(tf32_rna(v.y));
                hi.z = __uint_as_float(tf32_rna(v.z));
                hi.w = __uint_as_float(tf32_rna(v.w));
                lo.x = v.x - hi.x;
                lo.y = v.y - hi.y;
                lo.z = v.z - hi.z;
                lo.w = v.w - hi.w;
                X[e] = hi;
                XL[e] = lo;
            }
            ptx::fence_proxy_async_smem();
            asm volatile("bar.sync 1, 256;" ::: "memory");
            if (wt == 0) ptx::mbar_arrive(conv + s);
        }
    } else {
        // ---------------- epilogue (warps 10-13: lane groups 2, 3, 0, 1)
        const int q = warp & 3;
        const int row = q * 32 + lane, m = m0 + row;
        const uint32_t lane_base = (uint32_t)(q * 32) << 16;
        long long base = -1;
        if (m < a.R) {
            const int b = m / a.T, t = m - b * a.T;
            base = wb_row(a.sv, b, t);
        }
        float acc[NP];
#pragma unroll
        for (int o = 0; o < NP; o++) acc[o] = __ldg(a.brs + o);
        bool ok = true;
        for (int h = 0; h < H; h++) {
            const int b = h & 1;
            if (!ptx::mbar_wait(vfull + b, (h >> 1) & 1)) {
                if (lane == 0) atomicOr(a.dev_err, WB_DERR_TIMEOUT_MMA);
                ok = false;
                break;
            }
            ptx::tc_fence_after();
            const uint32_t Dm = tmem + (uint32_t)(b * 256) + lane_base, Dc = Dm + 128;
            // phase partials of this chunk: columns 64 .. 64 + NP
            {
                uint32_t r[32], rc[32];
                ptx::tmem_ld32(Dm + 64, r);
                ptx::tmem_ld32(Dc + 64, rc);
                ptx::tmem_ld_wait();
#pragma unroll
                for (int o = 0; o < NP; o++) acc[o] += __uint_as_float(r[o]) + __uint_as_float(rc[o]);
            }
            // values of head h: columns 0 .. 63
            float *vrow = base >= 0 ? a.sv.v + (base + (long long)h * a.sv.cap) * 64 : nullptr;
#pragma unroll 1
            for (int c = 0; c < 2; c++) {
                uint32_t r[32], rc[32];
                ptx::tmem_ld32(Dm + c * 32, r);
                ptx::tmem_ld32(Dc + c * 32, rc);
                ptx::tmem_ld_wait();
                if (c == 1) {
                    ptx::tc_fence_before();
                    ptx::mbar_arrive(vfree + b);
                }
                if (vrow) {
                    const float4 *bias4 = reinterpret_cast<const float4 *>(a.bias + h * 64 + c * 32);
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float4 bv = __ldg(bias4 + i);
                        float4 v;
                        v.x = __uint_as_float(r[4 * i]) + __uint_as_float(rc[4 * i]) + bv.x;
                        v.y = __uint_as_float(r[4 * i + 1]) + __uint_as_float(rc[4 * i + 1]) + bv.y;
                        v.z = __uint_as_float(r[4 * i + 2]) + __uint_as_float(rc[4 * i + 2]) + bv.z;
                        v.w = __uint_as_float(r[4 * i + 3]) + __uint_as_float(rc[4 * i + 3]) + bv.w;
                        reinterpret_cast<float4 *>(vrow + c * 32)[i] = v;
                    }
                }
            }
        }
        // phases and buckets of every head of this row (attn.rs:127, :171-174)
        if (ok && base >= 0) {
#pragma unroll
            for (int hh = 0; hh < H; hh++) {
                const float th = atan2f(acc[2 * hh + 1], acc[2 * hh]);
                a.sv.theta[base + (long long)hh * a.sv.cap] = th;
                a.sv.bucket[base + (long long)hh * a.sv.cap] = (uint8_t)phase_to_bucket(th);
            }
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) ptx::tmem_dealloc(tmem, 512);
}

static PFN_cuTensorMapEncodeTiled_v12000 proj_encode_fn() {
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

static int tmap_2d_f32(CUtensorMap *m, const void *base, uint64_t inner, uint64_t outer, std::string *msg,
                       uint32_t box_rows = 128) {
    auto fn = proj_encode_fn();
    if (!fn) {
        *msg = "cuTensorMapEncodeTiled unavailable";
        return WB_ECUDA;
    }
    const uint64_t dims[2] = {inner, outer};
    const uint64_t strides[1] = {inner * 4};
    const uint32_t box[2] = {PBK, box_rows};
    const uint32_t es[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *msg = "cuTensorMapEncodeTiled (projection) failed with CUresult " + std::to_string((int)r);
        return WB_ECUDA;
    }
    return WB_OK;
}

static float tf32_round_host(float x) {  // round to nearest, ties away (cvt.rna)
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) != 0x7f800000u) {
        u += 0x1000u;
        u &= 0xffffe000u;
    }
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

int proj_weights_upload(ProjTcWeights *p, const wb_attn_weights_desc *w, std::string *msg) {
    const int E = w->n_embd, H = w->n_head, hd = E / H, C = w->content_dim;
    p->E = E;
    p->H = H;
    p->hd = hd;
    p->C = C;
    p->n_v = H * hd;
    p->n_c = H * C;
    p->n_rs = 2 * H;
    p->N = p->n_v + p->n_c + p->n_rs;
    const size_t N = p->N;
    std::vector<float> W(N * E, 0.0f), bias(N, 0.0f);
    for (int h = 0; h < H; h++)
        for (int d = 0; d < hd; d++) {
            const size_t row = (size_t)h * hd + d;
            for (int j = 0; j < hd; j++) W[row * E + h * hd + j] = w->v_proj_w[((size_t)h * hd + d) * hd + j];
            bias[row] = w->v_proj_b[h * hd + d];
        }
    for (int h = 0; h < H; h++)
        for (int c = 0; c < C; c++) {
            const size_t row = p->n_v + (size_t)h * C + c;
            std::memcpy(&W[row * E], w->content_proj_w + ((size_t)h * C + c) * E, sizeof(float) * E);
            bias[row] = w->content_proj_b[h * C + c];
        }
    for (int h = 0; h < H; h++)
        for (int k = 0; k < 2; k++) {
            const size_t row = p->n_v + p->n_c + (size_t)h * 2 + k;
            std::memcpy(&W[row * E], w->phase_proj_w + ((size_t)h * 2 + k) * E, sizeof(float) * E);
            bias[row] = w->phase_proj_b[h * 2 + k];
        }
    std::vector<float> Wh(N * E), Wl(N * E);
    for (size_t i = 0; i < N * E; i++) {
        Wh[i] = tf32_round_host(W[i]);
        Wl[i] = W[i] - Wh[i];
    }
    if (cudaMalloc(&p->w_hi, N * E * 4) != cudaSuccess || cudaMalloc(&p->w_lo, N * E * 4) != cudaSuccess ||
        cudaMalloc(&p->bias, N * 4) != cudaSuccess) {
        cudaGetLastError();
        *msg = "cudaMalloc for projection weights failed";
        return WB_ENOMEM;
    }
    if (cudaMemcpy(p->w_hi, Wh.data(), N * E * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(p->w_lo, Wl.data(), N * E * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(p->bias, bias.data(), N * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        *msg = "upload of projection weights failed";
        return WB_ECUDA;
    }
    return WB_OK;
}

void proj_weights_free(ProjTcWeights *p) {
    if (p->w_hi) cudaFree(p->w_hi);
    if (p->w_lo) cudaFree(p->w_lo);
    if (p->bias) cudaFree(p->bias);
    p->w_hi = p->w_lo = p->bias = nullptr;
}

int launch_proj_tc(const ProjTcWeights &p, const float *wrs_t, const float *brs, const float *wv_t, const float *bv,
                   const float *x, int B, int T, const WbSeqView &sv, float *content, int h0, int Hg,
                   uint32_t *dev_err, cudaStream_t st, std::string *msg) {
    const long long R = (long long)B * T;
    if (R <= 0) return WB_OK;
    const bool simt_v = wv_t && bv && (p.hd == 64 || p.hd == 48) && Hg <= 16 && R <= INT32_MAX &&
                        (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(bv) & 15) == 0;
    // head_dim 64: values and phases on the tensor cores.  Every chunk's MMA
    // covers all heads' phases, so a head range runs the whole layer (the
    // rows of other heads are written but not read): the same kernel and
    // the same numbers as the full forward
    const bool tc_v = simt_v && p.hd == 64 && (p.H == 8 || p.H == 12 || p.H == 16);
    if (tc_v) {
        // values (3xTF32 tcgen05) and phase partial sums in one pass
        CUtensorMap tx, twh, twl;
        int rc;
        if ((rc = tmap_2d_f32(&tx, x, (uint64_t)p.E, (uint64_t)R, msg))) return rc;
        // 32-row boxes: value rows load as two boxes of 32 (64 rows), phase rows as one
        if ((rc = tmap_2d_f32(&twh, p.w_hi, (uint64_t)p.E, (uint64_t)p.N, msg, 32))) return rc;
        if ((rc = tmap_2d_f32(&twl, p.w_lo, (uint64_t)p.E, (uint64_t)p.N, msg, 32))) return rc;
        VtArgs va{(int)R, T, p.E, p.bias, brs, sv, dev_err};
        const int phase_row0 = p.n_v + p.n_c;  // the 2H phase rows of W (the last rows: 32-row boxes read zeros past them)
        ProfScope ps("proj_vphase", st);
        const unsigned grid = (unsigned)((R + VT_ROWS - 1) / VT_ROWS);
        if (p.H == 8) {
            cudaFuncSetAttribute(vphase_tc_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, VT_SMEM);
            vphase_tc_kernel<8><<<grid, VT_THREADS, VT_SMEM, st>>>(tx, twh, twl, phase_row0, va);
        } else if (p.H == 12) {
            cudaFuncSetAttribute(vphase_tc_kernel<12>, cudaFuncAttributeMaxDynamicSharedMemorySize, VT_SMEM);
            vphase_tc_kernel<12><<<grid, VT_THREADS, VT_SMEM, st>>>(tx, twh, twl, phase_row0, va);
        } else {
            cudaFuncSetAttribute(vphase_tc_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, VT_SMEM);
            vphase_tc_kernel<16><<<grid, VT_THREADS, VT_SMEM, st>>>(tx, twh, twl, phase_row0, va);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            *msg = std::string("projection launch failed: ") + cudaGetErrorString(e);
            return WB_ECUDA;
        }
        if (!content) return WB_OK;
    } else if (simt_v) {
        // values and phases in one fp32 pass; the GEMM below keeps only the
        // content columns (if any)
        VpArgs va{x, wv_t, bv, wrs_t, brs, (int)R, p.E, p.H, T, h0, Hg, sv};
        ProfScope ps("proj_vphase", st);
        const unsigned grid = (unsigned)((R + VP_ROWS - 1) / VP_ROWS);
        if (p.hd == 64) {
            cudaFuncSetAttribute(vproj_phase_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, VP_SMEM);
            vproj_phase_kernel<64><<<grid, VP_THREADS, VP_SMEM, st>>>(va);
        } else {
            cudaFuncSetAttribute(vproj_phase_kernel<48>, cudaFuncAttributeMaxDynamicSharedMemorySize, VP_SMEM);
            vproj_phase_kernel<48><<<grid, VP_THREADS, VP_SMEM, st>>>(va);
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) {
            *msg = std::string("projection launch failed: ") + cudaGetErrorString(e);
            return WB_ECUDA;
        }
        if (!content) return WB_OK;
    }
    if ((p.E * 4) % 16) {
        *msg = "n_embd must be a multiple of 4 for the tensor projections";
        return WB_ENOTSUP;
    }
    CUtensorMap tx, th, tl;
    int rc;
    if ((rc = tmap_2d_f32(&tx, x, (uint64_t)p.E, (uint64_t)R, msg))) return rc;
    if ((rc = tmap_2d_f32(&th, p.w_hi, (uint64_t)p.E, (uint64_t)p.N, msg))) return rc;
    if ((rc = tmap_2d_f32(&tl, p.w_lo, (uint64_t)p.E, (uint64_t)p.N, msg))) return rc;
    if (p.H > 32) {
        *msg = "the tensor projections support up to 32 heads";
        return WB_ENOTSUP;
    }
    // GEMM over the value and content columns only (phases below)
    const int n_gemm = p.n_v + p.n_c;
    const int v0 = h0 * p.hd, v1 = simt_v ? v0 : (h0 + Hg) * p.hd, c0 = p.n_v + h0 * p.C,
              c1 = p.n_v + (h0 + Hg) * p.C;
    ProjArgs a{(int)R, p.E, p.H, p.hd, p.C, T, p.n_v, p.n_c, p.n_rs, n_gemm, v0, v1, c0, c1, p.bias, sv, content,
               dev_err};
    const int n_tiles = (v1 - v0 + PBN - 1) / PBN + (content ? (c1 - c0 + PBN - 1) / PBN : 0);
    const unsigned grid = (unsigned)(((R + PBM - 1) / PBM) * n_tiles);
    {
        ProfScope ps("proj_tc", st);
        cudaFuncSetAttribute(proj_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM);
        proj_tc_kernel<<<grid, 128, P_SMEM, st>>>(tx, th, tl, a);
    }
    if (!simt_v) {
        ProfScope pp("phase_fma", st);
        const unsigned pg = (unsigned)((R + PH_ROWS - 1) / PH_ROWS);
        if (Hg <= 12)
            phase_fma_kernel<6, 32><<<pg, PH_THREADS, 0, st>>>(x, wrs_t, brs, (int)R, p.E, p.H, T, sv, h0, Hg);
        else if (Hg <= 16)
            phase_fma_kernel<8, 32><<<pg, PH_THREADS, 0, st>>>(x, wrs_t, brs, (int)R, p.E, p.H, T, sv, h0, Hg);
        else
            phase_fma_kernel<16, 16><<<pg, PH_THREADS, 0, st>>>(x, wrs_t, brs, (int)R, p.E, p.H, T, sv, h0, Hg);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("projection launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

}  // namespace wb
