// wb_dot.cu -- causal multi-head dot-product attention core: the legacy
// attention of ComputeBackend::attention (src/common/compute.rs:357-414,
// attention_cpu; the same math as model_forward.rs:124-180), between the
// c_attn and c_proj projections.
//
// qkv [R][3E] (row r = b*T + t: q, k, v of all heads) -> o [R][E].  One CTA
// = 64 queries of one (sequence, head), TPQ threads per query (2 up to
// head_dim 64, 8 above: a thread's serial work over the keys is what bounds
// a CTA's latency, e.g. one listed fallback tile): query q0 + tid/TPQ, the
// TPQ threads of a query holding PT head dims each -- two threads: the lower
// and upper halves; eight: dims p, p+8, p+16, ... (p = tid % 8, interleaved
// so that a warp's shared-memory reads of one key row are conflict-free) --
// with q and the output accumulator in registers.  Keys go
// through shared memory in tiles of 32 (k and v rows of the head); per tile
// each thread forms the 32 scores (its partial dot plus its partners', an
// xor butterfly that gives all TPQ the same sum), takes the tile maximum,
// rescales its running output and sum once, and accumulates p v.  This is
// the reference's softmax(max-shifted) and weighted sum reorganised as an
// online softmax: the same result up to fp32 rounding (the reference's
// running order: scores, max over all keys, exp, sum, divide, p v).
#include "wave_b200.h"
#include "wb_internal.h"

#include <algorithm>

namespace wb {

static constexpr int DQ = 64;   // queries per CTA
static constexpr int DKT = 32;  // keys per shared-memory tile

// One CTA's 64 queries q0 .. q0+63 of (sequence b, head h); TPQ threads per
// query, PT head dims per thread (TPQ * PT >= head_dim).
template <int PT, int TPQ>
__device__ __forceinline__ void dot_attn_tile(const float *__restrict__ qkv, int T, int E, int hd, float scale,
                                              float *__restrict__ o, int qt, int h, int b,
                                              float (&ks)[DKT][TPQ * PT + 1], float (&vs)[DKT][TPQ * PT + 1]) {
    constexpr int W = TPQ * PT;   // padded head width in shared memory
    constexpr int DT = DQ * TPQ;  // threads per CTA
    const int tid = threadIdx.x, part = tid & (TPQ - 1);
    const int q0 = qt * DQ, q = q0 + tid / TPQ;
    const bool qok = q < T;
    const long long rs = 3LL * E;  // qkv row stride
    const float *base = qkv + (long long)b * T * rs;
    // head dim of this thread's i-th register (measured: contiguous halves
    // are faster for two threads per query, interleaving for eight)
    auto dim = [&](int i) { return TPQ == 2 ? part * PT + i : part + TPQ * i; };
    float qr[PT], acc[PT];
#pragma unroll
    for (int i = 0; i < PT; i++) {
        const int d = dim(i);
        qr[i] = (qok && d < hd) ? base[(long long)q * rs + h * hd + d] : 0.0f;
        acc[i] = 0.0f;
    }
    // the tile columns past head_dim are never loaded: zero them once (they
    // meet zero q entries and feed accumulators that are not stored)
    __syncthreads();  // the previous tile of this CTA consumed
    for (int e = tid; e < DKT * (W - hd); e += DT) {
        const int kk = e / (W - hd), d = hd + e % (W - hd);
        ks[kk][d] = 0.0f;
        vs[kk][d] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    const int kend = min(T, q0 + DQ);  // keys 0 .. kend-1 can be seen by this CTA
    for (int j0 = 0; j0 < kend; j0 += DKT) {
        __syncthreads();  // previous tile consumed
        for (int e = tid; e < DKT * hd; e += DT) {
            const int kk = e / hd, d = e - kk * hd;
            const int k = j0 + kk;
            const bool ok = k < kend;
            ks[kk][d] = ok ? base[(long long)k * rs + E + h * hd + d] : 0.0f;
            vs[kk][d] = ok ? base[(long long)k * rs + 2 * E + h * hd + d] : 0.0f;
        }
        __syncthreads();
        float s[DKT];
        float mt = -INFINITY;
#pragma unroll
        for (int kk = 0; kk < DKT; kk++) {
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < PT; i++) dot = fmaf(qr[i], ks[kk][dim(i)], dot);
#pragma unroll
            for (int x = 1; x < TPQ; x <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, x);
            const int k = j0 + kk;
            s[kk] = (qok && k <= q) ? dot * scale : -INFINITY;  // causal (compute.rs:381)
            mt = fmaxf(mt, s[kk]);
        }
        if (mt == -INFINITY) continue;  // no visible key in this tile
        const float mn = fmaxf(m, mt);
        const float c = expf(m - mn);  // 0 on the first visible tile (m = -inf)
        l *= c;
#pragma unroll
        for (int i = 0; i < PT; i++) acc[i] *= c;
        m = mn;
#pragma unroll
        for (int kk = 0; kk < DKT; kk++) {
            const float pr = expf(s[kk] - mn);  // 0 for masked keys
            l += pr;
#pragma unroll
            for (int i = 0; i < PT; i++) acc[i] = fmaf(pr, vs[kk][dim(i)], acc[i]);
        }
    }
    if (qok) {
        const float inv = 1.0f / l;
        float *dst = o + ((long long)b * T + q) * E + h * hd;
#pragma unroll
        for (int i = 0; i < PT; i++) {
            const int d = dim(i);
            if (d < hd) dst[d] = acc[i] * inv;
        }
    }
}

template <int PT, int TPQ>
__global__ void __launch_bounds__(DQ *TPQ) dot_attn_kernel(const float *__restrict__ qkv, int T, int E, int H, int hd,
                                                           float scale, float *__restrict__ o) {
    __shared__ float ks[DKT][TPQ * PT + 1];
    __shared__ float vs[DKT][TPQ * PT + 1];
    dot_attn_tile<PT, TPQ>(qkv, T, E, hd, scale, o, blockIdx.x, blockIdx.y, blockIdx.z, ks, vs);
}

// The 128-query tiles listed in tiles[1 .. tiles[0]] (entries bh * n_qt128
// + tile, bh = b * H + h), two 64-query halves each, over a grid-stride loop.
template <int PT, int TPQ>
__global__ void __launch_bounds__(DQ *TPQ) dot_attn_tiles_kernel(const float *__restrict__ qkv, int T, int E, int H,
                                                                 int hd, float scale, float *__restrict__ o,
                                                                 const int *__restrict__ tiles) {
    __shared__ float ks[DKT][TPQ * PT + 1];
    __shared__ float vs[DKT][TPQ * PT + 1];
    const int n = 2 * tiles[0];
    const int n_qt = (T + 2 * DQ - 1) / (2 * DQ);
    for (int e = blockIdx.x; e < n; e += gridDim.x) {
        const int tile = tiles[1 + (e >> 1)];
        const int bh = tile / n_qt, qt = 2 * (tile - bh * n_qt) + (e & 1);
        if (qt * DQ >= T) continue;  // uniform over the CTA
        dot_attn_tile<PT, TPQ>(qkv, T, E, hd, scale, o, qt, bh % H, bh / H, ks, vs);
    }
}

// (head dims per thread, threads per query): two threads per query with
// 8, 16, 24 or 32 dims each up to head_dim 64, eight with 16 each up to 128;
// 0 above
static int dot_cfg(int hd) {
    if (hd <= 16) return 8;
    if (hd <= 32) return 16;
    if (hd <= 48) return 24;
    if (hd <= 64) return 32;
    if (hd <= 128) return 128;
    return 0;
}

int launch_dot_attn(const float *qkv, int B, int T, int E, int H, float *o, cudaStream_t st, std::string *msg) {
    const int hd = E / H;
    const dim3 grid((T + DQ - 1) / DQ, H, B);
    const float scale = 1.0f / sqrtf((float)hd);  // compute.rs:362
    ProfScope ps("dot_attn", st);
    switch (dot_cfg(hd)) {
        case 8: dot_attn_kernel<8, 2><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o); break;
        case 16: dot_attn_kernel<16, 2><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o); break;
        case 24: dot_attn_kernel<24, 2><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o); break;
        case 32: dot_attn_kernel<32, 2><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o); break;
        case 128: dot_attn_kernel<16, 8><<<grid, 8 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o); break;
        default: *msg = "dot-product attention supports head_dim <= 128"; return WB_ENOTSUP;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("dot attention launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

int launch_dot_attn_tiles(const float *qkv, int B, int T, int E, int H, float *o, const int *tiles, int max_tiles,
                          cudaStream_t st, std::string *msg) {
    const int hd = E / H;
    const float scale = 1.0f / sqrtf((float)hd);
    const int grid = std::max(1, std::min(2 * max_tiles, 256));
    ProfScope ps("dot_attn_fallback", st);
    switch (dot_cfg(hd)) {
        case 8: dot_attn_tiles_kernel<8, 2><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles); break;
        case 16: dot_attn_tiles_kernel<16, 2><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles); break;
        case 24: dot_attn_tiles_kernel<24, 2><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles); break;
        case 32: dot_attn_tiles_kernel<32, 2><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles); break;
        case 128: dot_attn_tiles_kernel<16, 8><<<grid, 8 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles); break;
        default: *msg = "listed dot-product attention tiles support head_dim <= 128"; return WB_ENOTSUP;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("dot attention fallback launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

}  // namespace wb
