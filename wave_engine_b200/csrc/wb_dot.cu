// wb_dot.cu -- causal multi-head dot-product attention core: the legacy
// attention of ComputeBackend::attention (src/common/compute.rs:357-414,
// attention_cpu; the same math as model_forward.rs:124-180), between the
// c_attn and c_proj projections.
//
// qkv [R][3E] (row r = b*T + t: q, k, v of all heads) -> o [R][E].  One CTA
// = 64 queries of one (sequence, head), 128 threads: query q0 + tid/2, the
// two threads of a query holding one half of the head dims each (q and the
// output accumulator in registers).  Keys go through shared memory in tiles
// of 32 (k and v rows of the head); per tile each thread forms the 32 scores
// (its half-dot plus the partner's, one shuffle), takes the tile maximum,
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

// One CTA's 64 queries q0 .. q0+63 of (sequence b, head h).
template <int HALF>
__device__ __forceinline__ void dot_attn_tile(const float *__restrict__ qkv, int T, int E, int hd, float scale,
                                              float *__restrict__ o, int qt, int h, int b,
                                              float (&ks)[DKT][2 * HALF + 1], float (&vs)[DKT][2 * HALF + 1]) {
    const int tid = threadIdx.x, half = tid & 1;
    const int q0 = qt * DQ, q = q0 + (tid >> 1);
    const bool qok = q < T;
    const int d0 = half * HALF;
    const int nd = min(HALF, hd - d0);  // this thread's dims (the second half may be shorter)
    const long long rs = 3LL * E;       // qkv row stride
    const float *base = qkv + (long long)b * T * rs;
    float qr[HALF], acc[HALF];
#pragma unroll
    for (int d = 0; d < HALF; d++) {
        qr[d] = (qok && d < nd) ? base[(long long)q * rs + h * hd + d0 + d] : 0.0f;
        acc[d] = 0.0f;
    }
    // the tile columns past head_dim are never loaded: zero them once (a
    // thread's half past nd multiplies them by its zero q entries)
    __syncthreads();  // the previous tile of this CTA consumed
    for (int e = tid; e < DKT * (2 * HALF - hd); e += 2 * DQ) {
        const int kk = e / (2 * HALF - hd), d = hd + e % (2 * HALF - hd);
        ks[kk][d] = 0.0f;
        vs[kk][d] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    const int kend = min(T, q0 + DQ);  // keys 0 .. kend-1 can be seen by this CTA
    for (int j0 = 0; j0 < kend; j0 += DKT) {
        __syncthreads();  // previous tile consumed
        for (int e = tid; e < DKT * hd; e += 2 * DQ) {
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
            float part = 0.0f;
#pragma unroll
            for (int d = 0; d < HALF; d++) part = fmaf(qr[d], ks[kk][d0 + d], part);
            const float dot = part + __shfl_xor_sync(0xffffffffu, part, 1);
            const int k = j0 + kk;
            s[kk] = (qok && k <= q) ? dot * scale : -INFINITY;  // causal (compute.rs:381)
            mt = fmaxf(mt, s[kk]);
        }
        if (mt == -INFINITY) continue;  // no visible key in this tile
        const float mn = fmaxf(m, mt);
        const float c = expf(m - mn);  // 0 on the first visible tile (m = -inf)
        l *= c;
#pragma unroll
        for (int d = 0; d < HALF; d++) acc[d] *= c;
        m = mn;
#pragma unroll
        for (int kk = 0; kk < DKT; kk++) {
            const float p = expf(s[kk] - mn);  // 0 for masked keys
            l += p;
#pragma unroll
            for (int d = 0; d < HALF; d++) acc[d] = fmaf(p, vs[kk][d0 + d], acc[d]);
        }
    }
    if (qok) {
        const float inv = 1.0f / l;
        float *dst = o + ((long long)b * T + q) * E + h * hd + d0;
#pragma unroll
        for (int d = 0; d < HALF; d++)
            if (d < nd) dst[d] = acc[d] * inv;
    }
}

template <int HALF>
__global__ void __launch_bounds__(2 * DQ) dot_attn_kernel(const float *__restrict__ qkv, int T, int E, int H,
                                                          int hd, float scale, float *__restrict__ o) {
    __shared__ float ks[DKT][2 * HALF + 1];
    __shared__ float vs[DKT][2 * HALF + 1];
    dot_attn_tile<HALF>(qkv, T, E, hd, scale, o, blockIdx.x, blockIdx.y, blockIdx.z, ks, vs);
}

// The 128-query tiles listed in tiles[1 .. tiles[0]] (entries bh * n_qt128
// + tile, bh = b * H + h), two 64-query halves each, over a grid-stride loop.
template <int HALF>
__global__ void __launch_bounds__(2 * DQ) dot_attn_tiles_kernel(const float *__restrict__ qkv, int T, int E, int H,
                                                                int hd, float scale, float *__restrict__ o,
                                                                const int *__restrict__ tiles) {
    __shared__ float ks[DKT][2 * HALF + 1];
    __shared__ float vs[DKT][2 * HALF + 1];
    const int n = 2 * tiles[0];
    const int n_qt = (T + 2 * DQ - 1) / (2 * DQ);
    for (int e = blockIdx.x; e < n; e += gridDim.x) {
        const int tile = tiles[1 + (e >> 1)];
        const int bh = tile / n_qt, qt = 2 * (tile - bh * n_qt) + (e & 1);
        if (qt * DQ >= T) continue;  // uniform over the CTA
        dot_attn_tile<HALF>(qkv, T, E, hd, scale, o, qt, bh % H, bh / H, ks, vs);
    }
}

int launch_dot_attn(const float *qkv, int B, int T, int E, int H, float *o, cudaStream_t st, std::string *msg) {
    const int hd = E / H;
    const int half = (hd + 1) / 2;
    const dim3 grid((T + DQ - 1) / DQ, H, B);
    const float scale = 1.0f / sqrtf((float)hd);  // compute.rs:362
    ProfScope ps("dot_attn", st);
    if (half <= 8) dot_attn_kernel<8><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o);
    else if (half <= 16) dot_attn_kernel<16><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o);
    else if (half <= 24) dot_attn_kernel<24><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o);
    else if (half <= 32) dot_attn_kernel<32><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o);
    else if (half <= 64) dot_attn_kernel<64><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o);
    else {
        *msg = "dot-product attention supports head_dim <= 128";
        return WB_ENOTSUP;
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
    const int half = (hd + 1) / 2;
    const float scale = 1.0f / sqrtf((float)hd);
    const int grid = std::max(1, std::min(2 * max_tiles, 256));
    ProfScope ps("dot_attn_fallback", st);
    if (half <= 8) dot_attn_tiles_kernel<8><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles);
    else if (half <= 16) dot_attn_tiles_kernel<16><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles);
    else if (half <= 24) dot_attn_tiles_kernel<24><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles);
    else if (half <= 32) dot_attn_tiles_kernel<32><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles);
    else if (half <= 64) dot_attn_tiles_kernel<64><<<grid, 2 * DQ, 0, st>>>(qkv, T, E, H, hd, scale, o, tiles);
    else {
        *msg = "listed dot-product attention tiles support head_dim <= 128";
        return WB_ENOTSUP;
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("dot attention fallback launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

}  // namespace wb
