// wb_serve.cu -- the serve-tier layer around the attention on the GPU
// (src/common/kv_cache.rs prefill :93-236 and forward_one :241-381): token
// embedding, LayerNorm (model.rs:154), the dual-maestro Kerr-ODE FFN as the
// serve tier runs it (ffn.rs:39-230 with a frozen ODE, no memory and the
// stencil ODE of fft_ode.rs:171-250), its adaptive gain control (agc.rs), the
// parallel residual, and the decoders (phase_native_decode kv_cache.rs:18-33,
// lm_head :365-378).
//
// These are row-wise and small next to the attention: maestro_dim is 16 at
// the 768-dim scale, the ODE is 16 RK4 steps over n_bands coupled only to
// their 4 neighbours.  The kernels keep the reference's arithmetic order --
// sequential sums, products rounded before the add (__fmul_rn / __fadd_rn,
// no contraction) -- so the all-fp32 path differs from the reference only by
// the last bits of tanhf / sinf / cosf / expf / logf and by the order of the
// LayerNorm, maestro squeeze and AGC reductions.  The large products (the FFN's out_proj and
// the decoders' vocabulary GEMMs) run as bf16x3 products on the tcgen05 GEMM
// (wb_tc.cu) unless the caller asks for WB_PATH_EXACT.
#include "wave_b200.h"
#include "wb_internal.h"
#include "wb_serve.h"

#include <algorithm>
#include <cmath>

namespace wb {

#define FM __fmul_rn
#define FA __fadd_rn

// (r, s) pairs of the Kerr ODE as packed fp32x2 arithmetic: mul.rn / add.rn
// .f32x2 round each half exactly as the scalar __fmul_rn / __fadd_rn, so the
// results are those of the scalar statements beside each helper, with half
// the instructions (the ODE kernel is issue-bound).
// (o0, o1) = (FA(x0, FM(a, y0)), FA(x1, FM(a, y1)))
__device__ __forceinline__ void pair_axpy(float &o0, float &o1, float x0, float x1, float a, float y0, float y1) {
    asm("{\n .reg .b64 px, pa, py;\n mov.b64 px, {%2, %3};\n mov.b64 pa, {%4, %4};\n mov.b64 py, {%5, %6};\n"
        " mul.rn.f32x2 py, pa, py;\n add.rn.f32x2 px, px, py;\n mov.b64 {%0, %1}, px;\n}\n"
        : "=f"(o0), "=f"(o1)
        : "f"(x0), "f"(x1), "f"(a), "f"(y0), "f"(y1));
}
// (x0, x1) += FM(dt, FA(FA(FA(FM(w0, k1), FM(w1, k2)), FM(w2, k3)), FM(w3, k4))), per half
__device__ __forceinline__ void pair_rk4_combine(float &x0, float &x1, float dt, float w0, float w1, float w2, float w3,
                                                 float k1a, float k1b, float k2a, float k2b, float k3a, float k3b,
                                                 float k4a, float k4b) {
    asm("{\n .reg .b64 px, pw, pk, pt, pu;\n"
        " mov.b64 pw, {%3, %3};\n mov.b64 pk, {%7, %8};\n mul.rn.f32x2 pt, pw, pk;\n"
        " mov.b64 pw, {%4, %4};\n mov.b64 pk, {%9, %10};\n mul.rn.f32x2 pu, pw, pk;\n add.rn.f32x2 pt, pt, pu;\n"
        " mov.b64 pw, {%5, %5};\n mov.b64 pk, {%11, %12};\n mul.rn.f32x2 pu, pw, pk;\n add.rn.f32x2 pt, pt, pu;\n"
        " mov.b64 pw, {%6, %6};\n mov.b64 pk, {%13, %14};\n mul.rn.f32x2 pu, pw, pk;\n add.rn.f32x2 pt, pt, pu;\n"
        " mov.b64 pw, {%2, %2};\n mul.rn.f32x2 pt, pw, pt;\n"
        " mov.b64 px, {%0, %1};\n add.rn.f32x2 px, px, pt;\n mov.b64 {%0, %1}, px;\n}\n"
        : "+f"(x0), "+f"(x1)
        : "f"(dt), "f"(w0), "f"(w1), "f"(w2), "f"(w3), "f"(k1a), "f"(k1b), "f"(k2a), "f"(k2b), "f"(k3a), "f"(k3b),
          "f"(k4a), "f"(k4b));
}

// ---------------------------------------------------------------------------
// LayerNorm: one warp per row, the row staged in shared memory by one batch
// of loads, lane-strided partial sums combined by a fixed shuffle tree (mean,
// then the variance about it), y = (x - mean) / sd * w + b.
// ---------------------------------------------------------------------------
__global__ void layer_norm_kernel(const float *__restrict__ x, int rows, int n, const float *__restrict__ w,
                                  const float *__restrict__ b, float *__restrict__ y) {
    extern __shared__ float lrow[];  // [warps][n]: the row staged by one batch of loads
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= rows) return;
    const float *xr = x + row * n;
    float *sr = lrow + (long long)warp * n;
    if ((n & 3) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
        for (int i = lane; i < n / 4; i += 32) reinterpret_cast<float4 *>(sr)[i] = __ldg(reinterpret_cast<const float4 *>(xr) + i);
    } else {
        for (int i = lane; i < n; i += 32) sr[i] = __ldg(xr + i);
    }
    __syncwarp();
    float s = 0.0f;
    for (int i = lane; i < n; i += 32) s = FA(s, sr[i]);
#pragma unroll
    for (int o = 16; o; o >>= 1) s = FA(s, __shfl_xor_sync(0xffffffffu, s, o));
    const float mean = __fdiv_rn(s, (float)n);
    float v = 0.0f;
    for (int i = lane; i < n; i += 32) {
        const float d = __fsub_rn(sr[i], mean);
        v = FA(v, FM(d, d));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) v = FA(v, __shfl_xor_sync(0xffffffffu, v, o));
    const float sd = __fsqrt_rn(FA(__fdiv_rn(v, (float)n), 1e-5f));
    float *yr = y + row * n;
    for (int i = lane; i < n; i += 32) yr[i] = FA(FM(__fdiv_rn(__fsub_rn(sr[i], mean), sd), __ldg(w + i)), __ldg(b + i));
}

int launch_layer_norm(const float *x, int rows, int n, const float *w, const float *b, float *y, cudaStream_t st) {
    if (rows <= 0) return WB_OK;
    int warps = 8;
    while (warps > 1 && (size_t)warps * n * sizeof(float) > 96 * 1024) warps >>= 1;
    const size_t smem = (size_t)warps * n * sizeof(float);
    if (smem > 200 * 1024) return WB_ENOTSUP;
    ProfScope ps("layer_norm", st);
    cudaFuncSetAttribute(layer_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    layer_norm_kernel<<<(rows + warps - 1) / warps, warps * 32, smem, st>>>(x, rows, n, w, b, y);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

// ---------------------------------------------------------------------------
// Maestro (compute.rs:356-360 / ffn.rs:61-66, :185-191): y = base + process_1
// . gelu(squeeze . x), squeeze [M][E] and process_1 [E][M] with biases; each
// output bias + sum (compute.rs:441-452).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float gelu_ref(float v) {
    // compute.rs:113-119: 0.5 v (1 + tanh(c (v + 0.044715 v^3)))
    const float c = 0.7978845608f;
    const float inner = FM(c, FA(v, FM(FM(FM(0.044715f, v), v), v)));
    return FM(FM(0.5f, v), FA(1.0f, tanhf(inner)));
}

// A CTA takes MR rows (staged in shared memory).  squeeze: one warp per
// (row, m) output, lanes along the inputs, the lane partials combined by a
// fixed shuffle tree (deterministic; the squeeze sums differ from the
// reference's sequential order by rounding only), then bias + sum and GELU.
// process_1: one thread per (row, i) output, the M products summed in the
// reference's order, then bias + sum and the residual base.
static constexpr int MR = 4;  // most rows per CTA (1 when few rows: more CTAs)

__global__ void __launch_bounds__(256) maestro_kernel(MaestroArgs a, int mr) {
    extern __shared__ float msm[];
    const int E = a.E, M = a.M;
    float *xs = msm;                  // [MR][E]
    float *act = xs + (size_t)MR * E; // [MR][M]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const long long r0 = (long long)blockIdx.x * mr;
    const int nr = (int)min((long long)mr, a.rows - r0);
    const float *xg = a.x + r0 * E;
    if ((E & 3) == 0 && (reinterpret_cast<uintptr_t>(xg) & 15) == 0) {
        for (int e = threadIdx.x; e < nr * E / 4; e += blockDim.x)
            reinterpret_cast<float4 *>(xs)[e] = __ldg(reinterpret_cast<const float4 *>(xg) + e);
    } else {
        for (int e = threadIdx.x; e < nr * E; e += blockDim.x) xs[e] = __ldg(xg + e);
    }
    __syncthreads();
    for (int t = warp; t < nr * M; t += nw) {
        const int r = t / M, m = t - r * M;
        const float *wr = a.sq_w + (long long)m * E;
        const float *xr = xs + r * E;
        float s = 0.0f;
        for (int j0 = lane; j0 < E; j0 += 8 * 32) {  // 8 loads in flight, then the sums in order
            float wv[8];
#pragma unroll
            for (int u = 0; u < 8; u++) wv[u] = j0 + 32 * u < E ? __ldg(wr + j0 + 32 * u) : 0.0f;
#pragma unroll
            for (int u = 0; u < 8; u++)
                if (j0 + 32 * u < E) s = FA(s, FM(wv[u], xr[j0 + 32 * u]));
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) s = FA(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (lane == 0) act[r * M + m] = gelu_ref(FA(__ldg(a.sq_b + m), s));
    }
    __syncthreads();
    for (int e = threadIdx.x; e < nr * E; e += blockDim.x) {
        const int r = e / E, i = e - r * E;
        const float *wc = a.pr_wt + i;  // column i of the [M][E] copy: consecutive threads, consecutive words
        float s = 0.0f;
        for (int m0 = 0; m0 < M; m0 += 16) {  // 16 loads in flight, then the sums in order
            float wv[16];
#pragma unroll
            for (int u = 0; u < 16; u++) wv[u] = m0 + u < M ? __ldg(wc + (long long)(m0 + u) * E) : 0.0f;
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (m0 + u < M) s = FA(s, FM(wv[u], act[r * M + m0 + u]));
        }
        const float out = FA(__ldg(a.pr_b + i), s);
        const float base = a.base ? a.base[(r0 + r) * E + i] : xs[r * E + i];
        a.y[(r0 + r) * E + i] = FA(base, out);
    }
}

int launch_maestro(const MaestroArgs &a, cudaStream_t st) {
    if (a.rows <= 0) return WB_OK;
    const size_t smem = sizeof(float) * ((size_t)MR * a.E + (size_t)MR * a.M);
    if (smem > 200 * 1024) return WB_ENOTSUP;
    ProfScope ps("maestro", st);
    const int mr = a.rows >= 4 * 148 ? MR : 1;
    cudaFuncSetAttribute(maestro_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    maestro_kernel<<<(unsigned)((a.rows + mr - 1) / mr), 256, smem, st>>>(a, mr);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

// ---------------------------------------------------------------------------
// AGC (agc.rs:134-213).  A call's rows form n_seg consecutive segments, each
// one reference FFN call (one request's rows): per segment the statistics of
// the band magnitudes that pass the 2 x ceiling filter, then one thread
// applies the segments' EMA updates in order and records each segment's
// threshold, which the ODE kernel uses for the knee compression of that
// segment's rows.  Partial sums per block of a fixed grid, reduced in block
// order (deterministic).
// ---------------------------------------------------------------------------
static constexpr int AGC_THREADS = 256, AGC_MAXB = 148;

__device__ __forceinline__ float band_mag(const float *p) { return __fsqrt_rn(FA(FM(p[0], p[0]), FM(p[1], p[1]))); }

// partial layout per segment: [0, B) sums, [B, 2B) counts, [2B, 3B) sums of
// squared deviations, [3B] mean, [3B + 1] count, [3B + 2] variance (B =
// blocks per segment).
template <int PASS>
__global__ void __launch_bounds__(AGC_THREADS) agc_partial_kernel(const float *__restrict__ pre, long long seg_mags,
                                                                  const AgcDev *agc, float *partial) {
    __shared__ float ss[AGC_THREADS], sc[AGC_THREADS];
    const int B = gridDim.x, seg = blockIdx.y;
    float *ps = partial + (long long)seg * (3 * B + 3);
    const float *p = pre + (long long)seg * seg_mags * 2;
    const float ceil2 = FM(agc->max_threshold, 2.0f);
    const float mean = PASS == 1 ? ps[3 * B] : 0.0f;
    float s = 0.0f, c = 0.0f;
    for (long long i = blockIdx.x * (long long)AGC_THREADS + threadIdx.x; i < seg_mags;
         i += (long long)B * AGC_THREADS) {
        const float m = band_mag(p + 2 * i);
        if (isfinite(m) && m < ceil2) {
            if (PASS == 0) {
                s = FA(s, m);
                c = FA(c, 1.0f);
            } else {
                const float d = __fsub_rn(m, mean);
                s = FA(s, FM(d, d));
            }
        }
    }
    ss[threadIdx.x] = s;
    sc[threadIdx.x] = c;
    __syncthreads();
    for (int h = AGC_THREADS / 2; h; h >>= 1) {
        if (threadIdx.x < h) {
            ss[threadIdx.x] = FA(ss[threadIdx.x], ss[threadIdx.x + h]);
            sc[threadIdx.x] = FA(sc[threadIdx.x], sc[threadIdx.x + h]);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        if (PASS == 0) {
            ps[blockIdx.x] = ss[0];
            ps[B + blockIdx.x] = sc[0];
        } else {
            ps[2 * B + blockIdx.x] = ss[0];
        }
    }
}

// one warp per segment: the fixed-order sum of its B block partials (PASS 0:
// sums and counts -> mean and count; PASS 1: squared deviations -> var)
template <int PASS>
__global__ void agc_reduce_kernel(float *partial, int n_seg, int B) {
    const int lane = threadIdx.x & 31;
    const int seg = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (seg >= n_seg) return;
    float *ps = partial + (long long)seg * (3 * B + 3);
    float s = 0.0f, c = 0.0f;
    for (int i = lane; i < B; i += 32) {
        if (PASS == 0) {
            s = FA(s, ps[i]);
            c = FA(c, ps[B + i]);
        } else {
            s = FA(s, ps[2 * B + i]);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        s = FA(s, __shfl_xor_sync(0xffffffffu, s, o));
        c = FA(c, __shfl_xor_sync(0xffffffffu, c, o));
    }
    if (lane == 0) {
        if (PASS == 0) {
            ps[3 * B + 1] = c;
            ps[3 * B] = c > 0.0f ? __fdiv_rn(s, c) : 0.0f;
        } else {
            ps[3 * B + 2] = ps[3 * B + 1] > 0.0f ? __fdiv_rn(s, ps[3 * B + 1]) : 0.0f;
        }
    }
}

// one thread: the segments' observations in order (agc.rs observe), each
// segment's threshold recorded for its compression
__global__ void agc_update_kernel(const float *partial, int n_seg, int B, AgcDev *agc, float *thresholds) {
    if (threadIdx.x || blockIdx.x) return;
    for (int seg = 0; seg < n_seg; seg++) {
        const float *ps = partial + (long long)seg * (3 * B + 3);
        const float c = ps[3 * B + 1];
        if (c > 0.0f) {  // no clean magnitude: the state stays
            const float mean = ps[3 * B], var = ps[3 * B + 2];
            if (isfinite(mean) && isfinite(var)) {
                agc->count += 1;
                if (agc->count < 10) {
                    agc->ema_mean = mean;
                    agc->ema_var = var;
                } else {
                    agc->ema_mean = FA(FM(agc->decay, agc->ema_mean), FM(__fsub_rn(1.0f, agc->decay), mean));
                    agc->ema_var = FA(FM(agc->decay, agc->ema_var), FM(__fsub_rn(1.0f, agc->decay), var));
                }
                const float sd = fmaxf(__fsqrt_rn(agc->ema_var), 0.01f);
                agc->threshold =
                    fminf(fmaxf(FA(agc->ema_mean, FM(agc->headroom, sd)), agc->min_threshold), agc->max_threshold);
            }
        }
        thresholds[seg] = agc->threshold;
    }
}

// requests small enough for one block: both passes inside the block, the
// block tree in a fixed order (deterministic), mean / count / variance
// written where agc_update_kernel reads them (B = 1 layout)
__global__ void __launch_bounds__(AGC_THREADS) agc_small_kernel(const float *__restrict__ pre, long long seg_mags,
                                                                const AgcDev *agc, float *partial) {
    __shared__ float ss[AGC_THREADS], sc[AGC_THREADS];
    const int seg = blockIdx.x;
    float *ps = partial + (long long)seg * 6;  // 3 * B + 3 with B = 1
    const float *p = pre + (long long)seg * seg_mags * 2;
    const float ceil2 = FM(agc->max_threshold, 2.0f);
    float s = 0.0f, c = 0.0f;
    for (long long i = threadIdx.x; i < seg_mags; i += AGC_THREADS) {
        const float m = band_mag(p + 2 * i);
        if (isfinite(m) && m < ceil2) {
            s = FA(s, m);
            c = FA(c, 1.0f);
        }
    }
    ss[threadIdx.x] = s;
    sc[threadIdx.x] = c;
    __syncthreads();
    for (int h = AGC_THREADS / 2; h; h >>= 1) {
        if (threadIdx.x < h) {
            ss[threadIdx.x] = FA(ss[threadIdx.x], ss[threadIdx.x + h]);
            sc[threadIdx.x] = FA(sc[threadIdx.x], sc[threadIdx.x + h]);
        }
        __syncthreads();
    }
    const float cnt = sc[0];
    const float mean = cnt > 0.0f ? __fdiv_rn(ss[0], cnt) : 0.0f;
    __syncthreads();
    float v = 0.0f;
    for (long long i = threadIdx.x; i < seg_mags; i += AGC_THREADS) {
        const float m = band_mag(p + 2 * i);
        if (isfinite(m) && m < ceil2) {
            const float d = __fsub_rn(m, mean);
            v = FA(v, FM(d, d));
        }
    }
    ss[threadIdx.x] = v;
    __syncthreads();
    for (int h = AGC_THREADS / 2; h; h >>= 1) {
        if (threadIdx.x < h) ss[threadIdx.x] = FA(ss[threadIdx.x], ss[threadIdx.x + h]);
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        ps[3] = mean;
        ps[4] = cnt;
        ps[5] = cnt > 0.0f ? __fdiv_rn(ss[0], cnt) : 0.0f;
    }
}

static int agc_blocks(long long seg_mags) {
    return (int)std::max(1LL, std::min((long long)AGC_MAXB, (seg_mags + 8LL * AGC_THREADS - 1) / (8LL * AGC_THREADS)));
}

size_t agc_scratch_floats(int n_seg, long long seg_mags) {
    return (size_t)n_seg * (3 * agc_blocks(seg_mags) + 3) + (size_t)n_seg;
}

int launch_agc_observe(const float *pre, int n_seg, long long seg_mags, AgcDev *agc, float *scratch,
                       float **thresholds, cudaStream_t st) {
    const int B = agc_blocks(seg_mags);
    float *partial = scratch;
    *thresholds = scratch + (size_t)n_seg * (3 * B + 3);
    if (n_seg <= 0) return WB_OK;
    if (n_seg > 65535) return WB_EINVAL;
    ProfScope ps("agc", st);
    if (B == 1) {  // small requests (a decode step): two launches
        agc_small_kernel<<<n_seg, AGC_THREADS, 0, st>>>(pre, seg_mags, agc, partial);
        agc_update_kernel<<<1, 32, 0, st>>>(partial, n_seg, B, agc, *thresholds);
        return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
    }
    const dim3 grid(B, n_seg);
    const unsigned rgrid = (unsigned)((n_seg + 7) / 8);
    agc_partial_kernel<0><<<grid, AGC_THREADS, 0, st>>>(pre, seg_mags, agc, partial);
    agc_reduce_kernel<0><<<rgrid, 256, 0, st>>>(partial, n_seg, B);
    agc_partial_kernel<1><<<grid, AGC_THREADS, 0, st>>>(pre, seg_mags, agc, partial);
    agc_reduce_kernel<1><<<rgrid, 256, 0, st>>>(partial, n_seg, B);
    agc_update_kernel<<<1, 32, 0, st>>>(partial, n_seg, B, agc, *thresholds);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

// ---------------------------------------------------------------------------
// Kerr ODE (fft_ode.rs:171-250 kerr_ode_fft): one CTA per position, threads
// over bands (BPT bands each), the precond compressed by its segment's AGC
// threshold on load, rk4_steps RK4 steps whose derivative reads the
// neighbours' |z|^2 from shared memory -- the plain stencil (fft_ode.rs:
// 123-141) below 256 bands, the FFT convolution's circular indexing over
// next_pow2(n_bands) zero-padded points from 256 on -- then the corrector
// plate (ffn.rs:162-181).
// ---------------------------------------------------------------------------
template <int BPT>
__global__ void __launch_bounds__(1024) kerr_ode_kernel(OdeArgs a) {
    extern __shared__ float msq[];  // [n_bands]
    const int n = a.n_bands;
    const long long row = blockIdx.x;
    const float *pre = a.pre + row * 2 * n;
    const float thr = a.thresholds[row / a.rows_per_seg];
    const float dt = __fdiv_rn(1.0f, (float)a.steps);
    const float hdt = FM(0.5f, dt);
    const float w0 = a.rk4_w[0], w1 = a.rk4_w[1], w2 = a.rk4_w[2], w3 = a.rk4_w[3];
    float r[BPT], s[BPT], g[BPT], om[BPT];
    float k1r[BPT], k1s[BPT], k2r[BPT], k2s[BPT], k3r[BPT], k3s[BPT], k4r[BPT], k4s[BPT];
#pragma unroll
    for (int u = 0; u < BPT; u++) {
        const int k = threadIdx.x + u * blockDim.x;
        r[u] = s[u] = g[u] = om[u] = 0.0f;
        if (k < n) {
            r[u] = pre[2 * k];
            s[u] = pre[2 * k + 1];
            const float mag = __fsqrt_rn(FA(FM(r[u], r[u]), FM(s[u], s[u])));
            if (mag > thr && mag > 0.001f) {  // agc.rs knee_compress
                const float comp = FA(thr, FM(thr, tanhf(__fdiv_rn(__fsub_rn(mag, thr), thr))));
                const float scale = __fdiv_rn(comp, mag);
                r[u] = FM(r[u], scale);
                s[u] = FM(s[u], scale);
            }
            g[u] = softplus_ref(a.gamma_raw[k]);
            om[u] = a.omega[k];
        }
    }
    // each band's four neighbours (k-2, k-1, k+1, k+2) as shared-memory
    // indices, -1 where the stencil has no neighbour: the plain stencil's
    // edges, or a circular index landing in the FFT's zero padding
    const int L = a.fft_len;
    int nb[BPT][4];
#pragma unroll
    for (int u = 0; u < BPT; u++) {
        const int k = threadIdx.x + u * blockDim.x;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int j = k + (q < 2 ? q - 2 : q - 1);
            const int jj = L ? (j & (L - 1)) : j;  // L is a power of two: the circular index
            nb[u][q] = (k < n && jj >= 0 && jj < n) ? jj : -1;
        }
    }
    auto eval = [&](const float(&vr)[BPT], const float(&vs)[BPT], float(&dr)[BPT], float(&ds)[BPT]) {
#pragma unroll
        for (int u = 0; u < BPT; u++) {
            const int k = threadIdx.x + u * blockDim.x;
            if (k < n) msq[k] = FA(FM(vr[u], vr[u]), FM(vs[u], vs[u]));
        }
        __syncthreads();
#pragma unroll
        for (int u = 0; u < BPT; u++) {
            const int k = threadIdx.x + u * blockDim.x;
            if (k >= n) continue;
            float ns = 0.0f;
#pragma unroll
            for (int q = 0; q < 4; q++)
                if (nb[u][q] >= 0) ns = FA(ns, msq[nb[u][q]]);
            const float phi = FA(FA(om[u], FM(a.alpha, msq[k])), FM(a.beta, ns));
            dr[u] = __fsub_rn(FM(-g[u], vr[u]), FM(phi, vs[u]));
            ds[u] = FA(FM(-g[u], vs[u]), FM(phi, vr[u]));
        }
        __syncthreads();  // msq is rewritten by the next evaluation
    };
    float rt[BPT], st[BPT];
    for (int step = 0; step < a.steps; step++) {
        eval(r, s, k1r, k1s);
#pragma unroll
        for (int u = 0; u < BPT; u++) pair_axpy(rt[u], st[u], r[u], s[u], hdt, k1r[u], k1s[u]);
        eval(rt, st, k2r, k2s);
#pragma unroll
        for (int u = 0; u < BPT; u++) pair_axpy(rt[u], st[u], r[u], s[u], hdt, k2r[u], k2s[u]);
        eval(rt, st, k3r, k3s);
#pragma unroll
        for (int u = 0; u < BPT; u++) pair_axpy(rt[u], st[u], r[u], s[u], dt, k3r[u], k3s[u]);
        eval(rt, st, k4r, k4s);
#pragma unroll
        for (int u = 0; u < BPT; u++)
            // r += FM(dt, FA(FA(FA(FM(w0, k1r), FM(w1, k2r)), FM(w2, k3r)), FM(w3, k4r))), s likewise
            pair_rk4_combine(r[u], s[u], dt, w0, w1, w2, w3, k1r[u], k1s[u], k2r[u], k2s[u], k3r[u], k3s[u], k4r[u],
                             k4s[u]);
    }
    float *out = a.out + row * 2 * n;
#pragma unroll
    for (int u = 0; u < BPT; u++) {
        const int k = threadIdx.x + u * blockDim.x;
        if (k >= n) continue;
        float ro = r[u], so = s[u];
        if (a.corrector) {
            const float sc = sinf(a.corrector[k]), cc = cosf(a.corrector[k]);
            ro = __fsub_rn(FM(r[u], cc), FM(s[u], sc));
            so = FA(FM(r[u], sc), FM(s[u], cc));
        }
        out[2 * k] = ro;
        out[2 * k + 1] = so;
    }
}

int launch_kerr_ode(const OdeArgs &a, long long rows, cudaStream_t st) {
    if (rows <= 0) return WB_OK;
    const int n = a.n_bands;
    int bpt = 1;
    while (n > 1024 * bpt && bpt < 4) bpt *= 2;
    if (n > 1024 * bpt) return WB_ENOTSUP;
    if (rows > 0x7fffffffLL) return WB_EINVAL;
    const int threads = std::max(32, std::min(1024, ((n + bpt - 1) / bpt + 31) / 32 * 32));
    const size_t smem = sizeof(float) * (size_t)n;
    ProfScope ps("kerr_ode", st);
    if (bpt == 1) kerr_ode_kernel<1><<<(unsigned)rows, threads, smem, st>>>(a);
    else if (bpt == 2) kerr_ode_kernel<2><<<(unsigned)rows, threads, smem, st>>>(a);
    else kerr_ode_kernel<4><<<(unsigned)rows, threads, smem, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

// ---------------------------------------------------------------------------
// out_proj (out_proj.rs:24-40) on the exact path: dense y = b + sum (one
// thread per output, sequential over the inputs), block-diagonal with the
// sum started at the group's bias.
// ---------------------------------------------------------------------------
__global__ void out_proj_exact_kernel(const float *__restrict__ x, long long rows, int E, int groups,
                                      const float *__restrict__ w, const float *__restrict__ b, float *__restrict__ y) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= rows * E) return;
    const long long r = i / E;
    const int o = (int)(i - r * E);
    const float *xr = x + r * E;
    if (groups <= 1) {
        const float *wr = w + (long long)o * E;
        float s = 0.0f;
        for (int j = 0; j < E; j++) s = FA(s, FM(wr[j], xr[j]));
        y[i] = FA(b[o], s);
    } else {
        const int gs = E / groups, gi = o / gs, oi = o - gi * gs;
        const float *gw = w + (long long)gi * ((long long)gs * gs + gs);
        float s = gw[(long long)gs * gs + oi];
        const float *wr = gw + (long long)oi * gs;
        for (int j = 0; j < gs; j++) s = FA(s, FM(wr[j], xr[gi * gs + j]));
        y[i] = s;
    }
}

int launch_out_proj_exact(const float *x, long long rows, int E, int groups, const float *w, const float *b, float *y,
                          cudaStream_t st) {
    const long long n = rows * E;
    if (n <= 0) return WB_OK;
    ProfScope ps("ffn_out_proj", st);
    out_proj_exact_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, rows, E, groups, w, b, y);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

// ---------------------------------------------------------------------------
// Residual, embedding, decoders.
// ---------------------------------------------------------------------------
__global__ void residual_kernel(float *__restrict__ h, const float *__restrict__ a, const float *__restrict__ b,
                                long long n) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i < n) h[i] = FA(h[i], FA(a[i], b[i]));  // kv_cache.rs:220: hidden += attn + ffn
}

int launch_residual(float *h, const float *a, const float *b, long long n, cudaStream_t st) {
    if (n <= 0) return WB_OK;
    residual_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(h, a, b, n);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

__global__ void embed_kernel(const int32_t *__restrict__ tok, const int32_t *__restrict__ widx, int rows, int E,
                             const float *__restrict__ wte, int vocab, const float *__restrict__ wpe, int n_pos,
                             float *__restrict__ out, uint32_t *dev_err) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)rows * E) return;
    const int r = (int)(i / E), j = (int)(i - (long long)r * E);
    const int t = tok[r];
    if (t < 0 || t >= vocab) {
        if (j == 0) atomicOr(dev_err, WB_DERR_BOUNDS);
        out[i] = 0.0f;
        return;
    }
    float v = wte[(long long)t * E + j];
    const int p = widx[r];
    if (wpe && p >= 0 && p < n_pos) v = FA(v, wpe[(long long)p * E + j]);
    out[i] = v;
}

int launch_embed(const int32_t *tok, const int32_t *widx, int rows, int E, const float *wte, int vocab,
                 const float *wpe, int n_pos, float *out, uint32_t *dev_err, cudaStream_t st) {
    const long long n = (long long)rows * E;
    if (n <= 0) return WB_OK;
    embed_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(tok, widx, rows, E, wte, vocab, wpe, n_pos, out,
                                                             dev_err);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

// phase_native_decode's corrector rotation (kv_cache.rs:19-26) of rows
// [rows][2 n_bands].
__global__ void rotate_bands_kernel(const float *__restrict__ x, long long rows, int n_bands,
                                    const float *__restrict__ corr, float *__restrict__ y) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= rows * n_bands) return;
    const int k = (int)(i % n_bands);
    const float sc = sinf(corr[k]), cc = cosf(corr[k]);
    const float r = x[2 * i], s = x[2 * i + 1];
    y[2 * i] = __fsub_rn(FM(r, cc), FM(s, sc));
    y[2 * i + 1] = FA(FM(r, sc), FM(s, cc));
}

int launch_rotate_bands(const float *x, long long rows, int n_bands, const float *corr, float *y, cudaStream_t st) {
    const long long n = rows * n_bands;
    if (n <= 0) return WB_OK;
    rotate_bands_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, rows, n_bands, corr, y);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

// logits[r][v] = sum_j x[r][j] * w[v][j], sequential over j (the exact path of
// both decoders: kv_cache.rs:27-31, :370-374).
__global__ void vocab_dot_kernel(const float *__restrict__ x, int rows, int E, const float *__restrict__ w, int vocab,
                                 float *__restrict__ logits) {
    const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (i >= (long long)rows * vocab) return;
    const int r = (int)(i / vocab), v = (int)(i - (long long)r * vocab);
    const float *xr = x + (long long)r * E, *wr = w + (long long)v * E;
    float s = 0.0f;
    for (int j = 0; j < E; j++) s = FA(s, FM(xr[j], wr[j]));
    logits[i] = s;
}

int launch_vocab_dot(const float *x, int rows, int E, const float *w, int vocab, float *logits, cudaStream_t st) {
    const long long n = (long long)rows * vocab;
    if (n <= 0) return WB_OK;
    ProfScope ps("vocab_dot", st);
    vocab_dot_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, rows, E, w, vocab, logits);
    return cudaGetLastError() == cudaSuccess ? WB_OK : WB_ECUDA;
}

#undef FM
#undef FA

}  // namespace wb
