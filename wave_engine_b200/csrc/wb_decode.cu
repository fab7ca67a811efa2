// wb_decode.cu -- KV-cache decode step (src/common/kv_cache.rs:263-335).
//
// Two launches per layer and decode step.
//
// decode_attn_kernel, grid (split, head, sequence), 128 keys per warp; a
// cache of up to 1536 keys takes one CTA of up to 12 warps per (sequence,
// head), a longer one 4-warp CTAs of 512 keys (split partials, ticket merge):
//   * every CTA projects the new position's phase theta_q = atan2f(s, r)
//     (kv_cache.rs:271) from the x row, then scans its split of the cached
//     keys: the bucket byte and phase of every key (coalesced, issued up
//     front), the score cos(n (theta_q - theta_k)) only for keys in buckets
//     b-1..b+1 or at the previous position (kv_cache.rs:285-298), and the
//     fp32 value row only of those keys, streamed with 128-bit loads by
//     groups of lanes, U loads per lane in flight;
//   * decode scores never exceed the self score 1.0 (kv_cache.rs:294), so the
//     softmax uses the fixed shift 1: p = exp(s - 1) exactly as the
//     reference's max-subtraction, and split partials (sum p, sum p v) merge
//     by plain addition, in split order (deterministic);
//   * split 0 also computes the new value v = Wv x_h + b (kv_cache.rs:272-277);
//     the warps of a CTA merge in shared memory, and with several splits the
//     last CTA of a (sequence, head) -- an atomic ticket in scratch -- merges
//     the split partials; it adds the self term (p = 1, v), normalises into
//     the merged head output o, and appends (phase, bucket, value) at
//     position n.
// decode_out_kernel runs out_proj (kv_cache.rs:330-335) on the merged
// outputs o and advances the cached lengths.  It is launched as a
// programmatic dependent of the attention grid: its first weight batch is
// loaded while that grid finishes, and it waits for the grid's completion
// before it reads o or touches a length (a CTA of the attention grid that
// starts late must still see the old length).
// Scratch: partials, new values, merged outputs and a ticket array that the
// kernel returns to zero.
#include "wb_decode.h"
#include "wb_ptx.cuh"

#include <algorithm>
#include <cstdlib>

namespace wb {

static constexpr int DEC_KEYS_PER_WARP = 128;
static constexpr int DEC_MAX_HD = 128;  // head_dim limit (one merge column per thread of a 4-warp CTA)

// Warps per attention CTA, from the cache capacity.  Up to 1536 keys a
// (sequence, head) is one CTA of up to 12 warps (4, 8, 10 or 12: warps past
// the capacity would run the prologue for no keys) whose partials merge in
// shared memory: no split partials in scratch, no ticket, one phase
// projection.  Longer caches use 4-warp CTAs of 512 keys and the ticket
// merge, which keeps many short CTAs in flight for long contexts.
static int decode_warps(int cap) {
    return cap <= 512 ? 4 : cap <= 1024 ? 8 : cap <= 1280 ? 10 : cap <= 1536 ? 12 : 4;
}
static int decode_nsplit(int cap) {
    const int chunk = decode_warps(cap) * DEC_KEYS_PER_WARP;
    return (cap + chunk - 1) / chunk;
}

// cudaLaunchKernelEx, optionally with the programmatic-stream-serialization
// attribute (the grid may begin while the previous grid of the stream runs;
// it calls griddep_wait() before it reads anything that grid writes).
template <typename... KArgs, typename... Args>
static cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             bool dependent, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dependent ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

struct DecodeArgs {
    WbSeqView sv;             // cache view of the layer (slot = seq ids)
    int32_t *len;             // [slots] cached positions (device truth)
    int cap, n_slots;
    const float *x;           // [n_seq][E]
    const float *wrs_h, *brs; // phase projection [H][E][2] (a head's weights contiguous), [H][2]
    const float *wv_t, *bv;   // value projection [H][hd(in)][hd(out)], [H][hd]
    const float *hn;          // [H]
    int n_seq, H, hd, E, nsplit;
    float *part;              // [n_seq][H][nsplit][hd + 1]
    float *vnew;              // [n_seq][H][hd]
    float *o;                 // [n_seq][E] merged, normalised head outputs
    unsigned int *ticket;     // [n_seq][H]
    uint32_t *dev_err;
};

// VEC consecutive floats of a value row, through the read-only path.
template <int VEC>
struct VRow {
    float v[VEC];
    __device__ __forceinline__ void load(const float *src) {
        if constexpr (VEC == 4) {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(src));
            v[0] = t.x;
            v[1] = t.y;
            v[2] = t.z;
            v[3] = t.w;
        } else if constexpr (VEC == 2) {
            const float2 t = __ldg(reinterpret_cast<const float2 *>(src));
            v[0] = t.x;
            v[1] = t.y;
        } else {
            v[0] = __ldg(src);
        }
    }
};

// G lanes per key row: enough VEC-wide lanes to cover hd (rounded up to a
// power of two dividing 32).
template <int VEC>
__device__ __forceinline__ int lanes_per_key(int hd) {
    const int need = (hd + VEC - 1) / VEC;
    int g = 1;
    while (g < need) g <<= 1;
    return g;
}

// p = exp(cos(a) - 1): the argument reduced to [-pi, pi] by Cody-Waite
// reduction with 2*pi split in two floats (hi = 2*pi rounded to float, lo =
// the remainder), then the hardware approximations __cosf and __expf
// (absolute error of a few 1e-7 on these ranges, far inside the 2e-3
// tolerance of the tensor path).
__device__ __forceinline__ float decode_weight(float arg) {
    constexpr float kTwoPiHi = 6.28318548202514648f;    // float nearest 2*pi
    constexpr float kTwoPiLo = -1.74845553146951e-07f;  // 2*pi - kTwoPiHi
    constexpr float kInvTwoPi = 0.159154943091895336f;
    const float k = rintf(arg * kInvTwoPi);
    float r = fmaf(-k, kTwoPiHi, arg);
    r = fmaf(-k, kTwoPiLo, r);
    return __expf(__cosf(r) - 1.0f);
}

// x row -> shared memory and this thread's partial sums of the phase
// projection (r, s) = W_rs x (kv_cache.rs:271): elements tid, tid + THREADS,
// ... summed in that order, XU loads of x and of W_rs in flight per batch.
// wrs_h: head h's (r, s) weight pairs, [E][2] (coalesced float2 loads).
template <int XU, int THREADS>
__device__ __forceinline__ void decode_x_phase(const float *xr, const float *wrs_h, int E, int tid, float *xs,
                                               float &r, float &s, int jbeg = 0) {
    for (int j0 = jbeg; j0 < E; j0 += XU * THREADS) {
        float xv[XU];
        float2 wv2[XU];
#pragma unroll
        for (int u = 0; u < XU; u++) {
            const int j = j0 + u * THREADS + tid;
            xv[u] = j < E ? __ldg(xr + j) : 0.0f;
            wv2[u] = j < E ? __ldg(reinterpret_cast<const float2 *>(wrs_h) + j) : make_float2(0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < XU; u++) {
            const int j = j0 + u * THREADS + tid;
            if (j < E) xs[j] = xv[u];
            r = fmaf(wv2[u].x, xv[u], r);
            s = fmaf(wv2[u].y, xv[u], s);
        }
    }
}

// theta_q = atan2(s, r) of the CTA's partial sums, in two steps: every
// warp's shuffle sums go to red[] (lane 0), and after a barrier one warp
// adds the bias and the warps' sums in warp order and leaves theta_q and
// its bucket in red[2 NW], red[2 NW + 1] for all threads after the next
// barrier -- the other warps meanwhile compute the new value's partials,
// instead of each repeating the sums, atan2f and the bucket.
template <int NW>
__device__ __forceinline__ void decode_theta_partials(float r, float s, float *red, int warp, int lane) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        r += __shfl_xor_sync(0xffffffffu, r, o);
        s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    if (lane == 0) {
        red[warp] = r;
        red[NW + warp] = s;
    }
}
template <int NW>
__device__ __forceinline__ void decode_theta_finish(float *red, float br, float bs, int lane) {
    float rr = br, ss = bs;
#pragma unroll
    for (int w = 0; w < NW; w++) {
        rr += red[w];
        ss += red[NW + w];
    }
    const float th = atan2f(ss, rr);
    if (lane == 0) {
        red[2 * NW] = th;
        red[2 * NW + 1] = __int_as_float(phase_to_bucket(th));
    }
}

// VEC: floats per value load.
static constexpr int DEC_U = 8;  // value loads per lane in flight (DEC_U * 32 / G rows per warp)
// NW: warps per CTA (4, 8, 10 or 12); the register cap keeps 8, 4 or 3 CTAs
// per SM resident so a serve-sized grid is one wave.  HD: head_dim as a
// compile-time constant (0: a.hd at run time) -- every thread derives its
// roles from divisions by head_dim, which are shifts for a constant 64 and
// software divide sequences otherwise.
template <int VEC, int NW, bool PAGED, int HD>
__global__ void __launch_bounds__(NW * 32, NW >= 10 ? 3 : (NW == 8 ? 4 : 8)) decode_attn_kernel(DecodeArgs a) {
    constexpr int DEC_THREADS = NW * 32;
    constexpr int DEC_WARPS = NW;
    constexpr int DEC_CHUNK = NW * DEC_KEYS_PER_WARP;  // keys per CTA
    extern __shared__ float dsm[];
    const int split = blockIdx.x, h = blockIdx.y, i = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = a.E, hd = HD ? HD : a.hd;
    float *xs = dsm;                                   // [E]
    // [DEC_WARPS][DEC_KEYS_PER_WARP] kept keys: (value-row offset as int bits, p)
    float2 *lkp = reinterpret_cast<float2 *>(xs + E);  // 8-byte aligned: E is even
    float *opart = reinterpret_cast<float *>(lkp + DEC_WARPS * DEC_KEYS_PER_WARP);  // [DEC_WARPS][hd]
    float *lpart = opart + DEC_WARPS * hd;             // [DEC_WARPS]
    float *red = lpart + DEC_WARPS;                    // [2 * DEC_WARPS + 2] phase reduction, theta_q, bucket
    float *vpart = red + 2 * DEC_WARPS + 2;            // [DEC_THREADS] new-value partial sums
    __shared__ int s_flag;

    // the out_proj grid may launch and load its weights
    ptx::griddep_launch_dependents();
    // With DecodeLaunch::chain this grid is a programmatic dependent of the
    // kernel before it in the stream -- the out_proj of another layer or
    // cache, which lets it launch once the attention grid before that is
    // complete: the slot, length, cached keys and weights, which that
    // out_proj does not write, are loaded before griddepcontrol.wait; x,
    // and every write, after it (without chain the wait returns at once).
    // ONE: one split per (sequence, head) (decode_warps).  The slot load
    // goes first with the phase weights; the length and key loads follow as
    // soon as the slot arrives, then the remaining weights, then x;
    // theta_q is ready after one barrier, before the length arrives.
    constexpr bool ONE = NW > 4;
    const float *xr = a.x + (long long)i * E;
    const float *wrs = a.wrs_h + (long long)h * E * 2;
    const int slot = a.sv.slot ? a.sv.slot[i] : i;
    // new value v = Wv x_h + b (kv_cache.rs:272-277): thread (vd, vq) sums
    // inputs [vq * kper, (vq + 1) * kper) of output vd, in input order
    const int P = DEC_THREADS / hd;
    const int vd = tid % hd, vq = tid / hd;
    const int kper = (hd + P - 1) / P;
    // value weights held in registers (ONE: ceil(64 / (NW * 32 / 64)) for head_dim 64)
    constexpr int VN = NW == 8 ? 16 : (NW == 10 ? 13 : 12);
    // x elements per thread in the first batch (ONE: the whole 768-wide row)
    constexpr int XU = NW == 8 ? 4 : (NW == 10 ? 3 : 2);
    const bool vearly = ONE && kper <= VN;
    float wl0[ONE ? VN : 1];
    float xv0[ONE ? XU : 1];
    float2 wv0[ONE ? XU : 1];
    float r = 0.0f, s = 0.0f;
    float hn = 0.0f, br = 0.0f, bs = 0.0f;
    float vpar = 0.0f;  // ONE: the bias b of output vd starts the slice-0 sum
    if constexpr (ONE) {
#pragma unroll
        for (int u = 0; u < XU; u++) {
            const int j = u * DEC_THREADS + tid;
            wv0[u] = j < E ? __ldg(reinterpret_cast<const float2 *>(wrs) + j) : make_float2(0.f, 0.f);
        }
    }
    if (slot < 0 || slot >= a.n_slots) {
        if (split == 0 && h == 0 && tid == 0) atomicOr(a.dev_err, WB_DERR_BOUNDS);
        return;
    }
    const int k0 = split * DEC_CHUNK + warp * DEC_KEYS_PER_WARP;
    // this warp's keys k0 .. k0 + 127 sit at index kbase + k: the slot's
    // contiguous row of head h, or (paged cache) one page of the slot's
    // page table -- an unmapped page holds no keys (kmapped false)
    long long kbase;
    bool kmapped = true;
    int kcap;  // positions the slot can hold
    if constexpr (PAGED) {
        kcap = a.sv.max_pages << WB_PAGE_SHIFT;
        const int pg = k0 < kcap ? __ldg(a.sv.pages + (long long)slot * a.sv.max_pages + (k0 >> WB_PAGE_SHIFT)) : -1;
        kmapped = pg >= 0;
        kbase = (long long)max(pg, 0) * a.sv.seq_stride + (long long)h * WB_PAGE - k0;
    } else {
        kcap = a.sv.cap;
        kbase = (long long)slot * a.sv.seq_stride + (long long)h * a.sv.cap;
    }
    const float *theta = a.sv.theta + kbase;
    const uint8_t *bucket = a.sv.bucket + kbase;
    const float *V = a.sv.v + kbase * hd;
    constexpr int KR = DEC_KEYS_PER_WARP / 32;
    uint8_t kb[KR];
    float kth[KR];
    const int n = a.len[slot];
    float thq;
    int qb;
    if constexpr (ONE) {
        // the whole cache row is this CTA's: the key loads (bucket byte +
        // phase) need only the slot, bounded by the allocated row, so they
        // go out together with the length load; keys at or past n are
        // dropped by the k < n test of the score loop
#pragma unroll
        for (int c = 0; c < KR; c++) {
            const int k = k0 + c * 32 + lane;
            kb[c] = kmapped && k < kcap ? __ldg(bucket + k) : (uint8_t)0xFF;
            kth[c] = kmapped && k < kcap ? __ldg(theta + k) : 0.0f;
        }
        // the weights needed after theta_q, behind the slot-dependent loads
        // in the memory pipeline
        hn = __ldg(a.hn + h);
        br = __ldg(a.brs + h * 2);
        bs = __ldg(a.brs + h * 2 + 1);
        if (vq == 0) vpar = __ldg(a.bv + h * hd + vd);
        if (vearly && vq < P) {
            const float *wv = a.wv_t + (long long)h * hd * hd + vd;
            const int j0 = vq * kper;
#pragma unroll
            for (int u = 0; u < VN; u++)
                wl0[u] = u < kper && j0 + u < hd ? __ldg(wv + (long long)(j0 + u) * hd) : 0.0f;
        }
        // x (and every write of this kernel) waits for the grid before
        ptx::griddep_wait();
#pragma unroll
        for (int u = 0; u < XU; u++) {
            const int j = u * DEC_THREADS + tid;
            xv0[u] = j < E ? __ldg(xr + j) : 0.0f;
        }
        // x row: the first batch, then any further batches
#pragma unroll
        for (int u = 0; u < XU; u++) {
            const int j = u * DEC_THREADS + tid;
            if (j < E) xs[j] = xv0[u];
            r = fmaf(wv0[u].x, xv0[u], r);
            s = fmaf(wv0[u].y, xv0[u], s);
        }
        decode_x_phase<XU, DEC_THREADS>(xr, wrs, E, tid, xs, r, s, XU * DEC_THREADS);
        decode_theta_partials<NW>(r, s, red, warp, lane);
        __syncthreads();  // xs and the warp partials visible
        if (warp == 0) decode_theta_finish<NW>(red, br, bs, lane);
        // the new value's partial sums (summed at the merge)
        if (vq < P) {
            const float *xh = xs + h * hd;
            const int j0 = vq * kper;
            if (vearly) {
#pragma unroll
                for (int u = 0; u < VN; u++)
                    if (u < kper && j0 + u < hd) vpar = fmaf(wl0[u], xh[j0 + u], vpar);
            } else {
                const float *wv = a.wv_t + (long long)h * hd * hd + vd;
                const int j1 = min(hd, j0 + kper);
                for (int jb = j0; jb < j1; jb += 16) {
                    float wl[16];
#pragma unroll
                    for (int u = 0; u < 16; u++)
                        wl[u] = jb + u < j1 ? __ldg(wv + (long long)(jb + u) * hd) : 0.0f;
#pragma unroll
                    for (int u = 0; u < 16; u++)
                        if (jb + u < j1) vpar = fmaf(wl[u], xh[jb + u], vpar);
                }
            }
        }
        vpart[tid] = vpar;
        __syncthreads();  // theta_q and its bucket
        thq = red[2 * NW];
        qb = __float_as_int(red[2 * NW + 1]);
    }
    if (n < 0 || n >= a.cap) {
        if (split == 0 && h == 0 && tid == 0) atomicOr(a.dev_err, WB_DERR_BOUNDS);
        return;
    }
    const int n_act = n > 0 ? (n + DEC_CHUNK - 1) / DEC_CHUNK : 1;
    if (split >= n_act) return;
    float *vnew = a.vnew + ((long long)i * a.H + h) * hd;
    if constexpr (!ONE) {
        // this warp's key loads, up to the length (most splits of a long
        // cache hold no keys of a short sequence), then the x row
#pragma unroll
        for (int c = 0; c < KR; c++) {
            const int k = k0 + c * 32 + lane;
            kb[c] = kmapped && k < n ? __ldg(bucket + k) : (uint8_t)0xFF;
            kth[c] = kmapped && k < n ? __ldg(theta + k) : 0.0f;
        }
        ptx::griddep_wait();  // x (and every write) waits for the grid before
        decode_x_phase<8, DEC_THREADS>(xr, wrs, E, tid, xs, r, s);
        decode_theta_partials<NW>(r, s, red, warp, lane);
        __syncthreads();  // xs and the warp partials visible
        if (warp == 0) decode_theta_finish<NW>(red, __ldg(a.brs + h * 2), __ldg(a.brs + h * 2 + 1), lane);
        // split 0: the new value, weight loads in batches of 16 before use
        if (split == 0 && vq < P) {
            const float *xh = xs + h * hd;
            const float *wv = a.wv_t + (long long)h * hd * hd + vd;
            const int j0 = vq * kper, j1 = min(hd, j0 + kper);
            for (int jb = j0; jb < j1; jb += 16) {
                float wl[16];
#pragma unroll
                for (int u = 0; u < 16; u++) wl[u] = jb + u < j1 ? __ldg(wv + (long long)(jb + u) * hd) : 0.0f;
#pragma unroll
                for (int u = 0; u < 16; u++)
                    if (jb + u < j1) vpar = fmaf(wl[u], xh[jb + u], vpar);
            }
        }
        vpart[tid] = vpar;
        hn = __ldg(a.hn + h);
        __syncthreads();  // theta_q, its bucket and the new value's partials
        thq = red[2 * NW];
        qb = __float_as_int(red[2 * NW + 1]);
        if (split == 0 && tid < hd) {  // hd <= DEC_MAX_HD <= DEC_THREADS (checked at launch)
            float v = __ldg(a.bv + h * hd + tid);
            for (int q = 0; q < P; q++) v += vpart[q * hd + tid];
            vnew[tid] = v;
        }
    }
    const uint32_t amask = allowed_bucket_mask(qb);

    // mask, score, p = exp(s - 1); compact (index, p) per warp
    int m = 0;
    float lsum = 0.0f;
    float2 *my_kp = lkp + warp * DEC_KEYS_PER_WARP;
#pragma unroll
    for (int c = 0; c < KR; c++) {
        const int k = k0 + c * 32 + lane;
        bool ok = false;
        float p = 0.0f;
        if (k < n && kmapped) {
            ok = ((amask >> kb[c]) & 1u) || k == n - 1;
            if (ok) {
                p = decode_weight(__fmul_rn(hn, __fsub_rn(thq, kth[c])));
                ok = p > 0.0f;  // kv_cache.rs:315 skips zero weights
            }
        }
        const unsigned bal = __ballot_sync(0xffffffffu, ok);
        if (ok) {
            const int pos = m + __popc(bal & ((1u << lane) - 1u));
            my_kp[pos] = make_float2(__int_as_float(k * hd), p);
        }
        m += __popc(bal);
        lsum += p;
    }
    __syncwarp();

    // stream value rows of the kept keys: G lanes per row, VEC floats per lane
    const int G = lanes_per_key<VEC>(hd);
    const int KPW = 32 / G;
    const int BATCH = KPW * DEC_U;  // rows per batch of loads (a power of two)
    const int slotk = lane / G, vi = lane - slotk * G;
    const bool vact = vi * VEC < hd;
    float acc[VEC];
#pragma unroll
    for (int u = 0; u < VEC; u++) acc[u] = 0.0f;
    // PAD (the 64-register CTAs of 4, 8 and 10 warps): the list padded to
    // whole batches with weight-0 copies of the last kept row, so the loads of
    // a batch need no bound; the 56-register 12-warp CTAs clamp the index
    // instead (the padded loop spills there).  Either way a batch's loads are all in
    // flight before the first is used, and rows past the list re-read the
    // last kept row with weight 0.
    constexpr bool PAD = NW != 12;
    if (PAD && m > 0) {
        const float2 last = make_float2(my_kp[m - 1].x, 0.0f);
        for (int t = m + lane; t < ((m + BATCH - 1) & ~(BATCH - 1)); t += 32) my_kp[t] = last;
        __syncwarp();
    }
    if (vact) {
        const float *Vl = V + vi * VEC;
        const float2 *lq = my_kp + slotk;
        for (int b0 = 0; b0 < m; b0 += BATCH) {
            VRow<VEC> rows[DEC_U];
            float pr[DEC_U];
#pragma unroll
            for (int u = 0; u < DEC_U; u++) {
                if constexpr (PAD) {
                    const float2 e = lq[b0 + u * KPW];
                    rows[u].load(Vl + __float_as_int(e.x));
                    pr[u] = e.y;
                } else {
                    const int j = b0 + u * KPW + slotk;
                    const float2 e = my_kp[min(j, m - 1)];
                    rows[u].load(Vl + __float_as_int(e.x));
                    pr[u] = j < m ? e.y : 0.0f;
                }
            }
#pragma unroll
            for (int u = 0; u < DEC_U; u++)
#pragma unroll
                for (int e = 0; e < VEC; e++) acc[e] = fmaf(pr[u], rows[u].v[e], acc[e]);
        }
    }
    for (int o = G; o < 32; o <<= 1)
#pragma unroll
        for (int u = 0; u < VEC; u++) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], o);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (lane < G && vact)
#pragma unroll
        for (int u = 0; u < VEC; u++)
            if (vi * VEC + u < hd) opart[warp * hd + vi * VEC + u] = acc[u];
    if (lane == 0) lpart[warp] = lsum;
    __syncthreads();

    float od = 0.0f, lall = 0.0f;
    if (n_act > 1) {
        // several splits: partial -> scratch, the last split merges
        float *pdst = a.part + (((long long)i * a.H + h) * a.nsplit + split) * (hd + 1);
        for (int d = tid; d < hd; d += DEC_THREADS) {
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < DEC_WARPS; w++) v += opart[w * hd + d];
            pdst[d] = v;
        }
        if (tid == 0) {
            float l = 0.0f;
#pragma unroll
            for (int w = 0; w < DEC_WARPS; w++) l += lpart[w];
            pdst[hd] = l;
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const unsigned t = atomicAdd(a.ticket + (long long)i * a.H + h, 1u);
            s_flag = (t == (unsigned)(n_act - 1));
        }
        __syncthreads();
        if (!s_flag) return;
        __threadfence();
        // merge the split partials in split order (hd <= DEC_THREADS: one
        // column per thread); the loads of 8 splits go out together
        if (tid < hd) {
            const float *pp = a.part + ((long long)i * a.H + h) * a.nsplit * (hd + 1);
            for (int sp0 = 0; sp0 < n_act; sp0 += 8) {
                float ov[8], lv[8];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int sp = sp0 + u;
                    ov[u] = sp < n_act ? __ldcg(pp + (long long)sp * (hd + 1) + tid) : 0.0f;
                    lv[u] = sp < n_act ? __ldcg(pp + (long long)sp * (hd + 1) + hd) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    od += ov[u];
                    lall += lv[u];
                }
            }
        }
    } else if (tid < hd) {
#pragma unroll
        for (int w = 0; w < DEC_WARPS; w++) {
            od += opart[w * hd + tid];
            lall += lpart[w];
        }
    }
    // ---- merge (i, h): self term p = exp(1 - 1) = 1 (kv_cache.rs:294, :318),
    // normalise, append (kv_cache.rs:323-326) at position n (a paged slot
    // without a page reserved for n is flagged and not appended)
    long long inew;
    if constexpr (PAGED) {
        const long long r = wb_row_slot(a.sv, slot, n);
        inew = r < 0 ? -1 : r + (long long)h * WB_PAGE;
        if (inew < 0 && tid == 0) atomicOr(a.dev_err, WB_DERR_BOUNDS);
    } else {
        inew = kbase + n;  // 0 <= n < cap (checked above)
    }
    if (tid < hd) {
        float vn;
        if constexpr (ONE) {
            vn = vpart[tid];  // slice 0 (with the bias), then the other slices
            for (int q = 1; q < P; q++) vn += vpart[q * hd + tid];
        } else {
            vn = __ldcg(vnew + tid);
        }
        a.o[(long long)i * E + (long long)h * hd + tid] = (od + vn) / (lall + 1.0f);
        if (!PAGED || inew >= 0) a.sv.v[inew * hd + tid] = vn;
    }
    if (tid == 0) {
        if (!PAGED || inew >= 0) {
            a.sv.theta[inew] = thq;
            a.sv.bucket[inew] = (uint8_t)qb;
        }
        if (n_act > 1) a.ticket[(long long)i * a.H + h] = 0u;
    }
}

// out_proj of the step's rows (kv_cache.rs:330-335), y = o W_o^T + b, and
// the length update.  Block = 8 rows x 32 columns; its 256 threads are 8
// column quads x 32 K slices: thread (slice, quad) accumulates 8 rows x 4
// columns over its slice, then the 32 slice partials of every output are
// summed in slice order.  The block's whole W_o column tile (K chunk of up
// to OUT_KC inputs x 32 columns) is copied into shared memory with cp.async
// before the dependency wait -- the attention grid does not write W_o, and
// the copy holds no registers -- so after the wait only the o rows (one
// batch of loads from L2) stand between the attention grid and the
// arithmetic.  Block (0, 0) advances the lengths: it reads them (and the
// bias) before the wait -- the attention grid only reads them -- and writes
// them after it, when every attention CTA of the step has read them.
static constexpr int OUT_THREADS = 256;
static constexpr int OUT_R = 8;                    // rows per block
static constexpr int OUT_C = 32;                   // columns per block
static constexpr int OUT_Q = OUT_C / 4;            // column quads
static constexpr int OUT_S = OUT_THREADS / OUT_Q;  // K slices (32)
static constexpr int OUT_KC = 1024;                // inputs per staged chunk (W tile 128 KB, o rows 32 KB)

struct DecodeOutArgs {
    const float *o;     // [n][E]
    const float *wo_t;  // [E(in)][E(out)]
    const float *bo;    // [E]
    float *y;           // [n][E]
    int n, E, cap;
    int32_t *len;
    const int32_t *slot;
    int n_slots;
    const int32_t *pages;  // paged cache: lengths advance only into mapped pages
    int max_pages;
};

// W_o[k0 .. k0+kn)[c0 .. c0+32) -> ws[kn][32]: cp.async where the 16 bytes
// are in range and aligned, plain loads (zero outside the matrix) elsewhere.
__device__ __forceinline__ void out_stage_w(const DecodeOutArgs &a, float *ws, int k0, int kn, int c0) {
    const int E = a.E;
    const bool vec = (E % 4) == 0 && c0 + OUT_C <= E;
    for (int e = threadIdx.x; e < kn * OUT_Q; e += OUT_THREADS) {
        const int kk = e / OUT_Q, cq = e % OUT_Q;
        const int c = c0 + cq * 4;
        float *dst = ws + kk * OUT_C + cq * 4;
        const float *src = a.wo_t + (long long)(k0 + kk) * E + c;
        if (vec) {
            ptx::cp_async<16>(dst, src);
        } else {
#pragma unroll
            for (int u = 0; u < 4; u++) dst[u] = c + u < E ? __ldg(src + u) : 0.0f;
        }
    }
    ptx::cp_async_commit();
}

__global__ void __launch_bounds__(OUT_THREADS) decode_out_kernel(DecodeOutArgs a) {
    extern __shared__ __align__(16) float osm[];
    const int E = a.E, n = a.n;
    const int c0 = blockIdx.x * OUT_C, r0 = blockIdx.y * OUT_R;
    const int tid = threadIdx.x, ks = tid / OUT_Q, cq = tid % OUT_Q;
    const int kc = min(E, OUT_KC);
    const int ost = ((kc + 3) & ~3) + 4;  // o row stride (floats; 16-byte rows, shifted banks)
    float *ws = osm;                       // [kc][OUT_C]
    float *os = ws + kc * OUT_C;           // [OUT_R][ost]
    float *red = os + OUT_R * ost;         // [OUT_S][OUT_R][OUT_C]
    float acc[OUT_R][4];
#pragma unroll
    for (int r = 0; r < OUT_R; r++)
#pragma unroll
        for (int u = 0; u < 4; u++) acc[r][u] = 0.0f;
    // W_o chunk 0, this thread's bias and (block (0, 0)) the lengths to
    // advance, under the attention grid's tail: that grid reads the lengths
    // and writes none of these
    out_stage_w(a, ws, 0, kc, c0);
    const int ro = tid / OUT_C, co = tid % OUT_C;  // this thread's output in the epilogue
    const float bias = c0 + co < E ? __ldg(a.bo + c0 + co) : 0.0f;
    const bool len_block = blockIdx.x == 0 && blockIdx.y == 0;
    int lslot = -1, lnew = 0;
    if (len_block && n <= OUT_THREADS && tid < n) {
        const int sl = a.slot ? a.slot[tid] : tid;
        if (sl >= 0 && sl < a.n_slots) {
            const int cur = a.len[sl];
            if (cur < a.cap && wb_pos_mapped(a.pages, a.max_pages, sl, cur)) {
                lslot = sl;
                lnew = cur + 1;
            }
        }
    }
    ptx::griddep_wait();
    // the attention grid is complete, and with it (by the same wait in every
    // grid of the chain) all earlier work of the stream: the next layer's
    // attention grid may launch and load its slot, length and keys
    ptx::griddep_launch_dependents();
    for (int kc0 = 0; kc0 < E; kc0 += kc) {
        const int kn = min(kc, E - kc0);
        if (kc0 > 0) {
            __syncthreads();  // previous chunk consumed
            out_stage_w(a, ws, kc0, kn, c0);
        }
        // o rows r0..r0+7, inputs kc0..kc0+kn: each thread one float4 of
        // every row, all loads in flight together (L2: written by the
        // attention grid), then the shared-memory stores
        {
            const int q4 = (kn + 3) / 4;  // float4 per row
            for (int qb = 0; qb < q4; qb += OUT_THREADS) {
                const int kq = qb + tid, k = kq * 4;
                if (kq < q4) {
                    float4 v[OUT_R];
#pragma unroll
                    for (int r = 0; r < OUT_R; r++) {
                        v[r] = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (r0 + r < n) {
                            const float *src = a.o + (long long)(r0 + r) * E + kc0 + k;
                            if ((E % 4) == 0 && k + 3 < kn) v[r] = __ldcg(reinterpret_cast<const float4 *>(src));
                            else {
                                if (k < kn) v[r].x = __ldcg(src);
                                if (k + 1 < kn) v[r].y = __ldcg(src + 1);
                                if (k + 2 < kn) v[r].z = __ldcg(src + 2);
                                if (k + 3 < kn) v[r].w = __ldcg(src + 3);
                            }
                        }
                    }
#pragma unroll
                    for (int r = 0; r < OUT_R; r++) *reinterpret_cast<float4 *>(os + r * ost + k) = v[r];
                }
            }
        }
        ptx::cp_async_wait<0>();
        __syncthreads();
        // this thread's K slice in steps of 4 inputs: 4 weight rows, 8 o quads
        const int kslice = ((kn + OUT_S - 1) / OUT_S + 3) & ~3;
        const int k0 = min(kn, ks * kslice), k1 = min(kn, k0 + kslice);
        for (int k = k0; k < k1; k += 4) {
            float4 w[4];
#pragma unroll
            for (int u = 0; u < 4; u++)
                w[u] = k + u < k1 ? *reinterpret_cast<const float4 *>(ws + (k + u) * OUT_C + cq * 4)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int r = 0; r < OUT_R; r++) {
                const float4 o4 = *reinterpret_cast<const float4 *>(os + r * ost + k);
                const float ov[4] = {o4.x, o4.y, o4.z, o4.w};
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    acc[r][0] = fmaf(w[u].x, ov[u], acc[r][0]);
                    acc[r][1] = fmaf(w[u].y, ov[u], acc[r][1]);
                    acc[r][2] = fmaf(w[u].z, ov[u], acc[r][2]);
                    acc[r][3] = fmaf(w[u].w, ov[u], acc[r][3]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < OUT_R; r++)
        *reinterpret_cast<float4 *>(red + (ks * OUT_R + r) * OUT_C + cq * 4) =
            make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    __syncthreads();
    {
        float v = 0.0f;  // one output per thread
#pragma unroll 8
        for (int q = 0; q < OUT_S; q++) v += red[(q * OUT_R + ro) * OUT_C + co];
        if (r0 + ro < n && c0 + co < E) a.y[(long long)(r0 + ro) * E + c0 + co] = v + bias;
    }
    if (len_block) {
        if (n <= OUT_THREADS) {
            if (lslot >= 0) a.len[lslot] = lnew;
        } else {
            for (int i = tid; i < n; i += OUT_THREADS) {
                const int slot = a.slot ? a.slot[i] : i;
                if (slot >= 0 && slot < a.n_slots && a.len[slot] < a.cap &&
                    wb_pos_mapped(a.pages, a.max_pages, slot, a.len[slot]))
                    a.len[slot] += 1;
            }
        }
    }
}

int launch_decode_out(const float *o, const float *wo_t, const float *bo, float *y, int n, int E, int cap,
                      int32_t *len, const int32_t *slot, int n_slots, cudaStream_t st, std::string *msg,
                      const int32_t *pages, int max_pages) {
    ProfScope ps("decode_out", st);
    DecodeOutArgs a{o, wo_t, bo, y, n, E, cap, len, slot, n_slots, pages, max_pages};
    const int kc = std::min(E, OUT_KC);
    const int ost = ((kc + 3) & ~3) + 4;
    const size_t smem = sizeof(float) * ((size_t)kc * OUT_C + (size_t)OUT_R * ost + (size_t)OUT_S * OUT_R * OUT_C);
    cudaFuncSetAttribute(decode_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((E + OUT_C - 1) / OUT_C, (n + OUT_R - 1) / OUT_R);
    cudaError_t e = launch_ex(decode_out_kernel, grid, dim3(OUT_THREADS), smem, st, true, a);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("decode out launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

struct DecodeScratch {
    size_t part, vnew, o, ticket, end;
};
static DecodeScratch decode_scratch_layout(int n_seq, int H, int hd, int E, int cap) {
    const int nsplit = decode_nsplit(cap);
    Carve c;
    DecodeScratch d;
    d.part = c.take<float>((size_t)n_seq * H * nsplit * (hd + 1));
    d.vnew = c.take<float>((size_t)n_seq * H * hd);
    d.o = c.take<float>((size_t)n_seq * E);
    d.ticket = c.take<unsigned int>((size_t)n_seq * H);
    d.end = c.off;
    return d;
}

size_t decode_scratch_bytes(int n_seq, int H, int hd, int E, int cap) {
    return decode_scratch_layout(n_seq, H, hd, E, cap).end;
}

void decode_scratch_tickets(int n_seq, int H, int hd, int E, int cap, size_t *offset, size_t *bytes) {
    const DecodeScratch d = decode_scratch_layout(n_seq, H, hd, E, cap);
    *offset = d.ticket;
    *bytes = d.end - d.ticket;
}

template <int VEC, int NW, bool PAGED, int HD>
static cudaError_t launch_attn_hd(const DecodeArgs &a, dim3 grid, cudaStream_t st, bool chain) {
    const size_t smem = sizeof(float) * ((size_t)a.E + 2 * NW * DEC_KEYS_PER_WARP + NW * a.hd + NW + 2 * NW + 2 +
                                         NW * 32);
    cudaFuncSetAttribute(decode_attn_kernel<VEC, NW, PAGED, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    cudaError_t e = launch_ex(decode_attn_kernel<VEC, NW, PAGED, HD>, grid, dim3(NW * 32), smem, st, chain, a);
    return e == cudaSuccess ? cudaGetLastError() : e;
}
template <int VEC, int NW, bool PAGED>
static cudaError_t launch_attn(const DecodeArgs &a, dim3 grid, cudaStream_t st, bool chain) {
    if constexpr (VEC == 4)
        if (a.hd == 64) return launch_attn_hd<4, NW, PAGED, 64>(a, grid, st, chain);
    return launch_attn_hd<VEC, NW, PAGED, 0>(a, grid, st, chain);
}

// the paged variant is a separate instantiation: its page lookups stay out
// of the contiguous cache's kernel
template <int VEC>
static cudaError_t launch_attn_nw(const DecodeArgs &a, int nw, dim3 grid, cudaStream_t st, bool chain) {
    if (a.sv.pages) {
        if (nw == 12) return launch_attn<VEC, 12, true>(a, grid, st, chain);
        if (nw == 10) return launch_attn<VEC, 10, true>(a, grid, st, chain);
        if (nw == 8) return launch_attn<VEC, 8, true>(a, grid, st, chain);
        return launch_attn<VEC, 4, true>(a, grid, st, chain);
    }
    if (nw == 12) return launch_attn<VEC, 12, false>(a, grid, st, chain);
    if (nw == 10) return launch_attn<VEC, 10, false>(a, grid, st, chain);
    if (nw == 8) return launch_attn<VEC, 8, false>(a, grid, st, chain);
    return launch_attn<VEC, 4, false>(a, grid, st, chain);
}

int launch_decode_attn(const DecodeLaunch &L, void *scratch, size_t scratch_bytes, float **o_out,
                       cudaStream_t st, std::string *msg) {
    const int nsplit = decode_nsplit(L.cap);
    const int nw = decode_warps(L.cap);
    if (nw > 4 && nsplit != 1) {
        *msg = "decode: internal split plan error";
        return WB_EINVAL;
    }
    // laid out for the cache's slot count (not this call's n_seq) so the
    // zeroed tickets stay at fixed offsets whatever the batch of the call
    if (L.n_seq > L.n_slots) {
        *msg = "more sequences than cache slots";
        return WB_EINVAL;
    }
    const DecodeScratch lay = decode_scratch_layout(L.n_slots, L.H, L.hd, L.E, L.cap);
    if (scratch_bytes < lay.end) {
        *msg = "decode scratch too small";
        return WB_EINVAL;
    }
    if (L.hd > DEC_MAX_HD) {
        *msg = "decode supports head_dim <= 128";
        return WB_ENOTSUP;
    }
    {
        // a value row is read by at most one warp's lanes, VEC floats each
        const int vec = L.hd % 4 == 0 ? 4 : (L.hd % 2 == 0 ? 2 : 1);
        if ((L.hd + vec - 1) / vec > 32) {
            *msg = "decode supports head_dim that is a multiple of 4, even and <= 64, or <= 32";
            return WB_ENOTSUP;
        }
    }
    char *s = (char *)scratch;
    DecodeArgs a;
    a.sv = L.sv;
    a.len = L.len;
    a.cap = L.cap;
    a.n_slots = L.n_slots;
    a.x = L.x;
    a.wrs_h = L.wrs_h;
    a.brs = L.brs;
    a.wv_t = L.wv_t;
    a.bv = L.bv;
    a.hn = L.hn;
    a.n_seq = L.n_seq;
    a.H = L.H;
    a.hd = L.hd;
    a.E = L.E;
    a.nsplit = nsplit;
    a.part = (float *)(s + lay.part);
    a.vnew = (float *)(s + lay.vnew);
    a.o = (float *)(s + lay.o);
    *o_out = a.o;
    a.ticket = (unsigned int *)(s + lay.ticket);
    a.dev_err = L.dev_err;
    dim3 grid(nsplit, L.H, L.n_seq);
    cudaError_t e;
    {
        ProfScope ps("decode_attn", st);
        if (L.hd % 4 == 0) e = launch_attn_nw<4>(a, nw, grid, st, L.chain);
        else if (L.hd % 2 == 0) e = launch_attn_nw<2>(a, nw, grid, st, L.chain);
        else e = launch_attn_nw<1>(a, nw, grid, st, L.chain);
    }
    if (e != cudaSuccess) {
        *msg = std::string("decode launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

}  // namespace wb
