// wb_decode.cu -- fused KV-cache decode step (src/common/kv_cache.rs:263-335).
//
// One launch per layer and decode step.  Grid (split, head, sequence):
//   * every CTA projects the new position's phase theta_q = atan2(s, r)
//     (kv_cache.rs:271) from the x row, then scans its split of the cached
//     keys: the bucket byte and phase of every key (coalesced), the score
//     cos(n (theta_q - theta_k)) only for keys in buckets b-1..b+1 or at the
//     previous position (kv_cache.rs:285-298), and the fp32 value row only of
//     those keys, streamed with 128-bit loads by groups of lanes.
//   * decode scores never exceed the self score 1.0 (kv_cache.rs:294), so the
//     softmax uses the fixed shift 1: p = exp(s - 1) exactly as the
//     reference's max-subtraction, and split partials (sum p, sum p v) merge
//     by plain addition, in split order (deterministic).
//   * the last CTA of a (sequence, head) -- an atomic ticket in scratch --
//     merges the partials, adds the self term (p = 1, the new value
//     v = Wv x_h + b), normalises, appends (phase, bucket, value) at
//     position n, and multiplies its 64-wide slice into out_proj; the last
//     head of a sequence sums the slices (head order) plus the bias into y.
//     The cached length is advanced by a separate launch afterwards: a CTA
//     of this launch that starts late must still see the old length.
// Scratch: per (sequence, head, split) partials, per (sequence, head) slices
// of y, and two ticket arrays that the kernel returns to zero.
#include "wb_decode.h"
#include "wb_ptx.cuh"

namespace wb {

static constexpr int DEC_THREADS = 256;
static constexpr int DEC_WARPS = DEC_THREADS / 32;
static constexpr int DEC_KEYS_PER_WARP = 256;
static constexpr int DEC_CHUNK = DEC_WARPS * DEC_KEYS_PER_WARP;  // keys per CTA (2048)

struct DecodeArgs {
    WbSeqView sv;             // cache view of the layer (slot = seq ids)
    int32_t *len;             // [slots] cached positions (device truth)
    int cap, n_slots;
    const float *x;           // [n_seq][E]
    const float *wrs_t, *brs; // phase projection [E][H][2], [H][2]
    const float *wv_t, *bv;   // value projection [H][hd(in)][hd(out)], [H][hd]
    const float *wo_t, *bo;   // out_proj [E(in)][E(out)], [E]
    const float *hn;          // [H]
    int n_seq, H, hd, E, nsplit;
    float *part;              // [n_seq][H][nsplit][hd + 1]
    float *yh;                // [n_seq][H][E]
    unsigned int *ticket;     // [n_seq][H]
    unsigned int *hticket;    // [n_seq]
    float *y;                 // [n_seq][E]
    uint32_t *dev_err;
};

template <int VEC>
struct VecT;
template <>
struct VecT<4> {
    using T = float4;
    __device__ static void fma(float *acc, float p, const float *src) {
        const float4 v = __ldg(reinterpret_cast<const float4 *>(src));
        acc[0] = fmaf(p, v.x, acc[0]);
        acc[1] = fmaf(p, v.y, acc[1]);
        acc[2] = fmaf(p, v.z, acc[2]);
        acc[3] = fmaf(p, v.w, acc[3]);
    }
};
template <>
struct VecT<2> {
    __device__ static void fma(float *acc, float p, const float *src) {
        const float2 v = __ldg(reinterpret_cast<const float2 *>(src));
        acc[0] = fmaf(p, v.x, acc[0]);
        acc[1] = fmaf(p, v.y, acc[1]);
    }
};
template <>
struct VecT<1> {
    __device__ static void fma(float *acc, float p, const float *src) { acc[0] = fmaf(p, __ldg(src), acc[0]); }
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

template <int VEC>
__global__ void __launch_bounds__(DEC_THREADS) decode_fused_kernel(DecodeArgs a) {
    extern __shared__ float dsm[];
    const int split = blockIdx.x, h = blockIdx.y, i = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = a.E, hd = a.hd;
    float *xs = dsm;                                   // [E]
    int *lidx = reinterpret_cast<int *>(xs + E);       // [DEC_WARPS][DEC_KEYS_PER_WARP]
    float *lp = reinterpret_cast<float *>(lidx + DEC_WARPS * DEC_KEYS_PER_WARP);
    float *opart = lp + DEC_WARPS * DEC_KEYS_PER_WARP; // [DEC_WARPS][hd]
    float *lpart = opart + DEC_WARPS * hd;             // [DEC_WARPS]
    float *red = lpart + DEC_WARPS;                    // [2 * DEC_WARPS] phase reduction
    float *vpart = red + 2 * DEC_WARPS;                // [DEC_THREADS] new-value partial sums
    __shared__ int s_flag;

    const int slot = a.sv.slot ? a.sv.slot[i] : i;
    if (slot < 0 || slot >= a.n_slots) {
        if (split == 0 && h == 0 && tid == 0) atomicOr(a.dev_err, WB_DERR_BOUNDS);
        return;
    }
    const int n = a.len[slot];
    if (n < 0 || n >= a.cap) {
        if (split == 0 && h == 0 && tid == 0) atomicOr(a.dev_err, WB_DERR_BOUNDS);
        return;
    }
    const int n_act = n > 0 ? (n + DEC_CHUNK - 1) / DEC_CHUNK : 1;
    if (split >= n_act) return;

    const long long base = wb_slot_base(a.sv, i, h);
    const float *theta = a.sv.theta + base;
    const uint8_t *bucket = a.sv.bucket + base;
    const float *V = a.sv.v + base * hd;
    const int k0 = split * DEC_CHUNK + warp * DEC_KEYS_PER_WARP;
    // issue this warp's key loads first (bucket byte + phase of every key;
    // kv_cache.rs:285-292 reads both for the keys it scores)
    constexpr int KR = DEC_KEYS_PER_WARP / 32;
    uint8_t kb[KR];
    float kth[KR];
#pragma unroll
    for (int c = 0; c < KR; c++) {
        const int k = k0 + c * 32 + lane;
        kb[c] = k < n ? __ldg(bucket + k) : (uint8_t)0xFF;
        kth[c] = k < n ? __ldg(theta + k) : 0.0f;
    }

    // x row; theta_q (kv_cache.rs:271, tree-summed) and, in the merging CTA,
    // the new value v = Wv x_h + b (kv_cache.rs:272-277)
    const float *xr = a.x + (long long)i * E;
    for (int j = tid; j < E; j += DEC_THREADS) xs[j] = __ldg(xr + j);
    __syncthreads();
    float r = 0.0f, s = 0.0f;
    for (int j = tid; j < E; j += DEC_THREADS) {
        const float2 w = __ldg(reinterpret_cast<const float2 *>(a.wrs_t + ((long long)j * a.H + h) * 2));
        r = fmaf(w.x, xs[j], r);
        s = fmaf(w.y, xs[j], s);
    }
    // new value: P parts of hd/P inputs per output, P = threads / hd
    const int P = DEC_THREADS / hd;
    const int vd = tid % hd, vq = tid / hd;
    const int kper = (hd + P - 1) / P;
    float vpar = 0.0f;
    if (vq < P) {  // every CTA: the merging split is only known at the end
        const float *xh = xs + h * hd;
        const float *wv = a.wv_t + (long long)h * hd * hd + vd;
        const int j0 = vq * kper, j1 = min(hd, j0 + kper);
#pragma unroll 8
        for (int j = j0; j < j1; j++) vpar = fmaf(__ldg(wv + (long long)j * hd), xh[j], vpar);
    }
    vpart[tid] = vpar;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        r += __shfl_xor_sync(0xffffffffu, r, o);
        s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    if (lane == 0) {
        red[warp] = r;
        red[DEC_WARPS + warp] = s;
    }
    __syncthreads();
    float rr = a.brs[h * 2], ss = a.brs[h * 2 + 1];
#pragma unroll
    for (int w = 0; w < DEC_WARPS; w++) {
        rr += red[w];
        ss += red[DEC_WARPS + w];
    }
    const float thq = atan2f(ss, rr);
    const int qb = phase_to_bucket(thq);
    const uint32_t amask = allowed_bucket_mask(qb);
    const float hn = a.hn[h];

    // mask, score, p = exp(s - 1); compact (index, p) per warp
    int m = 0;
    float lsum = 0.0f;
    int *my_idx = lidx + warp * DEC_KEYS_PER_WARP;
    float *my_p = lp + warp * DEC_KEYS_PER_WARP;
#pragma unroll
    for (int c = 0; c < KR; c++) {
        const int k = k0 + c * 32 + lane;
        bool ok = false;
        float p = 0.0f;
        if (k < n) {
            ok = ((amask >> kb[c]) & 1u) || k == n - 1;
            if (ok) {
                p = expf(cosf(__fmul_rn(hn, __fsub_rn(thq, kth[c]))) - 1.0f);
                ok = p > 0.0f;  // kv_cache.rs:315 skips zero weights
            }
        }
        const unsigned bal = __ballot_sync(0xffffffffu, ok);
        if (ok) {
            const int pos = m + __popc(bal & ((1u << lane) - 1u));
            my_idx[pos] = k;
            my_p[pos] = p;
        }
        m += __popc(bal);
        lsum += p;
    }
    __syncwarp();

    // stream value rows of the kept keys: G lanes per row, VEC floats per lane
    const int G = lanes_per_key<VEC>(hd);
    const int KPW = 32 / G;
    const int slotk = lane / G, vi = lane - slotk * G;
    const bool vact = vi * VEC < hd;
    float acc[VEC];
#pragma unroll
    for (int u = 0; u < VEC; u++) acc[u] = 0.0f;
    constexpr int U = 8;  // 8 * KPW rows in flight per warp
    for (int b0 = 0; b0 < m; b0 += KPW * U) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = b0 + u * KPW + slotk;
            if (j < m && vact) VecT<VEC>::fma(acc, my_p[j], V + (long long)my_idx[j] * hd + vi * VEC);
        }
    }
    // reduce over the key slots of the warp (lanes with the same vi)
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

    float *o_h = opart;  // merged head output [hd] (reuses warp 0's slot)
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
    }
    // ---- merge (i, h): sum partials, self term, normalise, append ----
    {
        const float *pp = a.part + ((long long)i * a.H + h) * a.nsplit * (hd + 1);
        float od = 0.0f, vn = 0.0f, lall = 0.0f;
        const int d = tid;
        if (d < hd) {
            if (n_act > 1) {
                for (int sp = 0; sp < n_act; sp++) {
                    od += __ldcg(pp + (long long)sp * (hd + 1) + d);
                    lall += __ldcg(pp + (long long)sp * (hd + 1) + hd);
                }
            } else {
#pragma unroll
                for (int w = 0; w < DEC_WARPS; w++) {
                    od += opart[w * hd + d];
                    lall += lpart[w];
                }
            }
            vn = a.bv[h * hd + d];
            for (int q = 0; q < P; q++) vn += vpart[q * hd + d];
        }
        __syncthreads();  // opart is overwritten below
        if (d < hd) {
            // self term p = exp(1 - 1) = 1 (kv_cache.rs:294, :318)
            o_h[d] = (od + vn) / (lall + 1.0f);
            a.sv.v[(base + n) * hd + d] = vn;  // append value (kv_cache.rs:324)
        }
    }
    if (tid == 0) {
        a.sv.theta[base + n] = thq;  // append phase and bucket (kv_cache.rs:323-326)
        a.sv.bucket[base + n] = (uint8_t)qb;
        if (n_act > 1) a.ticket[(long long)i * a.H + h] = 0u;
    }
    __syncthreads();
    // this head's slice of out_proj: yh[c] = sum_d Wo[c][h*hd + d] o_h[d]
    float *yh = a.yh + ((long long)i * a.H + h) * E;
    const float *wo = a.wo_t + (long long)h * hd * E;
    for (int c0 = tid; c0 < E; c0 += DEC_THREADS * 4) {
        float acc2[4];
#pragma unroll
        for (int q = 0; q < 4; q++) acc2[q] = 0.0f;
#pragma unroll 8
        for (int dd = 0; dd < hd; dd++) {
            const float od = o_h[dd];
            const float *wr = wo + (long long)dd * E;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const int c = c0 + q * DEC_THREADS;
                if (c < E) acc2[q] = fmaf(__ldg(wr + c), od, acc2[q]);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int c = c0 + q * DEC_THREADS;
            if (c < E) yh[c] = acc2[q];
        }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned t = atomicAdd(a.hticket + i, 1u);
        s_flag = (t == (unsigned)(a.H - 1));
    }
    __syncthreads();
    if (!s_flag) return;
    __threadfence();
    // last head of sequence i: y = b + sum_h yh (head order)
    const float *yall = a.yh + (long long)i * a.H * E;
    for (int c = tid; c < E; c += DEC_THREADS) {
        float v = 0.0f;
#pragma unroll 8
        for (int hh = 0; hh < a.H; hh++) v += __ldcg(yall + (long long)hh * E + c);
        a.y[(long long)i * E + c] = v + a.bo[c];
    }
    if (tid == 0) a.hticket[i] = 0u;
}

size_t decode_scratch_bytes(int n_seq, int H, int hd, int E, int cap) {
    const int nsplit = (cap + DEC_CHUNK - 1) / DEC_CHUNK;
    Carve c;
    c.take<float>((size_t)n_seq * H * nsplit * (hd + 1));
    c.take<float>((size_t)n_seq * H * E);
    c.take<unsigned int>((size_t)n_seq * H);
    c.take<unsigned int>((size_t)n_seq);
    return c.off;
}

int launch_decode_fused(const DecodeLaunch &L, void *scratch, size_t scratch_bytes, cudaStream_t st,
                        std::string *msg) {
    const int nsplit = (L.cap + DEC_CHUNK - 1) / DEC_CHUNK;
    if (scratch_bytes < decode_scratch_bytes(L.n_seq, L.H, L.hd, L.E, L.cap)) {
        *msg = "decode scratch too small";
        return WB_EINVAL;
    }
    Carve c;
    char *s = (char *)scratch;
    DecodeArgs a;
    a.sv = L.sv;
    a.len = L.len;
    a.cap = L.cap;
    a.n_slots = L.n_slots;
    a.x = L.x;
    a.wrs_t = L.wrs_t;
    a.brs = L.brs;
    a.wv_t = L.wv_t;
    a.bv = L.bv;
    a.wo_t = L.wo_t;
    a.bo = L.bo;
    a.hn = L.hn;
    a.n_seq = L.n_seq;
    a.H = L.H;
    a.hd = L.hd;
    a.E = L.E;
    a.nsplit = nsplit;
    a.part = (float *)(s + c.take<float>((size_t)L.n_seq * L.H * nsplit * (L.hd + 1)));
    a.yh = (float *)(s + c.take<float>((size_t)L.n_seq * L.H * L.E));
    a.ticket = (unsigned int *)(s + c.take<unsigned int>((size_t)L.n_seq * L.H));
    a.hticket = (unsigned int *)(s + c.take<unsigned int>((size_t)L.n_seq));
    a.y = L.y;
    a.dev_err = L.dev_err;
    const size_t smem = sizeof(float) * ((size_t)L.E + 2 * DEC_WARPS * DEC_KEYS_PER_WARP + DEC_WARPS * L.hd +
                                         DEC_WARPS + 2 * DEC_WARPS + DEC_THREADS);
    dim3 grid(nsplit, L.H, L.n_seq);
    ProfScope ps("decode_fused", st);
    if (L.hd % 4 == 0) {
        cudaFuncSetAttribute(decode_fused_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        decode_fused_kernel<4><<<grid, DEC_THREADS, smem, st>>>(a);
    } else if (L.hd % 2 == 0) {
        cudaFuncSetAttribute(decode_fused_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        decode_fused_kernel<2><<<grid, DEC_THREADS, smem, st>>>(a);
    } else {
        cudaFuncSetAttribute(decode_fused_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        decode_fused_kernel<1><<<grid, DEC_THREADS, smem, st>>>(a);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        *msg = std::string("decode launch failed: ") + cudaGetErrorString(e);
        return WB_ECUDA;
    }
    return WB_OK;
}

}  // namespace wb
