// wb_common.cuh -- shared definitions for the B200 wave-attention kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define WB_N_BUCKETS 8
// std::f32::consts::TAU rounded to f32 (6.2831855f).
#define WB_TAU 6.28318548202514648438f

// Device error word bits (ctx->dev_err).  Kernels never trap; they record
// the failure here and return.
#define WB_DERR_TIMEOUT_TMA 0x1u
#define WB_DERR_TIMEOUT_MMA 0x2u
#define WB_DERR_TIMEOUT_SOFTMAX 0x4u
#define WB_DERR_BOUNDS 0x8u
#define WB_DERR_TIMEOUT_DECODE 0x10u

namespace wb {

// Phase -> bucket, bit-exact restatement of src/common/kv_cache.rs:66-70
// (identical to attn.rs:171-174): IEEE fmodf, IEEE add and divide, then a
// saturating float->usize cast clamped to 7.
__device__ __forceinline__ int phase_to_bucket(float phase) {
    const float bucket_width = WB_TAU / (float)WB_N_BUCKETS;  // exact (power-of-two divide)
    float normalized = fmodf(__fadd_rn(fmodf(phase, WB_TAU), WB_TAU), WB_TAU);
    float q = __fdiv_rn(normalized, bucket_width);
    int b = (q != q || q <= 0.0f) ? 0 : (q >= 7.0f ? 7 : (int)q);
    return b;
}

// Bucket adjacency of src/common/attn.rs:189-196: key bucket in
// {qb-1, qb, qb+1} mod 8, expressed as an 8-bit allowed mask of the query.
__device__ __forceinline__ uint32_t allowed_bucket_mask(int qb) {
    uint32_t m = (1u << qb) | (1u << ((qb + 1) & 7)) | (1u << ((qb + 7) & 7));
    return m;
}

// softplus of src/common/math/core.rs:5 (host and device agree on the
// formula; the host computes it once per head with glibc).
__host__ __device__ inline float softplus_ref(float x) {
    return x > 20.0f ? x : logf(1.0f + expf(x));
}

// A warp's 32 x 32 fp32 block, thread = row with its 32 columns in r[],
// written to the warp's buffer (32 rows padded to 33 floats: conflict-free
// both ways) so that row j can then be read with the lanes along columns:
// buf[j * 33 + lane].  Used by the tensor-core epilogues: a store
// instruction then covers one contiguous 128-byte row segment instead of 32
// rows.
__device__ __forceinline__ void warp_stage32(float *buf, const uint32_t (&r)[32], int lane) {
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 32; i++) buf[lane * 33 + i] = __uint_as_float(r[i]);
    __syncwarp();
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace wb

// Per-sequence view of phases / buckets / values, shared by the attention
// forward (temporary slots, one per batch element) and the KV cache (one
// slot per sequence and layer).  Element (seq b, head h, pos t):
//   contiguous (pages == nullptr):
//     theta [slot(b)*seq_stride + h*cap + t]     (seq_stride = n_head * cap)
//   paged (a paged KV cache): position t lives in page
//     pages[slot(b)*max_pages + t / WB_PAGE], each page holding WB_PAGE
//     positions of every head:
//     theta [page*seq_stride + h*cap + t % WB_PAGE]  (cap = WB_PAGE,
//                                                     seq_stride = n_head * WB_PAGE)
//   bucket at the same index, V at index * hd + dd.
// Either way the index of (b, h, t) is row(b, t) + h * cap, which is what
// the row-wise kernels use; a page id < 0 (unmapped) gives index -1.
static constexpr int WB_PAGE = 128;  // positions per KV page (the decode kernel's keys per warp)
static constexpr int WB_PAGE_SHIFT = 7;

struct WbSeqView {
    float *theta;
    uint8_t *bucket;
    float *v;
    long long seq_stride;
    int cap;
    const int32_t *slot;              // batch index -> slot (nullptr = identity)
    const int32_t *pages = nullptr;   // paged: [slot][max_pages] page ids (-1 unmapped)
    int max_pages = 0;
};

// index of (slot, head 0, position t), or -1 when t's page is unmapped
__device__ __forceinline__ long long wb_row_slot(const WbSeqView &s, int slot, int t) {
    if (s.pages) {
        const int pg = s.pages[(long long)slot * s.max_pages + (t >> WB_PAGE_SHIFT)];
        return pg < 0 ? -1LL : (long long)pg * s.seq_stride + (t & (WB_PAGE - 1));
    }
    return (long long)slot * s.seq_stride + t;
}
__device__ __forceinline__ long long wb_row(const WbSeqView &s, int b, int t) {
    return wb_row_slot(s, s.slot ? s.slot[b] : b, t);
}
// index of (seq b, head h, position t), or -1 (unmapped page)
__device__ __forceinline__ long long wb_pos(const WbSeqView &s, int b, int h, int t) {
    const long long r = wb_row(s, b, t);
    return r < 0 ? -1LL : r + (long long)h * s.cap;
}

// a slot of a paged cache may hold position t only when t's page is mapped
// (always true without a page table)
__device__ __forceinline__ bool wb_pos_mapped(const int32_t *pages, int max_pages, int slot, int t) {
    if (!pages) return true;
    const int p = t >> WB_PAGE_SHIFT;
    return t >= 0 && p < max_pages && pages[(long long)slot * max_pages + p] >= 0;
}

// contiguous views only: index of (seq b, head h, position 0)
__device__ __forceinline__ long long wb_slot_base(const WbSeqView &s, int b, int h) {
    int slot = s.slot ? s.slot[b] : b;
    return (long long)slot * s.seq_stride + (long long)h * s.cap;
}
