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
//   theta [slot(b)*seq_stride + h*cap + t]
//   bucket[slot(b)*seq_stride + h*cap + t]
//   V     [(slot(b)*seq_stride + h*cap + t) * hd + dd]
struct WbSeqView {
    float *theta;
    uint8_t *bucket;
    float *v;
    long long seq_stride;  // = n_head * cap
    int cap;               // positions per (seq, head)
    const int32_t *slot;   // batch index -> slot (nullptr = identity)
};

__device__ __forceinline__ long long wb_slot_base(const WbSeqView &s, int b, int h) {
    int slot = s.slot ? s.slot[b] : b;
    return (long long)slot * s.seq_stride + (long long)h * s.cap;
}
