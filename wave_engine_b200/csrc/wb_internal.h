// wb_internal.h -- declarations shared by the library's translation units.
#pragma once
#include "wb_common.cuh"

#include <string>

namespace wb {

// Grow-only device buffer owned by a context.
struct Workspace {
    void *p = nullptr;
    size_t n = 0;
};

// Make *w at least `bytes` long.  Growing frees the old buffer (cudaFree
// synchronises the device, so no kernel still uses it).  Returns WB_OK or
// WB_ENOMEM with *msg set.
inline int ws_ensure(Workspace *w, size_t bytes, std::string *msg) {
    if (bytes <= w->n) return 0;
    if (w->p) cudaFree(w->p);
    w->p = nullptr;
    w->n = 0;
    const size_t want = bytes + bytes / 8;
    if (cudaMalloc(&w->p, want) != cudaSuccess) {
        cudaGetLastError();
        if (msg) *msg = "cudaMalloc of " + std::to_string(want) + " bytes failed";
        return -2;  // WB_ENOMEM
    }
    w->n = want;
    return 0;
}

// Bump allocator handing out 256-byte aligned offsets into one buffer.
struct Carve {
    size_t off = 0;
    template <class T>
    size_t take(size_t count) {
        size_t o = off;
        off += (count * sizeof(T) + 255) & ~size_t(255);
        return o;
    }
};

// ---- kernel timing (wb_context_profile) ---------------------------------
// When a profiler is active on the calling thread, prof_begin/prof_end
// bracket a named kernel launch with CUDA events on its stream.
struct Profiler;
Profiler *&prof_current();
void prof_begin(const char *name, cudaStream_t st);
void prof_end(cudaStream_t st);
Profiler *prof_create(const char *filter);
void prof_destroy(Profiler *p);
std::string prof_report(Profiler *p);
// RAII bracket used at launch sites.
struct ProfScope {
    cudaStream_t st;
    ProfScope(const char *name, cudaStream_t s) : st(s) { prof_begin(name, s); }
    ~ProfScope() { prof_end(st); }
};

enum { OUT_DENSE = 0, OUT_SEQ_V = 1 };
struct OutMap {
    int mode;
    float *y;       // OUT_DENSE: Y[r*ldy + n]
    long long ldy;
    WbSeqView sv;   // OUT_SEQ_V: value rows of head h
    int h;
    int T;
};

// Device weights in the SIMT (input-major) layouts used by the projections.
struct ProjWeights {
    int E, H, hd, C;
    const float *wrs_t, *brs;  // [E][H][2], [H][2]
    const float *wc_t, *bc;    // [E][H*C], [H*C]
    const float *wv_t, *bv;    // [H][hd][hd] (in, out), [H][hd]
};

// ---- SIMT (exact) kernels: wb_simt.cu ----
// phases/buckets/values into sv, (r,s) into rs [R][H][2], content into
// content [R][H*C] when non-null.
void launch_projections_exact(const ProjWeights &w, const float *x, int B, int T, const WbSeqView &sv, float *rs,
                              float *content, cudaStream_t st);
void launch_attn_simt_fallback_f32(const WbSeqView &sv, const float *content, int C, float content_scale,
                                   const float *harmonic_n, int B, int H, int T, int hd, float *o,
                                   const int *tile_list, int h0, int Hg, cudaStream_t st);
void launch_attn_simt_fallback_bf16(const WbSeqView &sv, const float *content, int C, float content_scale,
                                    const float *harmonic_n, int B, int H, int T, int hd, __nv_bfloat16 *o,
                                    const int *tile_list, int h0, int Hg, cudaStream_t st);
void launch_seqdot(const float *X, int R, int K, long long ldx, const float *Wt, int N,
                   const float *bias, int bias_first, const OutMap &om, cudaStream_t st);
void launch_phase(const float *rs, int R, int H, int T, const WbSeqView &sv, cudaStream_t st);
void launch_attn_simt(const WbSeqView &sv, const float *content, int C, float content_scale,
                      const float *harmonic_n, int B, int H, int T, int hd, float *o,
                      float *att_w, cudaStream_t st);
void launch_decode_simt(const WbSeqView &sv, const int32_t *len, const float *theta_new,
                        const float *v_new, const float *harmonic_n, int n_seq, int H, int hd,
                        float *o, uint32_t *dev_err, cudaStream_t st);
void launch_theta_only(const float *rs, int n, float *theta, cudaStream_t st);
// dst[0 .. n) = src[0 .. n) with 16-byte loads; n a multiple of 4, both
// 16-byte aligned (src may be the device alias of pinned host memory).
void launch_copy_f4(const float *src, float *dst, long long n, cudaStream_t st);
void launch_len_update(int32_t *len, const int32_t *slots, int n_seq, int value, int set, int n_slots, int cap,
                       cudaStream_t st, const int32_t *pages = nullptr, int max_pages = 0);
// Causal dot-product attention core (compute.rs:357-414): qkv [B*T][3E] ->
// o [B*T][E] (head-major columns).
int launch_dot_attn(const float *qkv, int B, int T, int E, int H, float *o, cudaStream_t st, std::string *msg);
// The same core for the 128-query tiles listed in tiles[1 .. tiles[0]]
// (device; entries (b * H + h) * ceil(T / 128) + tile), at most max_tiles.
int launch_dot_attn_tiles(const float *qkv, int B, int T, int E, int H, float *o, const int *tiles, int max_tiles,
                          cudaStream_t st, std::string *msg);
void launch_bucket_from_theta(const float *theta, uint8_t *bucket, long long n, cudaStream_t st);

}  // namespace wb
