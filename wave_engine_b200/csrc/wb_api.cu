// wb_api.cu -- C ABI entry points (include/wave_b200.h): argument checks,
// device-resident weights, workspace management and kernel sequencing.
#include "wave_b200.h"
#include "wave_b200_testing.h"
#include "wb_internal.h"
#include "wb_tc.h"
#include "wb_decode.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace {

thread_local std::string g_err;

int fail(int code, const std::string &msg) {
    g_err = msg;
    return code;
}

#define WB_CUDA(expr)                                                                     \
    do {                                                                                  \
        cudaError_t e_ = (expr);                                                          \
        if (e_ != cudaSuccess)                                                            \
            return fail(WB_ECUDA, std::string(#expr) + ": " + cudaGetErrorString(e_));   \
    } while (0)

#define WB_TRY(expr)                 \
    do {                             \
        int rc_ = (expr);            \
        if (rc_ != WB_OK) return rc_; \
    } while (0)

using DevBuf = wb::Workspace;

int ensure(DevBuf &b, size_t bytes) {
    std::string msg;
    int rc = wb::ws_ensure(&b, bytes, &msg);
    return rc == WB_OK ? rc : fail(rc, msg);
}

using wb::Carve;

// Restores the calling thread's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

bool is_device_ptr(const void *p) {
    if (!p) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

template <class T>
int upload(T **dst, const std::vector<T> &src) {
    *dst = nullptr;
    if (src.empty()) return WB_OK;
    if (cudaMalloc(dst, src.size() * sizeof(T)) != cudaSuccess) {
        cudaGetLastError();
        return fail(WB_ENOMEM, "cudaMalloc for weights failed");
    }
    WB_CUDA(cudaMemcpy(*dst, src.data(), src.size() * sizeof(T), cudaMemcpyHostToDevice));
    return WB_OK;
}

}  // namespace

struct wb_context {
    int device = 0;
    int sm_count = 0;
    cudaStream_t own = nullptr;
    cudaStream_t stream = nullptr;
    DevBuf ws;    // per-call scratch
    DevBuf io;    // staging of host inputs/outputs
    uint32_t *dev_err = nullptr;
    wb::Profiler *prof = nullptr;
};

// Makes ctx's profiler the calling thread's current one for one API call.
struct ProfBind {
    wb::Profiler *prev;
    explicit ProfBind(wb_context *c) : prev(wb::prof_current()) { wb::prof_current() = c->prof; }
    ~ProfBind() { wb::prof_current() = prev; }
};

struct wb_attn_layer {
    wb_context *ctx = nullptr;
    int device = 0;  // destroy must not touch ctx (it may already be gone)
    int E = 0, H = 0, hd = 0, C = 0;
    std::vector<float> hn_host;  // softplus(harmonic_raw)
    float *harmonic_n = nullptr; // [H]
    // SIMT layouts (transposed so threads read consecutive outputs)
    float *wrs_t = nullptr, *brs = nullptr;  // [E][H][2], [H][2]
    float *wrs_h = nullptr;                  // [H][E][2]: one head's phase weights contiguous (decode)
    float *wc_t = nullptr, *bc = nullptr;    // [E][H*C], [H*C]
    float *wv_t = nullptr, *bv = nullptr;    // [H][hd][hd] (in, out), [H][hd]
    float *wo_t = nullptr, *bo = nullptr;    // [E][E] (in, out), [E]
    // tensor-core layouts
    wb::TcLayerWeights tc;
};

static wb::ProjWeights proj_weights(const wb_attn_layer *L) {
    return wb::ProjWeights{L->E, L->H, L->hd, L->C, L->wrs_t, L->brs, L->wc_t, L->bc, L->wv_t, L->bv};
}

struct wb_dot_attn_layer {
    wb_context *ctx = nullptr;
    int device = 0;
    int E = 0, H = 0;
    float *w_qkv = nullptr, *wt_qkv = nullptr, *b_qkv = nullptr;  // [3E][E] (GEMM), [E][3E] (SIMT), [3E]
    float *w_o = nullptr, *wt_o = nullptr, *b_o = nullptr;        // [E][E], [E][E] transposed, [E]
};

struct wb_kv_cache {
    wb_context *ctx = nullptr;
    int device = 0;  // destroy must not touch ctx (it may already be gone)
    int L = 0, H = 0, hd = 0, S = 0, cap = 0;
    float *theta = nullptr;
    uint8_t *bucket = nullptr;
    float *v = nullptr;
    int32_t *len = nullptr;            // device [L][S] (the truth)
    wb::Workspace dscratch;            // decode partials + tickets, sized for (S, cap), zeroed
    std::vector<int32_t> len_host;     // host mirror [L][S]
    bool len_stale = false;            // a call with device seq ids changed lengths on the device
    // The last decode of this cache whose final kernel was the SIMT out_proj
    // (which lets a programmatic dependent launch before it completes): its
    // layer and stream, or -1.  The next tensor-path decode launches its
    // attention grid as such a dependent only on the same stream and for
    // another layer: that grid reads the layer's lengths and keys before it
    // waits, and the out_proj of the same layer may still be writing them.
    int out_layer = -1;
    cudaStream_t out_stream = nullptr;
    bool chain_ok(int layer, cudaStream_t st) const { return out_layer >= 0 && out_layer != layer && out_stream == st; }
    void note_decode(int layer, cudaStream_t st, bool ends_with_out) {
        out_layer = ends_with_out ? layer : -1;
        out_stream = st;
    }
    int refresh(cudaStream_t st) {
        if (!len_stale) return WB_OK;
        if (cudaStreamSynchronize(st) != cudaSuccess ||
            cudaMemcpy(len_host.data(), len, len_host.size() * sizeof(int32_t), cudaMemcpyDeviceToHost) !=
                cudaSuccess)
            return WB_ECUDA;
        len_stale = false;
        return WB_OK;
    }
    WbSeqView view(int layer, const int32_t *slots) const {
        const long long per_layer = (long long)S * H * cap;
        WbSeqView s;
        s.theta = theta + layer * per_layer;
        s.bucket = bucket + layer * per_layer;
        s.v = v + layer * per_layer * hd;
        s.seq_stride = (long long)H * cap;
        s.cap = cap;
        s.slot = slots;
        return s;
    }
};

extern "C" {

int wb_abi_version(void) { return WB_ABI_VERSION; }

const char *wb_last_error(void) { return g_err.c_str(); }

int wb_context_create(int device, wb_context **out) {
    if (!out) return fail(WB_EINVAL, "out is NULL");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return fail(WB_ENODEV, "no CUDA device visible");
    }
    if (device < 0 || device >= n) return fail(WB_EINVAL, "device ordinal out of range");
    cudaDeviceProp prop;
    WB_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(WB_ENODEV, std::string("device is not sm_100 (B200): ") + prop.name);
    DeviceGuard g(device);
    if (!g.ok) return fail(WB_ECUDA, "cudaSetDevice failed");
    wb_context *c = new wb_context();
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    if (cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->dev_err, sizeof(uint32_t)) != cudaSuccess ||
        cudaMemset(c->dev_err, 0, sizeof(uint32_t)) != cudaSuccess) {
        cudaGetLastError();
        if (c->own) cudaStreamDestroy(c->own);
        if (c->dev_err) cudaFree(c->dev_err);
        delete c;
        return fail(WB_ECUDA, "context allocation failed");
    }
    c->stream = c->own;
    *out = c;
    return WB_OK;
}

int wb_context_destroy(wb_context *ctx) {
    if (!ctx) return WB_OK;
    DeviceGuard g(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->ws.p) cudaFree(ctx->ws.p);
    if (ctx->io.p) cudaFree(ctx->io.p);
    if (ctx->dev_err) cudaFree(ctx->dev_err);
    if (ctx->own) cudaStreamDestroy(ctx->own);
    wb::prof_destroy(ctx->prof);
    delete ctx;
    return WB_OK;
}

int wb_context_set_stream(wb_context *ctx, void *cuda_stream) {
    if (!ctx) return fail(WB_EINVAL, "ctx is NULL");
    ctx->stream = (cudaStream_t)cuda_stream;  // NULL = the CUDA default (legacy) stream
    return WB_OK;
}

void *wb_context_own_stream(wb_context *ctx) { return ctx ? (void *)ctx->own : nullptr; }

int wb_context_synchronize(wb_context *ctx) {
    if (!ctx) return fail(WB_EINVAL, "ctx is NULL");
    DeviceGuard g(ctx->device);
    WB_CUDA(cudaStreamSynchronize(ctx->stream));
    return WB_OK;
}

int wb_context_take_device_error(wb_context *ctx, uint32_t *code_out) {
    if (!ctx) return fail(WB_EINVAL, "ctx is NULL");
    DeviceGuard g(ctx->device);
    uint32_t v = 0;
    WB_CUDA(cudaMemcpyAsync(&v, ctx->dev_err, sizeof(v), cudaMemcpyDeviceToHost, ctx->stream));
    WB_CUDA(cudaStreamSynchronize(ctx->stream));
    WB_CUDA(cudaMemsetAsync(ctx->dev_err, 0, sizeof(uint32_t), ctx->stream));
    if (code_out) *code_out = v;
    return WB_OK;
}

int wb_context_profile(wb_context *ctx, const char *name_filter) {
    if (!ctx) return fail(WB_EINVAL, "ctx is NULL");
    DeviceGuard g(ctx->device);
    if (ctx->prof) {
        cudaStreamSynchronize(ctx->stream);
        wb::prof_destroy(ctx->prof);
        ctx->prof = nullptr;
    }
    if (name_filter) ctx->prof = wb::prof_create(name_filter);
    return WB_OK;
}

int wb_context_profile_report(wb_context *ctx, char *buf, size_t len) {
    if (!ctx || !buf || len == 0) return fail(WB_EINVAL, "NULL argument");
    if (!ctx->prof) return fail(WB_EINVAL, "profiling is off (wb_context_profile)");
    DeviceGuard g(ctx->device);
    WB_CUDA(cudaStreamSynchronize(ctx->stream));
    std::string r = wb::prof_report(ctx->prof);
    if (r.size() + 1 > len) return fail(WB_EINVAL, "report buffer too small");
    memcpy(buf, r.c_str(), r.size() + 1);
    return WB_OK;
}

// ---------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------
int wb_attn_layer_create(wb_context *ctx, const wb_attn_weights_desc *w, wb_attn_layer **out) {
    if (!ctx || !w || !out) return fail(WB_EINVAL, "NULL argument");
    *out = nullptr;
    const int E = w->n_embd, H = w->n_head, C = w->content_dim;
    if (E <= 0 || H <= 0 || E % H) return fail(WB_EINVAL, "n_embd must be a positive multiple of n_head");
    if (C != 0 && C != 16) return fail(WB_EINVAL, "content_dim must be 0 or 16");
    const int hd = E / H;
    if (hd > 256) return fail(WB_EINVAL, "head_dim > 256 not supported");
    if (!w->harmonic_raw || !w->phase_proj_w || !w->phase_proj_b || !w->v_proj_w || !w->v_proj_b ||
        !w->out_proj_w || !w->out_proj_b || (C && (!w->content_proj_w || !w->content_proj_b)))
        return fail(WB_EINVAL, "missing weight array");
    DeviceGuard g(ctx->device);
    wb_attn_layer *L = new wb_attn_layer();
    L->ctx = ctx;
    L->device = ctx->device;
    L->E = E; L->H = H; L->hd = hd; L->C = C;
    L->hn_host.resize(H);
    for (int h = 0; h < H; h++) L->hn_host[h] = wb::softplus_ref(w->harmonic_raw[h]);

    std::vector<float> wrs((size_t)E * H * 2), brs((size_t)H * 2);
    for (int h = 0; h < H; h++)
        for (int c = 0; c < 2; c++) {
            brs[h * 2 + c] = w->phase_proj_b[h * 2 + c];
            for (int j = 0; j < E; j++) wrs[((size_t)j * H + h) * 2 + c] = w->phase_proj_w[((size_t)h * 2 + c) * E + j];
        }
    std::vector<float> wrs_h((size_t)H * E * 2);
    for (int h = 0; h < H; h++)
        for (int j = 0; j < E; j++)
            for (int c = 0; c < 2; c++) wrs_h[((size_t)h * E + j) * 2 + c] = w->phase_proj_w[((size_t)h * 2 + c) * E + j];
    std::vector<float> wc, bc;
    if (C) {
        wc.resize((size_t)E * H * C);
        bc.resize((size_t)H * C);
        for (int h = 0; h < H; h++)
            for (int d = 0; d < C; d++) {
                bc[h * C + d] = w->content_proj_b[h * C + d];
                for (int j = 0; j < E; j++)
                    wc[(size_t)j * H * C + h * C + d] = w->content_proj_w[((size_t)h * C + d) * E + j];
            }
    }
    std::vector<float> wv((size_t)H * hd * hd), bv((size_t)H * hd);
    for (int h = 0; h < H; h++)
        for (int dd = 0; dd < hd; dd++) {
            bv[h * hd + dd] = w->v_proj_b[h * hd + dd];
            for (int j = 0; j < hd; j++)
                wv[((size_t)h * hd + j) * hd + dd] = w->v_proj_w[((size_t)h * hd + dd) * hd + j];
        }
    std::vector<float> wo((size_t)E * E), bo(w->out_proj_b, w->out_proj_b + E);
    for (int i = 0; i < E; i++)
        for (int j = 0; j < E; j++) wo[(size_t)j * E + i] = w->out_proj_w[(size_t)i * E + j];

    int rc = WB_OK;
    if (rc == WB_OK) rc = upload(&L->harmonic_n, L->hn_host);
    if (rc == WB_OK) rc = upload(&L->wrs_t, wrs);
    if (rc == WB_OK) rc = upload(&L->wrs_h, wrs_h);
    if (rc == WB_OK) rc = upload(&L->brs, brs);
    if (rc == WB_OK) rc = upload(&L->wc_t, wc);
    if (rc == WB_OK) rc = upload(&L->bc, bc);
    if (rc == WB_OK) rc = upload(&L->wv_t, wv);
    if (rc == WB_OK) rc = upload(&L->bv, bv);
    if (rc == WB_OK) rc = upload(&L->wo_t, wo);
    if (rc == WB_OK) rc = upload(&L->bo, bo);
    if (rc == WB_OK) {
        std::string msg;
        L->tc.pw = proj_weights(L);
        L->tc.harmonic_n = L->harmonic_n;
        L->tc.b_o = L->bo;
        L->tc.wo_t = L->wo_t;
        L->tc.wrs_h = L->wrs_h;
        rc = wb::tc_layer_upload(&L->tc, w, &msg);
        if (rc != WB_OK) fail(rc, msg);
    }
    if (rc != WB_OK) {
        wb_attn_layer_destroy(L);
        return rc;
    }
    *out = L;
    return WB_OK;
}

int wb_attn_layer_destroy(wb_attn_layer *L) {
    if (!L) return WB_OK;
    DeviceGuard g(L->device);
    float *ptrs[] = {L->harmonic_n, L->wrs_t, L->wrs_h, L->brs, L->wc_t, L->bc, L->wv_t, L->bv, L->wo_t, L->bo};
    for (float *p : ptrs)
        if (p) cudaFree(p);
    wb::tc_layer_free(&L->tc);
    delete L;
    return WB_OK;
}

int wb_init_block_attn(uint64_t *rng_state, int n_head, int n_embd, int content_dim, float *harmonic_raw,
                       float *phase_proj_w, float *phase_proj_b, float *v_proj_w, float *v_proj_b,
                       float *content_proj_w, float *content_proj_b, float *out_proj_w, float *out_proj_b) {
    if (!rng_state || n_head <= 0 || n_embd <= 0 || n_embd % n_head || content_dim < 0)
        return fail(WB_EINVAL, "bad init_block_attn arguments");
    if (!harmonic_raw || !phase_proj_w || !phase_proj_b || !v_proj_w || !v_proj_b || !out_proj_w ||
        !out_proj_b || (content_dim && (!content_proj_w || !content_proj_b)))
        return fail(WB_EINVAL, "NULL buffer");
    // xorshift64 of src/common/rng.rs:24-39.
    uint64_t s = *rng_state;
    auto uniform = [&s](float limit) {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        float f = (float)(s >> 40) / (float)(1ull << 24);
        return (f * 2.0f - 1.0f) * limit;
    };
    const int hd = n_embd / n_head;
    const float le = 1.0f / std::sqrt((float)n_embd), ld = 1.0f / std::sqrt((float)hd);
    // init_block_attn (wave_model.rs:57-81): per head phase, value, content; then out_proj.
    for (int h = 0; h < n_head; h++) {
        for (size_t i = 0; i < (size_t)2 * n_embd; i++) phase_proj_w[(size_t)h * 2 * n_embd + i] = uniform(le);
        phase_proj_b[2 * h] = phase_proj_b[2 * h + 1] = 0.0f;
        for (size_t i = 0; i < (size_t)hd * hd; i++) v_proj_w[(size_t)h * hd * hd + i] = uniform(ld);
        for (int i = 0; i < hd; i++) v_proj_b[h * hd + i] = 0.0f;
        if (content_dim) {
            for (size_t i = 0; i < (size_t)content_dim * n_embd; i++)
                content_proj_w[(size_t)h * content_dim * n_embd + i] = uniform(le);
            for (int i = 0; i < content_dim; i++) content_proj_b[h * content_dim + i] = 0.0f;
        }
        harmonic_raw[h] = std::log((float)(h + 1) * 0.5f);
    }
    for (size_t i = 0; i < (size_t)n_embd * n_embd; i++) out_proj_w[i] = uniform(le);
    for (int i = 0; i < n_embd; i++) out_proj_b[i] = 0.0f;
    *rng_state = s;
    return WB_OK;
}

// ---------------------------------------------------------------------------
// prefill forward
// ---------------------------------------------------------------------------
static int run_projections_exact(wb_context *ctx, const wb_attn_layer *L, const float *x, int B, int T,
                                 const WbSeqView &sv, float *rs, float *content, bool use_content) {
    wb::launch_projections_exact(proj_weights(L), x, B, T, sv, rs, use_content ? content : nullptr, ctx->stream);
    WB_CUDA(cudaGetLastError());
    return WB_OK;
}

int wb_attn_forward_heads(wb_context *ctx, const wb_attn_layer *L, const float *x, int B, int T, int head_begin,
                          int head_end, int add_bias, int flags, float *y) {
    if (!ctx || !L || !x || !y) return fail(WB_EINVAL, "NULL argument");
    if (L->ctx != ctx) return fail(WB_EINVAL, "layer belongs to another context");
    if (flags & ~WB_NO_CONTENT) return fail(WB_EINVAL, "wb_attn_forward_heads takes WB_NO_CONTENT only (tensor path)");
    if (head_begin < 0 || head_end > L->H || head_begin >= head_end) return fail(WB_EINVAL, "bad head range");
    if (B < 0 || T < 0) return fail(WB_EINVAL, "negative batch or seq_len");
    if (B == 0 || T == 0) return WB_OK;
    const long long R = (long long)B * T;
    if (R > (1LL << 30)) return fail(WB_EINVAL, "batch*seq_len too large");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    const int E = L->E;
    const bool use_content = L->C > 0 && !(flags & WB_NO_CONTENT);
    const bool x_dev = is_device_ptr(x), y_dev = is_device_ptr(y);
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>(R * E);
    size_t o_y = y_dev ? 0 : io.take<float>(R * E);
    WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    float *yd = y_dev ? y : (float *)(iob + o_y);
    if (!x_dev) WB_CUDA(cudaMemcpyAsync((void *)xd, x, R * E * sizeof(float), cudaMemcpyHostToDevice, st));
    std::string msg;
    const int rc = wb::tc_attn_forward(L->tc, xd, B, T, use_content, yd, nullptr, &ctx->ws, ctx->dev_err,
                                       ctx->sm_count, st, &msg, head_begin, head_end, add_bias != 0);
    if (rc != WB_OK) return fail(rc, msg);
    if (!y_dev) {
        WB_CUDA(cudaMemcpyAsync(y, yd, R * E * sizeof(float), cudaMemcpyDeviceToHost, st));
        WB_CUDA(cudaStreamSynchronize(st));
        uint32_t derr = 0;
        WB_CUDA(cudaMemcpy(&derr, ctx->dev_err, sizeof(derr), cudaMemcpyDeviceToHost));
        if (derr) return fail(WB_ETIMEOUT, "device-side check failed, error word " + std::to_string(derr));
    }
    return WB_OK;
}

int wb_attn_forward(wb_context *ctx, const wb_attn_layer *L, const float *x, int B, int T, int flags,
                    float *y, float *att_w, float *phases_out) {
    if (!ctx || !L || !x || !y) return fail(WB_EINVAL, "NULL argument");
    if (L->ctx != ctx) return fail(WB_EINVAL, "layer belongs to another context");
    if (flags & WB_RETURN_PATHWAY)
        return fail(WB_ENOTSUP, "return_pathway_cache (WaveAttnCache for backward) is not supported");
    if (flags & ~(WB_PATH_EXACT | WB_NO_CONTENT)) return fail(WB_EINVAL, "unknown flag bits");
    if (B < 0 || T < 0) return fail(WB_EINVAL, "negative batch or seq_len");
    if (B == 0 || T == 0) return WB_OK;
    const long long R = (long long)B * T;
    if (R > (1LL << 30)) return fail(WB_EINVAL, "batch*seq_len too large");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    const int E = L->E, H = L->H, hd = L->hd;
    const bool use_content = L->C > 0 && !(flags & WB_NO_CONTENT);
    const bool exact = (flags & WB_PATH_EXACT) || att_w != nullptr;
    const bool x_dev = is_device_ptr(x), y_dev = is_device_ptr(y);
    const bool aw_dev = att_w && is_device_ptr(att_w), ph_dev = phases_out && is_device_ptr(phases_out);

    // staging for host buffers
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>(R * E);
    size_t o_y = y_dev ? 0 : io.take<float>(R * E);
    size_t o_aw = (att_w && !aw_dev) ? io.take<float>((size_t)B * H * T * T) : 0;
    size_t o_ph = (phases_out && !ph_dev) ? io.take<float>((size_t)B * H * T) : 0;
    WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    float *yd = y_dev ? y : (float *)(iob + o_y);
    float *awd = att_w ? (aw_dev ? att_w : (float *)(iob + o_aw)) : nullptr;
    if (!x_dev) WB_CUDA(cudaMemcpyAsync((void *)xd, x, R * E * sizeof(float), cudaMemcpyHostToDevice, st));

    int rc;
    if (exact) {
        Carve c;
        size_t o_rs = c.take<float>(R * 2 * H);
        size_t o_ct = c.take<float>(use_content ? R * H * L->C : 1);
        size_t o_th = c.take<float>(R * H);
        size_t o_bk = c.take<uint8_t>(R * H);
        size_t o_v = c.take<float>(R * H * hd);
        size_t o_o = c.take<float>(R * E);
        WB_TRY(ensure(ctx->ws, c.off));
        char *w = (char *)ctx->ws.p;
        WbSeqView sv;
        sv.theta = (float *)(w + o_th);
        sv.bucket = (uint8_t *)(w + o_bk);
        sv.v = (float *)(w + o_v);
        sv.seq_stride = (long long)H * T;
        sv.cap = T;
        sv.slot = nullptr;
        float *content = (float *)(w + o_ct), *o = (float *)(w + o_o);
        WB_TRY(run_projections_exact(ctx, L, xd, B, T, sv, (float *)(w + o_rs), content, use_content));
        wb::launch_attn_simt(sv, use_content ? content : nullptr, use_content ? L->C : 0,
                             use_content ? 1.0f / std::sqrt((float)L->C) : 0.0f, L->harmonic_n, B, H, T, hd, o,
                             awd, st);
        wb::OutMap om{wb::OUT_DENSE, yd, E, sv, 0, T};
        wb::launch_seqdot(o, (int)R, E, E, L->wo_t, E, L->bo, 0, om, st);
        if (phases_out) {
            float *phd = ph_dev ? phases_out : (float *)(iob + o_ph);
            WB_CUDA(cudaMemcpyAsync(phd, sv.theta, R * H * sizeof(float), cudaMemcpyDeviceToDevice, st));
        }
        WB_CUDA(cudaGetLastError());
    } else {
        std::string msg;
        float *phd = phases_out ? (ph_dev ? phases_out : (float *)(iob + o_ph)) : nullptr;
        rc = wb::tc_attn_forward(L->tc, xd, B, T, use_content, yd, phd, &ctx->ws, ctx->dev_err,
                                 ctx->sm_count, st, &msg);
        if (rc != WB_OK) return fail(rc, msg);
    }
    if (!y_dev) WB_CUDA(cudaMemcpyAsync(y, yd, R * E * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (att_w && !aw_dev)
        WB_CUDA(cudaMemcpyAsync(att_w, awd, (size_t)B * H * T * T * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (phases_out && !ph_dev)
        WB_CUDA(cudaMemcpyAsync(phases_out, iob + o_ph, R * H * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (!y_dev || (att_w && !aw_dev) || (phases_out && !ph_dev)) {
        WB_CUDA(cudaStreamSynchronize(st));
        uint32_t derr = 0;
        WB_CUDA(cudaMemcpy(&derr, ctx->dev_err, sizeof(derr), cudaMemcpyDeviceToHost));
        if (derr) return fail(WB_ETIMEOUT, "device-side check failed, error word " + std::to_string(derr));
    }
    return WB_OK;
}

// ---------------------------------------------------------------------------
// Dot-product attention (compute.rs:357-414)
// ---------------------------------------------------------------------------
int wb_dot_attn_layer_create(wb_context *ctx, int n_head, int n_embd, const float *c_attn_w, const float *c_attn_b,
                             const float *c_proj_w, const float *c_proj_b, wb_dot_attn_layer **out) {
    if (!ctx || !c_attn_w || !c_attn_b || !c_proj_w || !c_proj_b || !out) return fail(WB_EINVAL, "NULL argument");
    *out = nullptr;
    if (n_head <= 0 || n_embd <= 0 || n_embd % n_head) return fail(WB_EINVAL, "n_embd must be a multiple of n_head");
    if (n_embd / n_head > 128) return fail(WB_ENOTSUP, "dot-product attention supports head_dim <= 128");
    DeviceGuard g(ctx->device);
    const int E = n_embd;
    std::vector<float> wq(c_attn_w, c_attn_w + (size_t)3 * E * E), bq(c_attn_b, c_attn_b + 3 * E);
    std::vector<float> wo(c_proj_w, c_proj_w + (size_t)E * E), bo(c_proj_b, c_proj_b + E);
    std::vector<float> wqt((size_t)E * 3 * E), wot((size_t)E * E);
    for (int n = 0; n < 3 * E; n++)
        for (int j = 0; j < E; j++) wqt[(size_t)j * 3 * E + n] = wq[(size_t)n * E + j];
    for (int n = 0; n < E; n++)
        for (int j = 0; j < E; j++) wot[(size_t)j * E + n] = wo[(size_t)n * E + j];
    wb_dot_attn_layer *L = new wb_dot_attn_layer();
    L->ctx = ctx;
    L->device = ctx->device;
    L->E = E;
    L->H = n_head;
    int rc = upload(&L->w_qkv, wq);
    if (rc == WB_OK) rc = upload(&L->wt_qkv, wqt);
    if (rc == WB_OK) rc = upload(&L->b_qkv, bq);
    if (rc == WB_OK) rc = upload(&L->w_o, wo);
    if (rc == WB_OK) rc = upload(&L->wt_o, wot);
    if (rc == WB_OK) rc = upload(&L->b_o, bo);
    if (rc != WB_OK) {
        wb_dot_attn_layer_destroy(L);
        return rc;
    }
    *out = L;
    return WB_OK;
}

int wb_dot_attn_layer_destroy(wb_dot_attn_layer *L) {
    if (!L) return WB_OK;
    DeviceGuard g(L->device);
    float *ptrs[] = {L->w_qkv, L->wt_qkv, L->b_qkv, L->w_o, L->wt_o, L->b_o};
    for (float *p : ptrs)
        if (p) cudaFree(p);
    delete L;
    return WB_OK;
}

int wb_dot_attn_forward(wb_context *ctx, const wb_dot_attn_layer *L, const float *x, int B, int T, int flags,
                        float *y) {
    if (!ctx || !L || !x || !y) return fail(WB_EINVAL, "NULL argument");
    if (L->ctx != ctx) return fail(WB_EINVAL, "layer belongs to another context");
    if (flags & ~WB_PATH_EXACT) return fail(WB_EINVAL, "unknown flag bits");
    if (B < 0 || T < 0) return fail(WB_EINVAL, "negative batch or seq_len");
    if (B == 0 || T == 0) return WB_OK;
    const long long R = (long long)B * T;
    if (R > (1LL << 30)) return fail(WB_EINVAL, "batch*seq_len too large");
    const bool exact = flags & WB_PATH_EXACT;
    const int E = L->E, H = L->H;
    if (!exact && E % 4) return fail(WB_ENOTSUP, "the tensor path needs n_embd to be a multiple of 4");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    const bool x_dev = is_device_ptr(x), y_dev = is_device_ptr(y);
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>(R * E);
    size_t o_y = y_dev ? 0 : io.take<float>(R * E);
    WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    float *yd = y_dev ? y : (float *)(iob + o_y);
    if (!x_dev) WB_CUDA(cudaMemcpyAsync((void *)xd, x, R * E * sizeof(float), cudaMemcpyHostToDevice, st));
    Carve c;
    size_t o_qkv = c.take<float>(R * 3 * E);
    size_t o_o = c.take<float>(R * E);
    WB_TRY(ensure(ctx->ws, c.off));
    float *qkv = (float *)((char *)ctx->ws.p + o_qkv), *o = (float *)((char *)ctx->ws.p + o_o);
    std::string msg;
    WbSeqView none{};
    if (exact) {  // model.rs:144-150 linear: sequential products, then + bias
        wb::OutMap om{wb::OUT_DENSE, qkv, 3LL * E, none, 0, T};
        wb::launch_seqdot(xd, (int)R, E, E, L->wt_qkv, 3 * E, L->b_qkv, 0, om, st);
    } else {
        int rc = wb::tc_gemm_tf32(xd, L->w_qkv, L->b_qkv, qkv, (int)R, 3 * E, E, ctx->dev_err, st, &msg);
        if (rc != WB_OK) return fail(rc, msg);
    }
    int rc = wb::launch_dot_attn(qkv, B, T, E, H, o, st, &msg);
    if (rc != WB_OK) return fail(rc, msg);
    if (exact) {
        wb::OutMap om{wb::OUT_DENSE, yd, E, none, 0, T};
        wb::launch_seqdot(o, (int)R, E, E, L->wt_o, E, L->b_o, 0, om, st);
    } else {
        rc = wb::tc_gemm_tf32(o, L->w_o, L->b_o, yd, (int)R, E, E, ctx->dev_err, st, &msg);
        if (rc != WB_OK) return fail(rc, msg);
    }
    WB_CUDA(cudaGetLastError());
    if (!y_dev) {
        WB_CUDA(cudaMemcpyAsync(y, yd, R * E * sizeof(float), cudaMemcpyDeviceToHost, st));
        WB_CUDA(cudaStreamSynchronize(st));
        uint32_t derr = 0;
        WB_CUDA(cudaMemcpy(&derr, ctx->dev_err, sizeof(derr), cudaMemcpyDeviceToHost));
        if (derr) return fail(WB_ETIMEOUT, "device-side check failed, error word " + std::to_string(derr));
    }
    return WB_OK;
}

// ---------------------------------------------------------------------------
// KV cache
// ---------------------------------------------------------------------------
int wb_kv_cache_create(wb_context *ctx, int n_layers, int n_head, int head_dim, int max_seqs, int max_ctx,
                       wb_kv_cache **out) {
    if (!ctx || !out) return fail(WB_EINVAL, "NULL argument");
    *out = nullptr;
    if (n_layers <= 0 || n_head <= 0 || head_dim <= 0 || head_dim > 256 || max_seqs <= 0 || max_ctx <= 0)
        return fail(WB_EINVAL, "bad cache dimensions");
    DeviceGuard g(ctx->device);
    wb_kv_cache *c = new wb_kv_cache();
    c->ctx = ctx;
    c->device = ctx->device;
    c->L = n_layers; c->H = n_head; c->hd = head_dim; c->S = max_seqs; c->cap = max_ctx;
    const size_t n = (size_t)n_layers * max_seqs * n_head * max_ctx;
    if (cudaMalloc(&c->theta, n * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&c->bucket, n) != cudaSuccess ||
        cudaMalloc(&c->v, n * head_dim * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&c->len, (size_t)n_layers * max_seqs * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        wb_kv_cache_destroy(c);
        return fail(WB_ENOMEM, "KV cache allocation failed (" + std::to_string(n * (5 + 4 * head_dim)) + " bytes)");
    }
    {
        std::string msg;
        const size_t nb = wb::decode_scratch_bytes(max_seqs, n_head, head_dim, n_head * head_dim, max_ctx);
        if (wb::ws_ensure(&c->dscratch, nb, &msg) != 0) {
            wb_kv_cache_destroy(c);
            return fail(WB_ENOMEM, msg);
        }
        if (cudaMemset(c->dscratch.p, 0, c->dscratch.n) != cudaSuccess) {
            cudaGetLastError();
            wb_kv_cache_destroy(c);
            return fail(WB_ECUDA, "cudaMemset failed");
        }
    }
    if (cudaMemset(c->len, 0, (size_t)n_layers * max_seqs * sizeof(int32_t)) != cudaSuccess) {
        cudaGetLastError();
        wb_kv_cache_destroy(c);
        return fail(WB_ECUDA, "cudaMemset failed");
    }
    c->len_host.assign((size_t)n_layers * max_seqs, 0);
    *out = c;
    return WB_OK;
}

int wb_kv_cache_destroy(wb_kv_cache *c) {
    if (!c) return WB_OK;
    DeviceGuard g(c->device);  // cudaFree below waits for work using the buffers
    if (c->theta) cudaFree(c->theta);
    if (c->bucket) cudaFree(c->bucket);
    if (c->v) cudaFree(c->v);
    if (c->len) cudaFree(c->len);
    if (c->dscratch.p) cudaFree(c->dscratch.p);
    delete c;
    return WB_OK;
}

int wb_kv_cache_length(wb_kv_cache *c, int layer, int seq, int *len_out) {
    if (!c || !len_out) return fail(WB_EINVAL, "NULL argument");
    if (layer < 0 || layer >= c->L || seq < 0 || seq >= c->S) return fail(WB_EINVAL, "layer/seq out of range");
    DeviceGuard g(c->device);
    if (c->refresh(c->ctx->stream) != WB_OK) return fail(WB_ECUDA, "reading cache lengths failed");
    *len_out = c->len_host[(size_t)layer * c->S + seq];
    return WB_OK;
}

int wb_kv_cache_reset_seq(wb_kv_cache *c, int seq) {
    if (!c) return fail(WB_EINVAL, "NULL argument");
    if (seq < -1 || seq >= c->S) return fail(WB_EINVAL, "seq out of range");
    DeviceGuard g(c->device);
    if (seq == -1) {  // every slot of every layer
        WB_CUDA(cudaMemsetAsync(c->len, 0, c->len_host.size() * sizeof(int32_t), c->ctx->stream));
        std::fill(c->len_host.begin(), c->len_host.end(), 0);
        c->len_stale = false;
        return WB_OK;
    }
    if (c->refresh(c->ctx->stream) != WB_OK) return fail(WB_ECUDA, "reading cache lengths failed");
    for (int l = 0; l < c->L; l++) {
        c->len_host[(size_t)l * c->S + seq] = 0;
        WB_CUDA(cudaMemsetAsync(c->len + (size_t)l * c->S + seq, 0, sizeof(int32_t), c->ctx->stream));
    }
    return WB_OK;
}

int wb_kv_cache_load(wb_context *ctx, wb_kv_cache *c, int layer, int seq, int n, const float *phases,
                     const float *values) {
    if (!ctx || !c || !phases || !values) return fail(WB_EINVAL, "NULL argument");
    if (c->ctx != ctx) return fail(WB_EINVAL, "cache belongs to another context");
    if (layer < 0 || layer >= c->L || seq < 0 || seq >= c->S) return fail(WB_EINVAL, "layer/seq out of range");
    if (n < 0 || n > c->cap) return fail(WB_EINVAL, "n exceeds cache capacity");
    DeviceGuard g(ctx->device);
    cudaStream_t st = ctx->stream;
    if (c->refresh(st) != WB_OK) return fail(WB_ECUDA, "reading cache lengths failed");
    WbSeqView sv = c->view(layer, nullptr);
    const bool dev = is_device_ptr(phases);
    const cudaMemcpyKind kind = dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    for (int h = 0; h < c->H; h++) {
        const long long base = (long long)seq * sv.seq_stride + (long long)h * c->cap;
        if (n) {
            WB_CUDA(cudaMemcpyAsync(sv.theta + base, phases + (size_t)h * n, n * sizeof(float), kind, st));
            WB_CUDA(cudaMemcpyAsync(sv.v + base * c->hd, values + (size_t)h * n * c->hd,
                                    (size_t)n * c->hd * sizeof(float),
                                    is_device_ptr(values) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
            wb::launch_bucket_from_theta(sv.theta + base, sv.bucket + base, n, st);
        }
    }
    const int32_t nn = n;
    WB_CUDA(cudaMemcpyAsync(c->len + (size_t)layer * c->S + seq, &nn, sizeof(int32_t), cudaMemcpyHostToDevice, st));
    WB_CUDA(cudaStreamSynchronize(st));
    c->len_host[(size_t)layer * c->S + seq] = n;
    return WB_OK;
}

int wb_kv_cache_read(wb_context *ctx, wb_kv_cache *c, int layer, int seq, float *phases, uint8_t *buckets,
                     float *values) {
    if (!ctx || !c) return fail(WB_EINVAL, "NULL argument");
    if (layer < 0 || layer >= c->L || seq < 0 || seq >= c->S) return fail(WB_EINVAL, "layer/seq out of range");
    DeviceGuard g(ctx->device);
    cudaStream_t st = ctx->stream;
    WB_CUDA(cudaStreamSynchronize(st));
    if (c->refresh(st) != WB_OK) return fail(WB_ECUDA, "reading cache lengths failed");
    const int n = c->len_host[(size_t)layer * c->S + seq];
    WbSeqView sv = c->view(layer, nullptr);
    for (int h = 0; h < c->H && n > 0; h++) {
        const long long base = (long long)seq * sv.seq_stride + (long long)h * c->cap;
        if (phases) WB_CUDA(cudaMemcpy(phases + (size_t)h * n, sv.theta + base, n * sizeof(float), cudaMemcpyDefault));
        if (buckets) WB_CUDA(cudaMemcpy(buckets + (size_t)h * n, sv.bucket + base, n, cudaMemcpyDefault));
        if (values)
            WB_CUDA(cudaMemcpy(values + (size_t)h * n * c->hd, sv.v + base * c->hd, (size_t)n * c->hd * sizeof(float),
                               cudaMemcpyDefault));
    }
    return WB_OK;
}

// Sequence ids: host arrays are validated against the host length mirror
// and copied to the context's staging buffer; device arrays are used as
// they are (no host synchronisation, so the call can be captured in a CUDA
// graph) and the kernels check slots and capacity on the device.
struct SeqIds {
    const int32_t *dev = nullptr;
    std::vector<int32_t> host;
    bool on_device = false;
};

static int check_host_ids(wb_kv_cache *c, int layer_idx, const int32_t *ids, int n_seq, bool prefill, int T) {
    if (c->refresh(c->ctx->stream) != WB_OK) return fail(WB_ECUDA, "reading cache lengths failed");
    for (int i = 0; i < n_seq; i++) {
        if (ids[i] < 0 || ids[i] >= c->S) return fail(WB_EINVAL, "seq id out of range");
        const int len = c->len_host[(size_t)layer_idx * c->S + ids[i]];
        if (prefill && len != 0)
            return fail(WB_EINVAL, "prefill needs an empty slot (kv_cache.rs prefill starts from KvCache::new)");
        if (prefill && T > c->cap) return fail(WB_EINVAL, "seq_len exceeds cache capacity");
        if (!prefill && len >= c->cap) return fail(WB_EINVAL, "cache slot is full");
        for (int j = 0; j < i; j++)
            if (ids[j] == ids[i]) return fail(WB_EINVAL, "duplicate seq id");
    }
    return WB_OK;
}

static int common_kv_checks(wb_context *ctx, wb_kv_cache *c, int layer_idx, const wb_attn_layer *L,
                            const int32_t *seq_ids, const float *x, const float *y, int flags) {
    if (!ctx || !c || !L || !seq_ids || !x || !y) return fail(WB_EINVAL, "NULL argument");
    if (c->ctx != ctx || L->ctx != ctx) return fail(WB_EINVAL, "objects belong to another context");
    if (flags & ~(WB_PATH_EXACT | WB_NO_CONTENT)) return fail(WB_EINVAL, "unknown flag bits");
    if (layer_idx < 0 || layer_idx >= c->L) return fail(WB_EINVAL, "layer out of range");
    if (L->H != c->H || L->hd != c->hd) return fail(WB_EINVAL, "layer shape does not match cache");
    return WB_OK;
}

int wb_kv_prefill(wb_context *ctx, wb_kv_cache *c, int layer_idx, const wb_attn_layer *L, const int32_t *seq_ids,
                  int n_seq, const float *x, int T, int flags, float *y) {
    WB_TRY(common_kv_checks(ctx, c, layer_idx, L, seq_ids, x, y, flags));
    if (n_seq < 0 || T < 0) return fail(WB_EINVAL, "negative n_seq or seq_len");
    if (n_seq > c->S) return fail(WB_EINVAL, "more sequences than cache slots");
    if (n_seq == 0 || T == 0) return WB_OK;
    if (T > c->cap) return fail(WB_EINVAL, "seq_len exceeds cache capacity");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    const bool ids_dev = is_device_ptr(seq_ids);
    if (!ids_dev) WB_TRY(check_host_ids(c, layer_idx, seq_ids, n_seq, true, T));
    const long long R = (long long)n_seq * T;
    const int E = L->E, H = L->H, hd = L->hd;
    const bool x_dev = is_device_ptr(x), y_dev = is_device_ptr(y);
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>(R * E);
    size_t o_y = y_dev ? 0 : io.take<float>(R * E);
    size_t o_ids = ids_dev ? 0 : io.take<int32_t>(n_seq);
    if (io.off) WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    float *yd = y_dev ? y : (float *)(iob + o_y);
    const int32_t *ids_d = ids_dev ? seq_ids : (const int32_t *)(iob + o_ids);
    if (!ids_dev)
        WB_CUDA(cudaMemcpyAsync((void *)ids_d, seq_ids, n_seq * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    if (!x_dev) WB_CUDA(cudaMemcpyAsync((void *)xd, x, R * E * sizeof(float), cudaMemcpyHostToDevice, st));
    WbSeqView sv = c->view(layer_idx, ids_d);
    if (flags & WB_PATH_EXACT) {
        Carve cv;
        size_t o_rs = cv.take<float>(R * 2 * H);
        size_t o_o = cv.take<float>(R * E);
        WB_TRY(ensure(ctx->ws, cv.off));
        char *w = (char *)ctx->ws.p;
        float *o = (float *)(w + o_o);
        WB_TRY(run_projections_exact(ctx, L, xd, n_seq, T, sv, (float *)(w + o_rs), nullptr, false));
        wb::launch_attn_simt(sv, nullptr, 0, 0.0f, L->harmonic_n, n_seq, H, T, hd, o, nullptr, st);
        wb::OutMap om{wb::OUT_DENSE, yd, E, sv, 0, T};
        wb::launch_seqdot(o, (int)R, E, E, L->wo_t, E, L->bo, 0, om, st);
        WB_CUDA(cudaGetLastError());
    } else {
        std::string msg;
        int rc = wb::tc_kv_prefill(L->tc, sv, xd, n_seq, T, yd, &ctx->ws, ctx->dev_err, ctx->sm_count, st, &msg);
        if (rc != WB_OK) return fail(rc, msg);
    }
    wb::launch_len_update(c->len + (size_t)layer_idx * c->S, ids_d, n_seq, T, 1, c->S, c->cap, st);
    WB_CUDA(cudaGetLastError());
    if (ids_dev) c->len_stale = true;
    else
        for (int i = 0; i < n_seq; i++) c->len_host[(size_t)layer_idx * c->S + seq_ids[i]] = T;
    if (!y_dev) {
        WB_CUDA(cudaMemcpyAsync(y, yd, R * E * sizeof(float), cudaMemcpyDeviceToHost, st));
        WB_CUDA(cudaStreamSynchronize(st));
    }
    return WB_OK;
}

int wb_kv_decode(wb_context *ctx, wb_kv_cache *c, int layer_idx, const wb_attn_layer *L, const int32_t *seq_ids,
                 int n_seq, const float *x, int flags, float *y) {
    WB_TRY(common_kv_checks(ctx, c, layer_idx, L, seq_ids, x, y, flags));
    if (n_seq < 0) return fail(WB_EINVAL, "negative n_seq");
    if (n_seq > c->S) return fail(WB_EINVAL, "more sequences than cache slots");
    if (n_seq == 0) return WB_OK;
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    const bool ids_dev = is_device_ptr(seq_ids);
    if (!ids_dev) WB_TRY(check_host_ids(c, layer_idx, seq_ids, n_seq, false, 0));
    const int E = L->E, H = L->H, hd = L->hd;
    const bool x_dev = is_device_ptr(x), y_dev = is_device_ptr(y);
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>((size_t)n_seq * E);
    size_t o_y = y_dev ? 0 : io.take<float>((size_t)n_seq * E);
    size_t o_ids = ids_dev ? 0 : io.take<int32_t>(n_seq);
    if (io.off) WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    float *yd = y_dev ? y : (float *)(iob + o_y);
    const int32_t *ids_d = ids_dev ? seq_ids : (const int32_t *)(iob + o_ids);
    if (!ids_dev)
        WB_CUDA(cudaMemcpyAsync((void *)ids_d, seq_ids, n_seq * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    if (!x_dev) WB_CUDA(cudaMemcpyAsync((void *)xd, x, (size_t)n_seq * E * sizeof(float), cudaMemcpyHostToDevice, st));
    WbSeqView sv = c->view(layer_idx, ids_d);
    int32_t *len_l = c->len + (size_t)layer_idx * c->S;
    if (flags & WB_PATH_EXACT) {
        Carve cv;
        size_t o_rs = cv.take<float>((size_t)n_seq * 2 * H);
        size_t o_th = cv.take<float>((size_t)n_seq * H);
        size_t o_vn = cv.take<float>((size_t)n_seq * H * hd);
        size_t o_o = cv.take<float>((size_t)n_seq * E);
        WB_TRY(ensure(ctx->ws, cv.off));
        char *w = (char *)ctx->ws.p;
        float *rs = (float *)(w + o_rs), *th = (float *)(w + o_th), *vn = (float *)(w + o_vn), *o = (float *)(w + o_o);
        wb::OutMap rm{wb::OUT_DENSE, rs, 2LL * H, sv, 0, 1};
        wb::launch_seqdot(xd, n_seq, E, E, L->wrs_t, 2 * H, L->brs, 1, rm, st);
        wb::launch_theta_only(rs, n_seq * H, th, st);
        for (int h = 0; h < H; h++) {
            wb::OutMap vm{wb::OUT_DENSE, vn + (size_t)h * hd, (long long)H * hd, sv, 0, 1};
            wb::launch_seqdot(xd + (size_t)h * hd, n_seq, hd, E, L->wv_t + (size_t)h * hd * hd, hd,
                              L->bv + (size_t)h * hd, 0, vm, st);
        }
        wb::launch_decode_simt(sv, len_l, th, vn, L->harmonic_n, n_seq, H, hd, o, st);
        wb::OutMap om{wb::OUT_DENSE, yd, E, sv, 0, 1};
        wb::launch_seqdot(o, n_seq, E, E, L->wo_t, E, L->bo, 0, om, st);
        wb::launch_len_update(len_l, ids_d, n_seq, 1, 0, c->S, c->cap, st);
        c->note_decode(layer_idx, st, false);
        WB_CUDA(cudaGetLastError());
    } else {
        std::string msg;
        bool ends_with_out = false;
        int rc = wb::tc_kv_decode(L->tc, sv, len_l, c->cap, c->S, xd, n_seq, yd, c->dscratch.p, c->dscratch.n,
                                  ctx->dev_err, ctx->sm_count, st, &msg, c->chain_ok(layer_idx, st),
                                  &ends_with_out);
        c->note_decode(layer_idx, st, ends_with_out);
        if (rc != WB_OK) return fail(rc, msg);
    }
    if (ids_dev) c->len_stale = true;
    else
        for (int i = 0; i < n_seq; i++) c->len_host[(size_t)layer_idx * c->S + seq_ids[i]] += 1;
    if (!y_dev) {
        WB_CUDA(cudaMemcpyAsync(y, yd, (size_t)n_seq * E * sizeof(float), cudaMemcpyDeviceToHost, st));
        WB_CUDA(cudaStreamSynchronize(st));
    }
    return WB_OK;
}

int wb_test_gemm_bf16(wb_context *ctx, const uint16_t *A, const uint16_t *B, const float *bias, float *C, int M,
                      int N, int K) {
    if (!ctx || !A || !B || !bias || !C) return fail(WB_EINVAL, "NULL argument");
    DeviceGuard g(ctx->device);
    std::string msg;
    int rc = wb::tc_gemm_bf16((const __nv_bfloat16 *)A, (const __nv_bfloat16 *)B, bias, C, M, N, K, ctx->dev_err,
                              ctx->stream, &msg);
    return rc == WB_OK ? rc : fail(rc, msg);
}

int wb_test_gemm_tf32(wb_context *ctx, const float *A, const float *B, const float *bias, float *C, int M, int N,
                      int K) {
    if (!ctx || !A || !B || !bias || !C) return fail(WB_EINVAL, "NULL argument");
    DeviceGuard g(ctx->device);
    std::string msg;
    int rc = wb::tc_gemm_tf32(A, B, bias, C, M, N, K, ctx->dev_err, ctx->stream, &msg);
    return rc == WB_OK ? rc : fail(rc, msg);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// wb_kv_decode_noalloc: the tensor-path decode step with its scratch in a
// file-scope device array instead of memory the library allocates.
//
// Who needs it: callers that may not allocate device memory at the point
// where they decode -- a serving process that reserves its whole device
// budget at start-up and forbids allocation on the request path, a host
// application whose own memory pool owns the device, or a latency-bound
// loop that cannot take cudaMalloc's implicit synchronisation.  Everything else the call touches (weights, cache, x, y, seq
// ids) was allocated by the caller beforehand.
//
// The array below is WB_NOALLOC_SCRATCH_BYTES on every GPU that loads this
// library, held until the process exits.  Host code cannot use the name
// g_wb_noalloc_scratch as a device address (on the host it is only a
// stand-in symbol), so the first call on each device looks up the array's
// device address with cudaGetSymbolAddress, with that device current, and
// keeps it; make that first call before any stream capture.  Every call
// shares the one array and it keeps the last call's contents: the ticket
// counters the kernels rely on are cleared at the start of each call, and
// calls that overlap on the GPU (two streams, two contexts on the same
// device) race on the array and must not be issued.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_wb_noalloc_scratch[WB_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_addr[kMaxDevices] = {};

// Device address of the array on `device` (which must be current).
int noalloc_scratch_address(int device, void **out) {
    if (device < 0 || device >= kMaxDevices) return fail(WB_EINVAL, "device ordinal out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[device]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_wb_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return fail(WB_ECUDA, std::string("cudaGetSymbolAddress of the static decode scratch failed: ") +
                                      cudaGetErrorString(e));
        g_noalloc_addr[device] = p;
    }
    *out = g_noalloc_addr[device];
    return WB_OK;
}
}  // namespace

extern "C" int wb_kv_decode_noalloc(wb_context *ctx, wb_kv_cache *c, int layer_idx, const wb_attn_layer *L,
                                    const int32_t *seq_ids, int n_seq, const float *x, float *y) {
    if (!ctx || !c || !L || !seq_ids || !x || !y) return fail(WB_EINVAL, "NULL argument");
    if (c->ctx != ctx || L->ctx != ctx) return fail(WB_EINVAL, "objects belong to another context");
    if (layer_idx < 0 || layer_idx >= c->L) return fail(WB_EINVAL, "layer out of range");
    if (L->H != c->H || L->hd != c->hd) return fail(WB_EINVAL, "layer shape does not match cache");
    if (n_seq < 0 || n_seq > c->S) return fail(WB_EINVAL, "n_seq out of range for the cache");
    if (n_seq == 0) return WB_OK;
    if (!is_device_ptr(seq_ids) || !is_device_ptr(x) || !is_device_ptr(y))
        return fail(WB_EINVAL, "wb_kv_decode_noalloc needs device pointers for seq_ids, x and y (no staging)");
    const size_t need = wb::decode_scratch_bytes(c->S, c->H, c->hd, c->H * c->hd, c->cap);
    if (need > WB_NOALLOC_SCRATCH_BYTES)
        return fail(WB_EINVAL, "decode scratch for this cache needs " + std::to_string(need) +
                                   " bytes, above the static limit of " +
                                   std::to_string((size_t)WB_NOALLOC_SCRATCH_BYTES) +
                                   " (fewer slots or a smaller capacity fit; wb_kv_decode has no limit)");
    DeviceGuard g(ctx->device);
    if (!g.ok) return fail(WB_ECUDA, "cudaSetDevice failed");
    void *scratch = nullptr;
    WB_TRY(noalloc_scratch_address(ctx->device, &scratch));
    cudaStream_t st = ctx->stream;
    size_t t_off = 0, t_bytes = 0;
    wb::decode_scratch_tickets(c->S, c->H, c->hd, c->H * c->hd, c->cap, &t_off, &t_bytes);
    WB_CUDA(cudaMemsetAsync((char *)scratch + t_off, 0, t_bytes, st));
    WbSeqView sv = c->view(layer_idx, seq_ids);
    std::string msg;
    bool ends_with_out = false;
    int rc = wb::tc_kv_decode(L->tc, sv, c->len + (size_t)layer_idx * c->S, c->cap, c->S, x, n_seq, y, scratch,
                              WB_NOALLOC_SCRATCH_BYTES, ctx->dev_err, ctx->sm_count, st, &msg, false,
                              &ends_with_out);
    c->note_decode(layer_idx, st, ends_with_out);
    if (rc != WB_OK) return fail(rc, msg);
    c->len_stale = true;
    return WB_OK;
}
