// wb_api.cu -- C ABI entry points (include/wave_b200.h): argument checks,
// device-resident weights, workspace management and kernel sequencing.
#include "wave_b200.h"
#include "wave_b200_testing.h"
#include "wb_internal.h"
#include "wb_tc.h"
#include "wb_bwd.h"
#include "wb_decode.h"
#include "wb_serve.h"

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

// Where a caller's buffer lives.  Device (and managed) memory is used in
// place.  Pinned host memory (cudaHostAlloc, cudaHostRegister) is read and
// written by the copy engines without staging, and kernels may store to it
// through its device alias.  Pageable memory goes through the driver's
// staging copies.
struct MemInfo {
    bool device = false;
    void *alias = nullptr;  // device address of pinned host memory, else nullptr
};

MemInfo mem_info(const void *p) {
    MemInfo m;
    if (!p) return m;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return m;
    }
    m.device = a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
    if (a.type == cudaMemoryTypeHost) m.alias = a.devicePointer;
    return m;
}

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
    // host-buffer pipelines: copies up, copies down, and their events
    cudaStream_t cp_in = nullptr, cp_out = nullptr;
    std::vector<cudaEvent_t> ev;
};

// Creates ctx's copy streams and at least n events on first need.
static int copy_streams(wb_context *ctx, size_t n) {
    if (!ctx->cp_in && cudaStreamCreateWithFlags(&ctx->cp_in, cudaStreamNonBlocking) != cudaSuccess)
        return fail(WB_ECUDA, "copy stream creation failed");
    if (!ctx->cp_out && cudaStreamCreateWithFlags(&ctx->cp_out, cudaStreamNonBlocking) != cudaSuccess)
        return fail(WB_ECUDA, "copy stream creation failed");
    while (ctx->ev.size() < n) {
        cudaEvent_t e;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
            return fail(WB_ECUDA, "event creation failed");
        ctx->ev.push_back(e);
    }
    return WB_OK;
}

// One call over n_seq independent sequences whose input rows x and output
// rows y (seq_elems floats per sequence each) may be host memory: the
// sequences run in chunks, chunk i's rows going up on ctx->cp_in while
// chunk i-1 computes on the call's stream (fn(first_seq, n_seqs)) and
// chunk i-2's outputs come down on ctx->cp_out.  x_host / y_host are nullptr
// where the caller's buffer is device memory (xd / yd are then that buffer);
// otherwise xd / yd are device staging rows of the whole call.  On return
// the call's stream is ordered after every copy (the caller synchronises it
// when y is host memory).  Chunks hold >= 2 MB of rows and number <= 16.
template <class F>
static int run_chunked(wb_context *ctx, int n_seq, size_t seq_elems, const float *x_host, const float *xd,
                       float *y_host, float *yd, F &&fn) {
    cudaStream_t st = ctx->stream;
    const size_t seq_b = seq_elems * sizeof(float);
    const size_t min_seqs = (((size_t)2 << 20) + seq_b - 1) / seq_b;
    const int g = (int)std::min<size_t>((size_t)n_seq, std::max<size_t>((n_seq + 15) / 16, min_seqs));
    const int nch = (n_seq + g - 1) / g;
    WB_TRY(copy_streams(ctx, 2 * (size_t)nch + 2));
    cudaEvent_t *ev = ctx->ev.data();  // [0] start, [1] copies down done, [2 + i] up, [2 + nch + i] computed
    WB_CUDA(cudaEventRecord(ev[0], st));
    WB_CUDA(cudaStreamWaitEvent(ctx->cp_in, ev[0], 0));
    WB_CUDA(cudaStreamWaitEvent(ctx->cp_out, ev[0], 0));
    auto rows = [&](int i, size_t *off, size_t *bytes) {
        const size_t s0 = (size_t)i * g;
        *off = s0 * seq_elems;
        *bytes = std::min<size_t>(g, n_seq - s0) * seq_b;
    };
    auto up = [&](int i) -> int {
        size_t off, bytes;
        rows(i, &off, &bytes);
        if (x_host)
            WB_CUDA(cudaMemcpyAsync((void *)(xd + off), x_host + off, bytes, cudaMemcpyHostToDevice, ctx->cp_in));
        WB_CUDA(cudaEventRecord(ev[2 + i], ctx->cp_in));
        return WB_OK;
    };
    auto down = [&](int i) -> int {
        if (!y_host) return WB_OK;
        size_t off, bytes;
        rows(i, &off, &bytes);
        WB_CUDA(cudaStreamWaitEvent(ctx->cp_out, ev[2 + nch + i], 0));
        WB_CUDA(cudaMemcpyAsync(y_host + off, yd + off, bytes, cudaMemcpyDeviceToHost, ctx->cp_out));
        return WB_OK;
    };
    int rc = up(0);
    for (int i = 0; i < nch && rc == WB_OK; i++) {
        rc = cudaStreamWaitEvent(st, ev[2 + i], 0) == cudaSuccess ? WB_OK : fail(WB_ECUDA, "stream wait failed");
        if (rc == WB_OK) rc = fn(i * g, std::min(g, n_seq - i * g));
        if (rc == WB_OK && cudaEventRecord(ev[2 + nch + i], st) != cudaSuccess)
            rc = fail(WB_ECUDA, "event record failed");
        if (rc == WB_OK && i + 1 < nch) rc = up(i + 1);
        if (rc == WB_OK && i > 0) rc = down(i - 1);
    }
    if (rc == WB_OK) rc = down(nch - 1);
    if (rc != WB_OK) {  // nothing the caller frees may still be in flight
        cudaStreamSynchronize(ctx->cp_in);
        cudaStreamSynchronize(ctx->cp_out);
        cudaStreamSynchronize(st);
        return rc;
    }
    WB_CUDA(cudaEventRecord(ev[1], ctx->cp_out));
    WB_CUDA(cudaStreamWaitEvent(st, ev[1], 0));
    return WB_OK;
}

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
    float *harmonic_raw = nullptr; // [H] (backward: d softplus = sigmoid(raw))
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

struct wb_ffn_layer {
    wb_context *ctx = nullptr;
    int device = 0;  // destroy must not touch ctx
    int E = 0, M = 0, nb = 0, steps = 0, corr = 0, groups = 1;
    float alpha = 0.0f, beta = 0.0f;
    // squeeze [M][E]; process_1 stored transposed, [M][E]
    float *mi_sq_w = nullptr, *mi_sq_b = nullptr, *mi_pr_w = nullptr, *mi_pr_b = nullptr;
    float *mo_sq_w = nullptr, *mo_sq_b = nullptr, *mo_pr_w = nullptr, *mo_pr_b = nullptr;
    float *gamma_raw = nullptr, *omega = nullptr, *phase_corr = nullptr, *rk4w = nullptr;
    float *out_w = nullptr, *out_b = nullptr;
    __nv_bfloat16 *out_hi = nullptr, *out_lo = nullptr;  // dense out_w as a bf16 split (tensor path)
};

struct wb_agc {
    wb_context *ctx = nullptr;
    int device = 0;
    wb::AgcDev *dev = nullptr;
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
    // The device copy of the last host seq-id list a decode used and the
    // stream it was uploaded on: a decode with the same list on the same
    // stream reuses it instead of uploading the ids again.
    int32_t *ids_mirror = nullptr;
    std::vector<int32_t> ids_last;
    cudaStream_t ids_stream = nullptr;
    // Paged caches: each layer holds n_pages pages of WB_PAGE positions (all
    // heads); a slot's positions 128p .. 128p+127 live in page
    // pages[slot][p] (device table + host mirror, -1 unmapped), reserved by
    // wb_kv_seq_reserve as a prefix p < reserved[slot] from a free list.
    bool paged = false;
    int n_pages = 0, max_pages = 0;
    int32_t *pages = nullptr;
    std::vector<int32_t> pages_host;
    std::vector<int> reserved;
    std::vector<int32_t> free_pages;
    int seq_cap(int seq) const { return paged ? reserved[seq] * WB_PAGE : cap; }
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
        const long long per_layer = paged ? (long long)n_pages * H * WB_PAGE : (long long)S * H * cap;
        WbSeqView s;
        s.theta = theta + layer * per_layer;
        s.bucket = bucket + layer * per_layer;
        s.v = v + layer * per_layer * hd;
        s.seq_stride = paged ? (long long)H * WB_PAGE : (long long)H * cap;
        s.cap = paged ? WB_PAGE : cap;
        s.slot = slots;
        s.pages = paged ? pages : nullptr;
        s.max_pages = max_pages;
        return s;
    }
    // the host index of (seq, head h, position t) of a layer view: see
    // WbSeqView (the caller keeps t below seq_cap(seq))
    long long host_pos(int seq, int h, int t) const {
        if (!paged) return (long long)seq * H * cap + (long long)h * cap + t;
        const int pg = pages_host[(size_t)seq * max_pages + (t >> WB_PAGE_SHIFT)];
        return (long long)pg * H * WB_PAGE + (long long)h * WB_PAGE + (t & (WB_PAGE - 1));
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
    if (ctx->cp_in) {
        cudaStreamSynchronize(ctx->cp_in);
        cudaStreamDestroy(ctx->cp_in);
    }
    if (ctx->cp_out) {
        cudaStreamSynchronize(ctx->cp_out);
        cudaStreamDestroy(ctx->cp_out);
    }
    for (cudaEvent_t e : ctx->ev) cudaEventDestroy(e);
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
    if (rc == WB_OK) rc = upload(&L->harmonic_raw, std::vector<float>(w->harmonic_raw, w->harmonic_raw + H));
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
    float *ptrs[] = {L->harmonic_n, L->harmonic_raw, L->wrs_t, L->wrs_h, L->brs, L->wc_t, L->bc, L->wv_t, L->bv,
                     L->wo_t, L->bo};
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
    const bool chunked = !exact && (!x_dev || !y_dev) && (!phases_out || ph_dev);
    if (!x_dev && !chunked)
        WB_CUDA(cudaMemcpyAsync((void *)xd, x, R * E * sizeof(float), cudaMemcpyHostToDevice, st));

    int rc;
    bool y_down = false;  // y already copied to the host
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
    } else if (chunked) {
        // host rows: sequence chunks, copies overlapped with the compute
        const size_t seq_elems = (size_t)T * E;
        WB_TRY(run_chunked(ctx, B, seq_elems, x_dev ? nullptr : x, xd, y_dev ? nullptr : y, yd, [&](int s0, int n) {
            std::string msg;
            const int r = wb::tc_attn_forward(L->tc, xd + s0 * seq_elems, n, T, use_content, yd + s0 * seq_elems,
                                              phases_out ? phases_out + (size_t)s0 * H * T : nullptr, &ctx->ws,
                                              ctx->dev_err, ctx->sm_count, st, &msg);
            return r == WB_OK ? r : fail(r, msg);
        }));
        y_down = true;
    } else {
        std::string msg;
        float *phd = phases_out ? (ph_dev ? phases_out : (float *)(iob + o_ph)) : nullptr;
        rc = wb::tc_attn_forward(L->tc, xd, B, T, use_content, yd, phd, &ctx->ws, ctx->dev_err,
                                 ctx->sm_count, st, &msg);
        if (rc != WB_OK) return fail(rc, msg);
    }
    if (!y_dev && !y_down) WB_CUDA(cudaMemcpyAsync(y, yd, R * E * sizeof(float), cudaMemcpyDeviceToHost, st));
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
// Forward with the backward's cache (attn.rs:90 with return_pathway_cache =
// true) and the backward (attn.rs:346-430)
// ---------------------------------------------------------------------------

int wb_attn_forward_cache(wb_context *ctx, const wb_attn_layer *L, const float *x, int B, int T, int flags,
                          float *y, const wb_attn_cache_desc *cache) {
    if (!ctx || !L || !x || !y || !cache) return fail(WB_EINVAL, "NULL argument");
    if (L->ctx != ctx) return fail(WB_EINVAL, "layer belongs to another context");
    if (flags & ~WB_NO_CONTENT) return fail(WB_EINVAL, "wb_attn_forward_cache takes WB_NO_CONTENT only");
    if (!cache->phases || !cache->phase_rs || !cache->v_all || !cache->att_w || !cache->out_merged)
        return fail(WB_EINVAL, "missing cache array");
    if (B < 0 || T < 0) return fail(WB_EINVAL, "negative batch or seq_len");
    if (B == 0 || T == 0) return WB_OK;
    const long long R = (long long)B * T;
    if (R > (1LL << 30) || (long long)B * L->H * T * T > (1LL << 34)) return fail(WB_EINVAL, "batch*seq_len too large");
    const int E = L->E, H = L->H, hd = L->hd, C = L->C;
    const bool use_content = C > 0 && !(flags & WB_NO_CONTENT);
    if (use_content && !cache->content) return fail(WB_EINVAL, "the layer has content: cache.content is required");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    // outputs and their sizes
    float *outs[6] = {y, cache->phases, cache->phase_rs, cache->v_all, use_content ? cache->content : nullptr,
                      cache->out_merged};
    const size_t out_n[6] = {(size_t)R * E, (size_t)R * H, (size_t)R * H * 2, (size_t)R * H * hd,
                             (size_t)R * H * (use_content ? C : 0), (size_t)R * E};
    const size_t aw_n = (size_t)B * H * T * T;
    const bool x_dev = is_device_ptr(x), aw_dev = is_device_ptr(cache->att_w);
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>(R * E);
    size_t o_out[6];
    for (int i = 0; i < 6; i++) o_out[i] = (outs[i] && !is_device_ptr(outs[i])) ? io.take<float>(out_n[i]) : 0;
    size_t o_aw = aw_dev ? 0 : io.take<float>(aw_n);
    WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    float *outd[6];
    for (int i = 0; i < 6; i++) outd[i] = !outs[i] ? nullptr : is_device_ptr(outs[i]) ? outs[i] : (float *)(iob + o_out[i]);
    float *awd = aw_dev ? cache->att_w : (float *)(iob + o_aw);
    if (!x_dev) WB_CUDA(cudaMemcpyAsync((void *)xd, x, R * E * sizeof(float), cudaMemcpyHostToDevice, st));
    // the exact forward (WB_PATH_EXACT): its intermediates are the cache
    Carve c;
    size_t o_rs = c.take<float>(R * 2 * H);
    size_t o_ct = c.take<float>(use_content ? R * H * C : 1);
    size_t o_bk = c.take<uint8_t>(R * H);
    WB_TRY(ensure(ctx->ws, c.off));
    char *w = (char *)ctx->ws.p;
    WbSeqView sv;
    sv.theta = outd[1];  // [B][H][T]
    sv.bucket = (uint8_t *)(w + o_bk);
    sv.v = outd[3];      // [B][H][T][hd]
    sv.seq_stride = (long long)H * T;
    sv.cap = T;
    sv.slot = nullptr;
    float *rs = (float *)(w + o_rs), *content = (float *)(w + o_ct);
    WB_TRY(run_projections_exact(ctx, L, xd, B, T, sv, rs, content, use_content));
    wb::launch_attn_simt(sv, use_content ? content : nullptr, use_content ? C : 0,
                         use_content ? 1.0f / std::sqrt((float)C) : 0.0f, L->harmonic_n, B, H, T, hd, outd[5], awd, st);
    wb::OutMap om{wb::OUT_DENSE, outd[0], E, sv, 0, T};
    wb::launch_seqdot(outd[5], (int)R, E, E, L->wo_t, E, L->bo, 0, om, st);
    wb::launch_rows_to_heads(rs, B, T, H, 2, outd[2], st);
    if (use_content) wb::launch_rows_to_heads(content, B, T, H, C, outd[4], st);
    WB_CUDA(cudaGetLastError());
    bool host_out = !aw_dev;
    for (int i = 0; i < 6; i++)
        if (outs[i] && !is_device_ptr(outs[i])) {
            WB_CUDA(cudaMemcpyAsync(outs[i], outd[i], out_n[i] * sizeof(float), cudaMemcpyDeviceToHost, st));
            host_out = true;
        }
    if (!aw_dev) WB_CUDA(cudaMemcpyAsync(cache->att_w, awd, aw_n * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (host_out) WB_CUDA(cudaStreamSynchronize(st));
    return WB_OK;
}

int wb_attn_backward(wb_context *ctx, const wb_attn_layer *L, const float *x, const float *d_y, int B, int T,
                     int flags, const wb_attn_cache_desc *cache, float *d_x, const wb_attn_grads_desc *grads) {
    if (!ctx || !L || !x || !d_y || !cache || !d_x) return fail(WB_EINVAL, "NULL argument");
    if (L->ctx != ctx) return fail(WB_EINVAL, "layer belongs to another context");
    if (flags & ~WB_NO_CONTENT) return fail(WB_EINVAL, "wb_attn_backward takes WB_NO_CONTENT only");
    if (!cache->phases || !cache->phase_rs || !cache->v_all || !cache->att_w || !cache->out_merged)
        return fail(WB_EINVAL, "missing cache array");
    if (B < 0 || T < 0) return fail(WB_EINVAL, "negative batch or seq_len");
    if (B == 0 || T == 0) return WB_OK;
    const long long R = (long long)B * T;
    if (R > (1LL << 30) || (long long)B * L->H * T * T > (1LL << 34)) return fail(WB_EINVAL, "batch*seq_len too large");
    const int E = L->E, H = L->H, hd = L->hd, C = L->C;
    const bool use_content = C > 0 && !(flags & WB_NO_CONTENT);
    if (use_content && !cache->content) return fail(WB_EINVAL, "the layer has content: cache.content is required");
    if (hd > 128) return fail(WB_ENOTSUP, "the backward supports head_dim <= 128");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    // inputs: x, d_y, the cache arrays
    const float *ins[8] = {x, d_y, cache->phases, cache->phase_rs, cache->v_all, use_content ? cache->content : nullptr,
                           cache->att_w, cache->out_merged};
    const size_t in_n[8] = {(size_t)R * E, (size_t)R * E, (size_t)R * H, (size_t)R * H * 2, (size_t)R * H * hd,
                            (size_t)R * H * (use_content ? C : 0), (size_t)B * H * T * T, (size_t)R * E};
    // outputs: d_x and the gradients (any may be NULL)
    wb_attn_grads_desc gz{};
    const wb_attn_grads_desc &gd = grads ? *grads : gz;
    float *outs[10] = {d_x, gd.harmonic_raw, gd.phase_proj_w, gd.phase_proj_b, gd.v_proj_w, gd.v_proj_b,
                       use_content ? gd.content_proj_w : nullptr, use_content ? gd.content_proj_b : nullptr,
                       gd.out_proj_w, gd.out_proj_b};
    const size_t out_n[10] = {(size_t)R * E, (size_t)H, (size_t)H * 2 * E, (size_t)H * 2, (size_t)H * hd * hd,
                              (size_t)H * hd, (size_t)H * C * E, (size_t)H * C, (size_t)E * E, (size_t)E};
    Carve io;
    size_t o_in[8], o_out[10];
    for (int i = 0; i < 8; i++) o_in[i] = (ins[i] && !is_device_ptr(ins[i])) ? io.take<float>(in_n[i]) : 0;
    for (int i = 0; i < 10; i++) o_out[i] = (outs[i] && !is_device_ptr(outs[i])) ? io.take<float>(out_n[i]) : 0;
    const size_t o_scr = io.take<uint8_t>(wb::attn_backward_scratch_bytes(B, H, T, hd, use_content ? C : 0, E));
    WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *ind[8];
    for (int i = 0; i < 8; i++) {
        ind[i] = !ins[i] ? nullptr : is_device_ptr(ins[i]) ? ins[i] : (const float *)(iob + o_in[i]);
        if (ins[i] && !is_device_ptr(ins[i]))
            WB_CUDA(cudaMemcpyAsync((void *)ind[i], ins[i], in_n[i] * sizeof(float), cudaMemcpyHostToDevice, st));
    }
    float *outd[10];
    for (int i = 0; i < 10; i++) outd[i] = !outs[i] ? nullptr : is_device_ptr(outs[i]) ? outs[i] : (float *)(iob + o_out[i]);
    wb::BwdLayer bl{E, H, hd, use_content ? C : 0, L->tc.w_o32, L->harmonic_n, L->harmonic_raw, L->wrs_t, L->wv_t,
                    use_content ? L->wc_t : nullptr};
    wb::BwdCache bc{ind[2], ind[3], ind[4], ind[5], ind[6], ind[7]};
    wb::BwdGrads bg{outd[1], outd[2], outd[3], outd[4], outd[5], outd[6], outd[7], outd[8], outd[9]};
    std::string msg;
    int rc = wb::attn_backward(bl, bc, ind[0], ind[1], B, T, outd[0], bg, iob + o_scr, st, &msg);
    if (rc != WB_OK) return fail(rc, msg);
    bool host_out = false;
    for (int i = 0; i < 10; i++)
        if (outs[i] && !is_device_ptr(outs[i])) {
            WB_CUDA(cudaMemcpyAsync(outs[i], outd[i], out_n[i] * sizeof(float), cudaMemcpyDeviceToHost, st));
            host_out = true;
        }
    if (host_out) WB_CUDA(cudaStreamSynchronize(st));
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
    // the tensor path's core runs on tcgen05 (head_dim <= 128)
    const bool tc_core = !exact && E / H <= 128;
    Carve c;
    size_t o_qkv = c.take<float>(R * 3 * E);
    size_t o_o = c.take<float>(R * E);
    size_t o_core = tc_core ? c.take<char>(wb::tc_dot_core_bytes(B, T, E, H)) : 0;
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
    int rc = tc_core ? wb::tc_dot_attention(qkv, B, T, E, H, o, (char *)ctx->ws.p + o_core, 0, ctx->dev_err,
                                            ctx->sm_count, st, &msg)
                     : wb::launch_dot_attn(qkv, B, T, E, H, o, st, &msg);
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
static int kv_create(wb_context *ctx, int n_layers, int n_head, int head_dim, int max_seqs, int max_ctx, int n_pages,
                     wb_kv_cache **out) {
    if (!ctx || !out) return fail(WB_EINVAL, "NULL argument");
    *out = nullptr;
    if (n_layers <= 0 || n_head <= 0 || head_dim <= 0 || head_dim > 256 || max_seqs <= 0 || max_ctx <= 0 ||
        n_pages < 0)
        return fail(WB_EINVAL, "bad cache dimensions");
    DeviceGuard g(ctx->device);
    wb_kv_cache *c = new wb_kv_cache();
    c->ctx = ctx;
    c->device = ctx->device;
    c->L = n_layers; c->H = n_head; c->hd = head_dim; c->S = max_seqs; c->cap = max_ctx;
    size_t n = (size_t)n_layers * max_seqs * n_head * max_ctx;
    if (n_pages > 0) {
        c->paged = true;
        c->n_pages = n_pages;
        c->max_pages = (max_ctx + WB_PAGE - 1) / WB_PAGE;
        c->cap = c->max_pages * WB_PAGE;  // a slot's capacity: whole pages
        n = (size_t)n_layers * n_pages * n_head * WB_PAGE;
    }
    if (cudaMalloc(&c->theta, n * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&c->bucket, n) != cudaSuccess ||
        cudaMalloc(&c->v, n * head_dim * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&c->len, (size_t)n_layers * max_seqs * sizeof(int32_t)) != cudaSuccess ||
        (c->paged && cudaMalloc(&c->pages, (size_t)max_seqs * c->max_pages * sizeof(int32_t)) != cudaSuccess)) {
        cudaGetLastError();
        wb_kv_cache_destroy(c);
        return fail(WB_ENOMEM, "KV cache allocation failed (" + std::to_string(n * (5 + 4 * head_dim)) + " bytes)");
    }
    {
        std::string msg;
        const size_t nb = wb::decode_scratch_bytes(max_seqs, n_head, head_dim, n_head * head_dim, c->cap);
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
    if (cudaMemset(c->len, 0, (size_t)n_layers * max_seqs * sizeof(int32_t)) != cudaSuccess ||
        (c->paged && cudaMemset(c->pages, 0xFF, (size_t)max_seqs * c->max_pages * sizeof(int32_t)) != cudaSuccess)) {
        cudaGetLastError();
        wb_kv_cache_destroy(c);
        return fail(WB_ECUDA, "cudaMemset failed");
    }
    c->len_host.assign((size_t)n_layers * max_seqs, 0);
    if (c->paged) {
        c->pages_host.assign((size_t)max_seqs * c->max_pages, -1);
        c->reserved.assign(max_seqs, 0);
        for (int p = n_pages - 1; p >= 0; p--) c->free_pages.push_back(p);  // pages 0, 1, ... handed out first
    }
    *out = c;
    return WB_OK;
}

int wb_kv_cache_create(wb_context *ctx, int n_layers, int n_head, int head_dim, int max_seqs, int max_ctx,
                       wb_kv_cache **out) {
    return kv_create(ctx, n_layers, n_head, head_dim, max_seqs, max_ctx, 0, out);
}

int wb_kv_cache_create_paged(wb_context *ctx, int n_layers, int n_head, int head_dim, int max_seqs, int max_ctx,
                             int n_pages, wb_kv_cache **out) {
    if (n_pages <= 0) return fail(WB_EINVAL, "n_pages must be positive");
    return kv_create(ctx, n_layers, n_head, head_dim, max_seqs, max_ctx, n_pages, out);
}

int wb_kv_seq_reserve(wb_kv_cache *c, int seq, int n_positions) {
    if (!c) return fail(WB_EINVAL, "NULL argument");
    if (seq < 0 || seq >= c->S) return fail(WB_EINVAL, "seq out of range");
    if (n_positions < 0 || n_positions > c->cap) return fail(WB_EINVAL, "n_positions exceeds the slot capacity");
    if (!c->paged) return WB_OK;  // contiguous slots hold max_ctx positions already
    const int need = (n_positions + WB_PAGE - 1) / WB_PAGE;
    const int have = c->reserved[seq];
    if (need <= have) return WB_OK;
    if ((size_t)(need - have) > c->free_pages.size())
        return fail(WB_ENOMEM, "out of KV pages (" + std::to_string(c->free_pages.size()) + " free, " +
                                   std::to_string(need - have) + " needed)");
    DeviceGuard g(c->device);
    int32_t *row = c->pages_host.data() + (size_t)seq * c->max_pages;
    for (int p = have; p < need; p++) {
        row[p] = c->free_pages.back();
        c->free_pages.pop_back();
    }
    c->reserved[seq] = need;
    // kernels of earlier calls never read entries >= have (unmapped then),
    // so the update goes in stream order without a wait
    WB_CUDA(cudaMemcpyAsync(c->pages + (size_t)seq * c->max_pages + have, row + have, (need - have) * sizeof(int32_t),
                            cudaMemcpyHostToDevice, c->ctx->stream));
    return WB_OK;
}

int wb_kv_seq_release(wb_kv_cache *c, int seq) {
    if (!c) return fail(WB_EINVAL, "NULL argument");
    if (seq < 0 || seq >= c->S) return fail(WB_EINVAL, "seq out of range");
    WB_TRY(wb_kv_cache_reset_seq(c, seq));
    if (!c->paged || c->reserved[seq] == 0) return WB_OK;
    DeviceGuard g(c->device);
    // calls still in flight may read the slot's pages: the pages return to
    // the free list once the stream has passed them
    WB_CUDA(cudaStreamSynchronize(c->ctx->stream));
    int32_t *row = c->pages_host.data() + (size_t)seq * c->max_pages;
    for (int p = c->reserved[seq] - 1; p >= 0; p--) {
        c->free_pages.push_back(row[p]);
        row[p] = -1;
    }
    c->reserved[seq] = 0;
    WB_CUDA(cudaMemcpy(c->pages + (size_t)seq * c->max_pages, row, c->max_pages * sizeof(int32_t),
                       cudaMemcpyHostToDevice));
    return WB_OK;
}

int wb_kv_cache_free_pages(wb_kv_cache *c, int *n_free) {
    if (!c || !n_free) return fail(WB_EINVAL, "NULL argument");
    *n_free = c->paged ? (int)c->free_pages.size() : 0;
    return WB_OK;
}

int wb_kv_cache_destroy(wb_kv_cache *c) {
    if (!c) return WB_OK;
    DeviceGuard g(c->device);  // cudaFree below waits for work using the buffers
    if (c->theta) cudaFree(c->theta);
    if (c->bucket) cudaFree(c->bucket);
    if (c->v) cudaFree(c->v);
    if (c->len) cudaFree(c->len);
    if (c->ids_mirror) cudaFree(c->ids_mirror);
    if (c->pages) cudaFree(c->pages);
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
    if (n < 0 || n > c->seq_cap(seq)) return fail(WB_EINVAL, "n exceeds the slot's (reserved) capacity");
    DeviceGuard g(ctx->device);
    cudaStream_t st = ctx->stream;
    if (c->refresh(st) != WB_OK) return fail(WB_ECUDA, "reading cache lengths failed");
    WbSeqView sv = c->view(layer, nullptr);
    const cudaMemcpyKind kind = is_device_ptr(phases) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    const cudaMemcpyKind vkind = is_device_ptr(values) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
    // runs of positions contiguous in the view: the whole row, or one page
    const int run = c->paged ? WB_PAGE : std::max(n, 1);
    for (int h = 0; h < c->H; h++) {
        for (int t0 = 0; t0 < n; t0 += run) {
            const int m = std::min(run, n - t0);
            const long long base = c->host_pos(seq, h, t0);
            WB_CUDA(cudaMemcpyAsync(sv.theta + base, phases + (size_t)h * n + t0, m * sizeof(float), kind, st));
            WB_CUDA(cudaMemcpyAsync(sv.v + base * c->hd, values + ((size_t)h * n + t0) * c->hd,
                                    (size_t)m * c->hd * sizeof(float), vkind, st));
            wb::launch_bucket_from_theta(sv.theta + base, sv.bucket + base, m, st);
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
    const int run = c->paged ? WB_PAGE : std::max(n, 1);
    for (int h = 0; h < c->H && n > 0; h++) {
        for (int t0 = 0; t0 < n; t0 += run) {
            const int m = std::min(run, n - t0);
            const long long base = c->host_pos(seq, h, t0);
            const size_t o = (size_t)h * n + t0;
            if (phases) WB_CUDA(cudaMemcpy(phases + o, sv.theta + base, m * sizeof(float), cudaMemcpyDefault));
            if (buckets) WB_CUDA(cudaMemcpy(buckets + o, sv.bucket + base, m, cudaMemcpyDefault));
            if (values)
                WB_CUDA(cudaMemcpy(values + o * c->hd, sv.v + base * c->hd, (size_t)m * c->hd * sizeof(float),
                                   cudaMemcpyDefault));
        }
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
        if (prefill && T > c->seq_cap(ids[i]))
            return fail(WB_EINVAL, c->paged ? "seq_len exceeds the slot's reserved pages (wb_kv_seq_reserve)"
                                            : "seq_len exceeds cache capacity");
        if (!prefill && len >= c->seq_cap(ids[i]))
            return fail(WB_EINVAL, c->paged ? "the slot's reserved pages are full (wb_kv_seq_reserve)"
                                            : "cache slot is full");
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

// Prefill of sequences whose rows (xd, yd) and slots (ids_d) are on the
// device: the body of wb_kv_prefill for one chunk of its sequences.
static int kv_prefill_rows(wb_context *ctx, wb_kv_cache *c, int layer_idx, const wb_attn_layer *L,
                           const int32_t *ids_d, int n_seq, const float *xd, int T, int flags, float *yd) {
    cudaStream_t st = ctx->stream;
    const long long R = (long long)n_seq * T;
    const int E = L->E, H = L->H, hd = L->hd;
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
        return WB_OK;
    }
    std::string msg;
    int rc = wb::tc_kv_prefill(L->tc, sv, xd, n_seq, T, yd, &ctx->ws, ctx->dev_err, ctx->sm_count, st, &msg);
    return rc == WB_OK ? rc : fail(rc, msg);
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
    const int E = L->E;
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
    if (x_dev && y_dev) {
        WB_TRY(kv_prefill_rows(ctx, c, layer_idx, L, ids_d, n_seq, xd, T, flags, yd));
    } else {
        // host rows: sequence chunks, copies overlapped with the compute
        const size_t seq_elems = (size_t)T * E;
        WB_TRY(run_chunked(ctx, n_seq, seq_elems, x_dev ? nullptr : x, xd, y_dev ? nullptr : y, yd,
                           [&](int s0, int n) {
                               return kv_prefill_rows(ctx, c, layer_idx, L, ids_d + s0, n, xd + s0 * seq_elems,
                                                      T, flags, yd + s0 * seq_elems);
                           }));
    }
    wb::launch_len_update(c->len + (size_t)layer_idx * c->S, ids_d, n_seq, T, 1, c->S, c->cap, st, c->pages,
                          c->max_pages);
    WB_CUDA(cudaGetLastError());
    if (ids_dev) c->len_stale = true;
    else
        for (int i = 0; i < n_seq; i++) c->len_host[(size_t)layer_idx * c->S + seq_ids[i]] = T;
    if (!y_dev) WB_CUDA(cudaStreamSynchronize(st));
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
    const MemInfo xm = mem_info(x), ym = mem_info(y);
    const bool x_dev = xm.device;
    // pinned host y on the tensor path's plain-store out_proj: the kernel
    // writes the caller's rows directly, with no copy back
    const bool y_alias = !ym.device && ym.alias && !(flags & WB_PATH_EXACT) &&
                         n_seq < wb::tc_decode_plain_store_rows();
    const bool y_dev = ym.device || y_alias;
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>((size_t)n_seq * E);
    size_t o_y = y_dev ? 0 : io.take<float>((size_t)n_seq * E);
    if (io.off) WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    float *yd = ym.device ? y : (y_alias ? (float *)ym.alias : (float *)(iob + o_y));
    const int32_t *ids_d = seq_ids;
    if (!ids_dev) {
        const bool same = c->ids_mirror && c->ids_stream == st && c->ids_last.size() == (size_t)n_seq &&
                          std::memcmp(c->ids_last.data(), seq_ids, n_seq * sizeof(int32_t)) == 0;
        if (!same) {
            if (!c->ids_mirror) WB_CUDA(cudaMalloc(&c->ids_mirror, (size_t)c->S * sizeof(int32_t)));
            // decodes on another stream may still read the previous list
            if (c->ids_stream && c->ids_stream != st) WB_CUDA(cudaStreamSynchronize(c->ids_stream));
            WB_CUDA(cudaMemcpyAsync(c->ids_mirror, seq_ids, n_seq * sizeof(int32_t), cudaMemcpyHostToDevice, st));
            c->ids_last.assign(seq_ids, seq_ids + n_seq);
            c->ids_stream = st;
        }
        ids_d = c->ids_mirror;
    }
    if (!x_dev) {
        const size_t nx = (size_t)n_seq * E;
        if (xm.alias && nx % 4 == 0 && reinterpret_cast<uintptr_t>(xm.alias) % 16 == 0) {
            wb::launch_copy_f4((const float *)xm.alias, (float *)xd, (long long)nx, st);  // pinned: read over the bus
            WB_CUDA(cudaGetLastError());
        } else {
            WB_CUDA(cudaMemcpyAsync((void *)xd, x, nx * sizeof(float), cudaMemcpyHostToDevice, st));
        }
    }
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
        wb::launch_decode_simt(sv, len_l, th, vn, L->harmonic_n, n_seq, H, hd, o, ctx->dev_err, st);
        wb::OutMap om{wb::OUT_DENSE, yd, E, sv, 0, 1};
        wb::launch_seqdot(o, n_seq, E, E, L->wo_t, E, L->bo, 0, om, st);
        wb::launch_len_update(len_l, ids_d, n_seq, 1, 0, c->S, c->cap, st, c->pages, c->max_pages);
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
    if (!y_dev) WB_CUDA(cudaMemcpyAsync(y, yd, (size_t)n_seq * E * sizeof(float), cudaMemcpyDeviceToHost, st));
    if (!ym.device) WB_CUDA(cudaStreamSynchronize(st));
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

// ---------------------------------------------------------------------------
// the serve-tier layer around the attention
// ---------------------------------------------------------------------------
static int dev_copy(float **dst, const float *src, size_t n) {
    *dst = nullptr;
    if (!src || n == 0) return WB_OK;
    if (cudaMalloc(dst, n * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        return fail(WB_ENOMEM, "cudaMalloc failed for FFN weights");
    }
    if (cudaMemcpy(*dst, src, n * sizeof(float), cudaMemcpyDefault) != cudaSuccess)
        return fail(WB_ECUDA, "weight upload failed");
    return WB_OK;
}

int wb_ffn_layer_destroy(wb_ffn_layer *f) {
    if (!f) return WB_OK;
    DeviceGuard g(f->device);
    for (float *p : {f->mi_sq_w, f->mi_sq_b, f->mi_pr_w, f->mi_pr_b, f->mo_sq_w, f->mo_sq_b, f->mo_pr_w, f->mo_pr_b,
                     f->gamma_raw, f->omega, f->phase_corr, f->rk4w, f->out_w, f->out_b})
        if (p) cudaFree(p);
    if (f->out_hi) cudaFree(f->out_hi);
    delete f;
    return WB_OK;
}

int wb_ffn_layer_create(wb_context *ctx, const wb_ffn_weights_desc *w, wb_ffn_layer **out) {
    if (!ctx || !w || !out) return fail(WB_EINVAL, "NULL argument");
    *out = nullptr;
    const int E = w->n_embd, M = w->maestro_dim, G = w->out_groups;
    if (E <= 0 || E % 2 || M <= 0 || w->rk4_steps <= 0 || G <= 0 || E % G)
        return fail(WB_EINVAL, "bad FFN dimensions (n_embd even, maestro_dim > 0, rk4_steps > 0, groups divide n_embd)");
    if (E / 2 > 4096) return fail(WB_ENOTSUP, "the ODE kernel supports up to 4096 bands");
    if ((size_t)8 * (E + M) * sizeof(float) > 200 * 1024) return fail(WB_ENOTSUP, "n_embd too large for the maestro kernel");
    if (!w->mi_squeeze_w || !w->mi_squeeze_b || !w->mi_process_w || !w->mi_process_b || !w->mo_squeeze_w ||
        !w->mo_squeeze_b || !w->mo_process_w || !w->mo_process_b || !w->gamma_raw || !w->omega ||
        !w->phase_correction || !w->rk4_weights || !w->out_w || (G == 1 && !w->out_b))
        return fail(WB_EINVAL, "missing FFN weight array");
    DeviceGuard g(ctx->device);
    wb_ffn_layer *f = new wb_ffn_layer();
    f->ctx = ctx;
    f->device = ctx->device;
    f->E = E; f->M = M; f->nb = E / 2; f->steps = w->rk4_steps; f->corr = w->use_corrector != 0; f->groups = G;
    f->alpha = w->alpha; f->beta = w->beta;
    const size_t me = (size_t)M * E, gs = E / G;
    int rc = WB_OK;
    auto up = [&](float **d, const float *src, size_t n) { if (rc == WB_OK) rc = dev_copy(d, src, n); };
    up(&f->mi_sq_w, w->mi_squeeze_w, me); up(&f->mi_sq_b, w->mi_squeeze_b, M);
    // process_1 [E][M] is kept transposed ([M][E]): the maestro kernel's threads read a column each
    std::vector<float> tr((size_t)M * E);
    auto transpose = [&](const float *src) {
        std::vector<float> h((size_t)M * E);
        if (cudaMemcpy(h.data(), src, h.size() * sizeof(float), cudaMemcpyDefault) != cudaSuccess) rc = WB_ECUDA;
        for (int i = 0; i < E; i++)
            for (int m = 0; m < M; m++) tr[(size_t)m * E + i] = h[(size_t)i * M + m];
        return tr.data();
    };
    if (rc == WB_OK) up(&f->mi_pr_w, transpose(w->mi_process_w), me);
    up(&f->mi_pr_b, w->mi_process_b, E);
    up(&f->mo_sq_w, w->mo_squeeze_w, me); up(&f->mo_sq_b, w->mo_squeeze_b, M);
    if (rc == WB_OK) up(&f->mo_pr_w, transpose(w->mo_process_w), me);
    up(&f->mo_pr_b, w->mo_process_b, E);
    up(&f->gamma_raw, w->gamma_raw, E / 2); up(&f->omega, w->omega, E / 2);
    up(&f->phase_corr, w->phase_correction, E / 2); up(&f->rk4w, w->rk4_weights, 4);
    if (G == 1) {
        up(&f->out_w, w->out_w, (size_t)E * E);
        up(&f->out_b, w->out_b, E);
        if (rc == WB_OK && E % 8 == 0) {
            if (cudaMalloc(&f->out_hi, (size_t)2 * E * E * sizeof(__nv_bfloat16)) != cudaSuccess) {
                cudaGetLastError();
                rc = fail(WB_ENOMEM, "cudaMalloc failed for FFN weights");
            } else {
                f->out_lo = f->out_hi + (size_t)E * E;
                if (wb::split_bf16(f->out_w, (long long)E * E, f->out_hi, f->out_lo, 0) != WB_OK ||
                    cudaDeviceSynchronize() != cudaSuccess)
                    rc = fail(WB_ECUDA, "out_proj split failed");
            }
        }
    } else {
        up(&f->out_w, w->out_w, (size_t)G * (gs * gs + gs));
    }
    if (rc != WB_OK) {
        wb_ffn_layer_destroy(f);
        return rc;
    }
    *out = f;
    return WB_OK;
}

int wb_agc_create(wb_context *ctx, float alpha, float beta, wb_agc **out) {
    if (!ctx || !out) return fail(WB_EINVAL, "NULL argument");
    *out = nullptr;
    // agc.rs from_coupling -> with_ceiling
    float ceiling = std::sqrt(1.57079637050628662109f / (alpha + 4.0f * beta));
    ceiling = std::max(ceiling, 0.5f);
    wb::AgcDev h{};
    h.ema_mean = 1.0f;
    h.ema_var = 0.5f;
    h.headroom = 3.0f;
    h.decay = 0.995f;
    h.min_threshold = std::max(ceiling * 0.3f, 0.5f);
    h.max_threshold = ceiling;
    h.threshold = std::max(ceiling * 0.75f, 0.5f);
    h.count = 0;
    DeviceGuard g(ctx->device);
    wb_agc *a = new wb_agc();
    a->ctx = ctx;
    a->device = ctx->device;
    if (cudaMalloc(&a->dev, sizeof(wb::AgcDev)) != cudaSuccess ||
        cudaMemcpy(a->dev, &h, sizeof(h), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaGetLastError();
        if (a->dev) cudaFree(a->dev);
        delete a;
        return fail(WB_ENOMEM, "AGC state allocation failed");
    }
    *out = a;
    return WB_OK;
}

int wb_agc_destroy(wb_agc *a) {
    if (!a) return WB_OK;
    DeviceGuard g(a->device);
    if (a->dev) cudaFree(a->dev);
    delete a;
    return WB_OK;
}

int wb_agc_read(wb_agc *a, float *state) {
    if (!a || !state) return fail(WB_EINVAL, "NULL argument");
    DeviceGuard g(a->device);
    wb::AgcDev h{};
    WB_CUDA(cudaStreamSynchronize(a->ctx->stream));
    WB_CUDA(cudaMemcpy(&h, a->dev, sizeof(h), cudaMemcpyDeviceToHost));
    const float v[8] = {h.ema_mean, h.ema_var, h.headroom, h.decay, h.min_threshold, h.max_threshold, h.threshold,
                        (float)h.count};
    memcpy(state, v, sizeof(v));
    return WB_OK;
}

int wb_ffn_forward(wb_context *ctx, const wb_ffn_layer *f, wb_agc *agc, const float *x, int n_rows, int rows_per_call,
                   int flags, float *y) {
    if (!ctx || !f || !agc || !x || !y) return fail(WB_EINVAL, "NULL argument");
    if (f->ctx != ctx || agc->ctx != ctx) return fail(WB_EINVAL, "objects belong to another context");
    if (flags & ~WB_PATH_EXACT) return fail(WB_EINVAL, "unknown flag bits");
    if (n_rows < 0) return fail(WB_EINVAL, "negative n_rows");
    if (n_rows == 0) return WB_OK;
    if (rows_per_call <= 0 || n_rows % rows_per_call) return fail(WB_EINVAL, "rows_per_call must divide n_rows");
    const int n_seg = n_rows / rows_per_call;
    if (n_seg > 65535) return fail(WB_EINVAL, "more than 65535 calls in one batch");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    const long long R = n_rows;
    const int E = f->E;
    const bool x_dev = is_device_ptr(x), y_dev = is_device_ptr(y);
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>(R * E);
    size_t o_y = y_dev ? 0 : io.take<float>(R * E);
    if (io.off) WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    float *yd = y_dev ? y : (float *)(iob + o_y);
    if (!x_dev) WB_CUDA(cudaMemcpyAsync((void *)xd, x, R * E * sizeof(float), cudaMemcpyHostToDevice, st));
    const bool bf3 = !(flags & WB_PATH_EXACT) && f->out_hi;  // out_proj as a bf16x3 tensor-core product
    Carve cv;
    const size_t o_pre = cv.take<float>(R * E), o_ko = cv.take<float>(R * E), o_reg = cv.take<float>(R * E);
    const size_t o_agc = cv.take<float>(wb::agc_scratch_floats(n_seg, (long long)rows_per_call * f->nb));
    const size_t o_split = bf3 ? cv.take<__nv_bfloat16>(2 * R * E) : 0;
    WB_TRY(ensure(ctx->ws, cv.off));
    char *w = (char *)ctx->ws.p;
    float *pre = (float *)(w + o_pre), *ko = (float *)(w + o_ko), *reg = (float *)(w + o_reg);
    int rc;
    // 1-2. maestro_in and precond = x + maestro_in(x) (ffn.rs:61-66)
    wb::MaestroArgs mi{xd, nullptr, f->mi_sq_w, f->mi_sq_b, f->mi_pr_w, f->mi_pr_b, R, E, f->M, pre};
    if ((rc = wb::launch_maestro(mi, st))) return fail(rc, "maestro_in launch failed");
    // AGC (ffn.rs:69-79), one observation per reference call
    float *thr = nullptr;
    if ((rc = wb::launch_agc_observe(pre, n_seg, (long long)rows_per_call * f->nb, agc->dev, (float *)(w + o_agc),
                                     &thr, st)))
        return fail(rc, "AGC launch failed");
    // 3. the frozen ODE (fft_ode.rs:171-250) and the corrector plate
    int fft_len = 0;
    if (f->nb >= 256) {
        fft_len = 1;
        while (fft_len < f->nb) fft_len <<= 1;
    }
    wb::OdeArgs oa{pre, thr, rows_per_call, f->gamma_raw, f->omega, f->rk4w, f->corr ? f->phase_corr : nullptr,
                   f->alpha, f->beta, f->nb, f->steps, fft_len, ko};
    if ((rc = wb::launch_kerr_ode(oa, R, st))) return fail(rc, "Kerr ODE launch failed");
    // 4-5. maestro_out and regulated = kerr_out + maestro_out(kerr_out)
    wb::MaestroArgs mo{ko, nullptr, f->mo_sq_w, f->mo_sq_b, f->mo_pr_w, f->mo_pr_b, R, E, f->M, reg};
    if ((rc = wb::launch_maestro(mo, st))) return fail(rc, "maestro_out launch failed");
    // 6. out_proj
    if (!bf3) {
        if ((rc = wb::launch_out_proj_exact(reg, R, E, f->groups, f->out_w, f->out_b, yd, st)))
            return fail(rc, "out_proj launch failed");
    } else {
        std::string msg;
        __nv_bfloat16 *a_hi = (__nv_bfloat16 *)(w + o_split), *a_lo = a_hi + R * E;
        if ((rc = wb::split_bf16(reg, R * E, a_hi, a_lo, st))) return fail(rc, "split launch failed");
        if ((rc = wb::tc_gemm_bf16x3(a_hi, a_lo, f->out_hi, f->out_lo, f->out_b, yd, (int)R, E, E, ctx->dev_err, st,
                                     &msg)))
            return fail(rc, msg);
    }
    if (!y_dev) {
        WB_CUDA(cudaMemcpyAsync(y, yd, R * E * sizeof(float), cudaMemcpyDeviceToHost, st));
        WB_CUDA(cudaStreamSynchronize(st));
    }
    return WB_OK;
}

int wb_layer_norm(wb_context *ctx, const float *x, int n_rows, int n, const float *weight, const float *bias,
                  float *y) {
    if (!ctx || !x || !weight || !bias || !y) return fail(WB_EINVAL, "NULL argument");
    if (n_rows < 0 || n <= 0) return fail(WB_EINVAL, "bad shape");
    if (n_rows == 0) return WB_OK;
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    const long long R = n_rows;
    const bool x_dev = is_device_ptr(x), y_dev = is_device_ptr(y), w_dev = is_device_ptr(weight),
               b_dev = is_device_ptr(bias);
    Carve io;
    size_t o_x = x_dev ? 0 : io.take<float>(R * n), o_y = y_dev ? 0 : io.take<float>(R * n);
    size_t o_w = w_dev ? 0 : io.take<float>(n), o_b = b_dev ? 0 : io.take<float>(n);
    if (io.off) WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *xd = x_dev ? x : (const float *)(iob + o_x);
    const float *wd = w_dev ? weight : (const float *)(iob + o_w), *bd = b_dev ? bias : (const float *)(iob + o_b);
    float *yd = y_dev ? y : (float *)(iob + o_y);
    if (!x_dev) WB_CUDA(cudaMemcpyAsync((void *)xd, x, R * n * sizeof(float), cudaMemcpyHostToDevice, st));
    if (!w_dev) WB_CUDA(cudaMemcpyAsync((void *)wd, weight, n * sizeof(float), cudaMemcpyHostToDevice, st));
    if (!b_dev) WB_CUDA(cudaMemcpyAsync((void *)bd, bias, n * sizeof(float), cudaMemcpyHostToDevice, st));
    if (wb::launch_layer_norm(xd, n_rows, n, wd, bd, yd, st)) return fail(WB_ECUDA, "layer_norm launch failed");
    if (!y_dev) {
        WB_CUDA(cudaMemcpyAsync(y, yd, R * n * sizeof(float), cudaMemcpyDeviceToHost, st));
        WB_CUDA(cudaStreamSynchronize(st));
    }
    return WB_OK;
}

int wb_residual_add(wb_context *ctx, float *hidden, const float *a, const float *b, long long n) {
    if (!ctx || !hidden || !a || !b) return fail(WB_EINVAL, "NULL argument");
    if (n < 0) return fail(WB_EINVAL, "negative n");
    if (!is_device_ptr(hidden) || !is_device_ptr(a) || !is_device_ptr(b))
        return fail(WB_EINVAL, "wb_residual_add takes device pointers");
    DeviceGuard g(ctx->device);
    if (wb::launch_residual(hidden, a, b, n, ctx->stream)) return fail(WB_ECUDA, "residual launch failed");
    return WB_OK;
}

int wb_embed(wb_context *ctx, const int32_t *tokens, const int32_t *wpe_index, int n_rows, const float *wte,
             int vocab, const float *wpe, int n_pos, int n_embd, float *hidden) {
    if (!ctx || !tokens || !wpe_index || !wte || !hidden) return fail(WB_EINVAL, "NULL argument");
    if (n_rows < 0 || vocab <= 0 || n_embd <= 0 || n_pos < 0) return fail(WB_EINVAL, "bad shape");
    if (n_rows == 0) return WB_OK;
    if (!is_device_ptr(wte) || (wpe && !is_device_ptr(wpe)))
        return fail(WB_EINVAL, "wte / wpe must be device pointers");
    DeviceGuard g(ctx->device);
    cudaStream_t st = ctx->stream;
    const bool t_dev = is_device_ptr(tokens), i_dev = is_device_ptr(wpe_index), h_dev = is_device_ptr(hidden);
    const long long R = n_rows;
    Carve io;
    size_t o_t = t_dev ? 0 : io.take<int32_t>(R), o_i = i_dev ? 0 : io.take<int32_t>(R);
    size_t o_h = h_dev ? 0 : io.take<float>(R * n_embd);
    if (io.off) WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const int32_t *td = t_dev ? tokens : (const int32_t *)(iob + o_t);
    const int32_t *id = i_dev ? wpe_index : (const int32_t *)(iob + o_i);
    float *hd = h_dev ? hidden : (float *)(iob + o_h);
    if (!t_dev) WB_CUDA(cudaMemcpyAsync((void *)td, tokens, R * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    if (!i_dev) WB_CUDA(cudaMemcpyAsync((void *)id, wpe_index, R * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    if (wb::launch_embed(td, id, n_rows, n_embd, wte, vocab, wpe, wpe ? n_pos : 0, hd, ctx->dev_err, st))
        return fail(WB_ECUDA, "embedding launch failed");
    if (!h_dev) {
        WB_CUDA(cudaMemcpyAsync(hidden, hd, R * n_embd * sizeof(float), cudaMemcpyDeviceToHost, st));
        WB_CUDA(cudaStreamSynchronize(st));
    }
    return WB_OK;
}

// logits of rows of hidden (optionally rotated band by band first) against a
// device vocabulary table [vocab][n_embd]
static int vocab_logits(wb_context *ctx, const float *hidden, int n_rows, int n_embd, const float *corrector,
                        const float *table, int vocab, int flags, float *logits) {
    if (!ctx || !hidden || !table || !logits) return fail(WB_EINVAL, "NULL argument");
    if (flags & ~WB_PATH_EXACT) return fail(WB_EINVAL, "unknown flag bits");
    if (n_rows < 0 || n_embd <= 0 || n_embd % 2 || vocab <= 0) return fail(WB_EINVAL, "bad shape");
    if (n_rows == 0) return WB_OK;
    if (!is_device_ptr(table) || (corrector && !is_device_ptr(corrector)))
        return fail(WB_EINVAL, "the vocabulary table and corrector must be device pointers");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    cudaStream_t st = ctx->stream;
    const long long R = n_rows;
    const bool h_dev = is_device_ptr(hidden), l_dev = is_device_ptr(logits);
    Carve io;
    size_t o_h = h_dev ? 0 : io.take<float>(R * n_embd), o_l = l_dev ? 0 : io.take<float>(R * vocab);
    if (io.off) WB_TRY(ensure(ctx->io, io.off));
    char *iob = (char *)ctx->io.p;
    const float *hd = h_dev ? hidden : (const float *)(iob + o_h);
    float *ld = l_dev ? logits : (float *)(iob + o_l);
    if (!h_dev) WB_CUDA(cudaMemcpyAsync((void *)hd, hidden, R * n_embd * sizeof(float), cudaMemcpyHostToDevice, st));
    const bool bf3 = !(flags & WB_PATH_EXACT) && n_embd % 8 == 0;  // bf16x3 tensor-core product
    Carve cv;
    const size_t o_rot = corrector ? cv.take<float>(R * n_embd) : 0;
    const size_t o_a = bf3 ? cv.take<__nv_bfloat16>(2 * R * n_embd) : 0;
    const size_t o_t = bf3 ? cv.take<__nv_bfloat16>(2 * (size_t)vocab * n_embd) : 0;
    if (cv.off) WB_TRY(ensure(ctx->ws, cv.off));
    char *w = (char *)ctx->ws.p;
    const float *src = hd;
    if (corrector) {
        float *rot = (float *)(w + o_rot);
        if (wb::launch_rotate_bands(hd, R, n_embd / 2, corrector, rot, st))
            return fail(WB_ECUDA, "rotation launch failed");
        src = rot;
    }
    int rc;
    if (!bf3) {
        rc = wb::launch_vocab_dot(src, n_rows, n_embd, table, vocab, ld, st);
        if (rc) return fail(rc, "vocabulary dot launch failed");
    } else {
        std::string msg;
        __nv_bfloat16 *a_hi = (__nv_bfloat16 *)(w + o_a), *a_lo = a_hi + R * n_embd;
        __nv_bfloat16 *t_hi = (__nv_bfloat16 *)(w + o_t), *t_lo = t_hi + (size_t)vocab * n_embd;
        if ((rc = wb::split_bf16(src, R * n_embd, a_hi, a_lo, st)) ||
            (rc = wb::split_bf16(table, (long long)vocab * n_embd, t_hi, t_lo, st)))
            return fail(rc, "split launch failed");
        if ((rc = wb::tc_gemm_bf16x3(a_hi, a_lo, t_hi, t_lo, nullptr, ld, n_rows, vocab, n_embd, ctx->dev_err, st,
                                     &msg)))
            return fail(rc, msg);
    }
    if (!l_dev) {
        WB_CUDA(cudaMemcpyAsync(logits, ld, R * vocab * sizeof(float), cudaMemcpyDeviceToHost, st));
        WB_CUDA(cudaStreamSynchronize(st));
    }
    return WB_OK;
}

int wb_phase_native_decode(wb_context *ctx, const float *hidden, int n_rows, int n_embd, const float *corrector,
                           const float *wte, int vocab, int flags, float *logits) {
    if (!corrector) return fail(WB_EINVAL, "NULL corrector");
    return vocab_logits(ctx, hidden, n_rows, n_embd, corrector, wte, vocab, flags, logits);
}

int wb_lm_head(wb_context *ctx, const float *hidden, int n_rows, int n_embd, const float *lm_head, int vocab,
               int flags, float *logits) {
    return vocab_logits(ctx, hidden, n_rows, n_embd, nullptr, lm_head, vocab, flags, logits);
}

int wb_test_dot_core(wb_context *ctx, const float *qkv, int B, int T, int E, int H, int mode, float *o) {
    if (!ctx || !qkv || !o) return fail(WB_EINVAL, "NULL argument");
    if (B <= 0 || T <= 0 || H <= 0 || E <= 0 || E % H || mode < 0 || mode > 2) return fail(WB_EINVAL, "bad shape or mode");
    DeviceGuard g(ctx->device);
    ProfBind pb(ctx);
    std::string msg;
    int rc;
    if (mode == 2) {
        rc = wb::launch_dot_attn(qkv, B, T, E, H, o, ctx->stream, &msg);
    } else {
        WB_TRY(ensure(ctx->ws, wb::tc_dot_core_bytes(B, T, E, H)));
        rc = wb::tc_dot_attention(qkv, B, T, E, H, o, ctx->ws.p, mode == 1, ctx->dev_err, ctx->sm_count, ctx->stream,
                                  &msg);
    }
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
