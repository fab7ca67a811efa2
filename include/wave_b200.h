/*
 * wave_b200.h -- C ABI of the B200 (sm_100a) wave-attention library.
 *
 * This is the drop-in boundary for wave-engine's causal multi-head wave
 * attention forward.  Each entry point replaces one reference interface
 * (cited as path:line inside the wave-engine source tree):
 *
 *   wb_attn_forward   <- src/common/attn.rs:90  wave_attention_forward(...)
 *                        (callers: src/cpu/forward.rs:113,240,
 *                         src/common/block.rs:47, and the Candle CustomOp
 *                         src/candle_tier/custom_attn.rs:89-130 cpu_fwd)
 *   wb_kv_prefill     <- src/common/kv_cache.rs:121-193 (attention part of
 *                        prefill: phases, values, buckets, scores, out_proj)
 *   wb_kv_decode      <- src/common/kv_cache.rs:263-335 (attention part of
 *                        forward_one)
 *   wb_attn_layer_*   <- src/common/attn.rs:19-46 WaveAttnHeadWeights /
 *                        WaveAttnWeights (device-resident copy)
 *   wb_kv_cache_*     <- src/common/kv_cache.rs:36-54 HeadCache/LayerCache/
 *                        KvCache (device-resident, one slot per sequence)
 *   wb_attn_forward_cache <- src/common/attn.rs:90 with return_pathway_cache
 *                        = true (WaveAttnCache, attn.rs:51-70)
 *   wb_attn_backward  <- src/common/attn.rs:346 wave_attention_backward_full
 *                        and :432 wave_attention_backward_pathway (caller:
 *                        src/candle_tier/custom_attn.rs:132 bwd)
 *   wb_ffn_*, wb_agc_* <- src/common/ffn.rs:39-230 ffn_forward_via_backend as
 *                        the serve tier calls it (kv_cache.rs:199-209,
 *                        :341-351), agc.rs OdeAgc
 *   wb_layer_norm     <- src/common/model.rs:154 layer_norm
 *   wb_embed, wb_residual_add, wb_phase_native_decode, wb_lm_head
 *                     <- the rest of kv_cache.rs prefill / forward_one
 *                        (:106-113, :220, :18-33, :365-378)
 *
 * Conventions
 *   - Every function returns int status: WB_OK (0) or a negative WB_E*.
 *     No exceptions cross the ABI; nothing aborts or traps.  The message of
 *     the last failure on the calling thread is returned by wb_last_error().
 *   - All floating point data is fp32, row-major, in the reference's
 *     layouts (a Rust Vec<Vec<f32>> [rows][cols] flattened row by row).
 *   - Data pointers may be host or device memory; the library detects which
 *     (cudaPointerGetAttributes).  Host inputs are copied into the
 *     context's device staging buffer with cudaMemcpyAsync (pinned host
 *     memory makes that copy asynchronous); when an output is host memory
 *     the call synchronises the context's stream before returning.  With
 *     device pointers only, the call is asynchronous on the context's
 *     stream.
 *   - A context is bound to one device and one stream and is not
 *     thread-safe; use one context per thread (the reference runs attention
 *     on a thread per batch element / per HTTP request).
 *   - Results are pure functions of (weights, x, flags).  The prefill path
 *     WB_PATH_TENSOR computes scores and PV on tcgen05 tensor cores in bf16
 *     with fp32 accumulation (max-abs error vs the reference <= 2e-3);
 *     WB_PATH_EXACT runs all-fp32 SIMT kernels that follow the reference's
 *     operation order (max-abs error <= 1e-5).
 */
#ifndef WAVE_B200_H
#define WAVE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WB_ABI_VERSION 1

#if defined(__GNUC__)
#define WB_API __attribute__((visibility("default")))
#else
#define WB_API
#endif

/* status codes */
#define WB_OK 0
#define WB_EINVAL -1    /* bad argument or shape */
#define WB_ENOMEM -2    /* device or pinned allocation failed */
#define WB_ECUDA -3     /* CUDA runtime / driver error */
#define WB_ENOTSUP -4   /* feature not supported (e.g. pathway cache) */
#define WB_ETIMEOUT -5  /* a device-side bounded wait gave up */
#define WB_ENODEV -6    /* no usable sm_100 device */

/* flags for wb_attn_forward / wb_kv_prefill / wb_kv_decode */
#define WB_PATH_TENSOR 0x0      /* default: tcgen05 bf16 scores + PV */
#define WB_PATH_EXACT 0x1       /* all-fp32 SIMT kernels, reference order */
#define WB_NO_CONTENT 0x2       /* ignore content_proj even if present */
#define WB_RETURN_PATHWAY 0x4   /* return_pathway_cache=true: WB_ENOTSUP */

typedef struct wb_context wb_context;
typedef struct wb_attn_layer wb_attn_layer;
typedef struct wb_kv_cache wb_kv_cache;
typedef struct wb_dot_attn_layer wb_dot_attn_layer;
typedef struct wb_ffn_layer wb_ffn_layer;
typedef struct wb_agc wb_agc;

/* Host-side view of one block's attention weights (attn.rs:19-46),
 * flattened per head.  All pointers are HOST memory and are only read
 * during wb_attn_layer_create.
 *   harmonic_raw  [n_head]                 (n_h = softplus(harmonic_raw))
 *   phase_proj_w  [n_head][2][n_embd]      phase_proj_b [n_head][2]
 *   v_proj_w      [n_head][hd][hd]         v_proj_b     [n_head][hd]
 *   content_proj_w[n_head][C][n_embd]      content_proj_b [n_head][C]
 *                 (C = content_dim, 0 or 16; NULL when 0)
 *   out_proj_w    [n_embd][n_embd]         out_proj_b   [n_embd]
 * with hd = n_embd / n_head. */
typedef struct {
    int32_t n_embd;
    int32_t n_head;
    int32_t content_dim;
    const float *harmonic_raw;
    const float *phase_proj_w;
    const float *phase_proj_b;
    const float *v_proj_w;
    const float *v_proj_b;
    const float *content_proj_w;
    const float *content_proj_b;
    const float *out_proj_w;
    const float *out_proj_b;
} wb_attn_weights_desc;

/* ---- library / context ------------------------------------------------ */
WB_API int wb_abi_version(void);
/* Thread-local message for the last non-zero status on this thread. */
WB_API const char *wb_last_error(void);
/* Create a context on `device` (CUDA ordinal) using its own stream.
 * Layers and caches created on a context must be destroyed before it;
 * their destroy functions stay safe to call after it (they only free
 * device memory). */
WB_API int wb_context_create(int device, wb_context **out);
WB_API int wb_context_destroy(wb_context *ctx);
/* Run later calls on an external cudaStream_t.  As everywhere in CUDA, NULL
 * is the legacy default stream (e.g. torch's default stream), not the
 * context's own stream; wb_context_own_stream returns the latter. */
WB_API int wb_context_set_stream(wb_context *ctx, void *cuda_stream);
WB_API void *wb_context_own_stream(wb_context *ctx);
WB_API int wb_context_synchronize(wb_context *ctx);
/* Device error word: non-zero when a bounded device-side wait gave up or a
 * kernel-side check failed since the last reset.  Resets it. */
WB_API int wb_context_take_device_error(wb_context *ctx, uint32_t *code_out);

/* Kernel timing: with name_filter non-NULL, every later compute call on this
 * context brackets its named kernels whose name contains name_filter ("" =
 * all) with CUDA events on the context's stream; NULL turns timing off.
 * Replaces the reference's --monitor PROFILE timers (src/common/dims.rs:14,
 * src/cpu/forward.rs:60) with device-side timing. */
WB_API int wb_context_profile(wb_context *ctx, const char *name_filter);
/* Synchronise, then write "kernel<TAB>launches<TAB>total_ms" lines for the
 * launches recorded since the last report into buf (NUL-terminated). */
WB_API int wb_context_profile_report(wb_context *ctx, char *buf, size_t len);

/* ---- weights (attn.rs:19-46) ------------------------------------------ */
WB_API int wb_attn_layer_create(wb_context *ctx, const wb_attn_weights_desc *w, wb_attn_layer **out);
WB_API int wb_attn_layer_destroy(wb_attn_layer *layer);
/* Reference weight initialisation (src/common/wave_model.rs:39-81,
 * init_linear + init_block_attn) on the xorshift64 stream of
 * src/common/rng.rs:24-39.  *rng_state advances exactly as the reference's
 * Rng does.  Buffers are host memory in the layouts above. */
WB_API int wb_init_block_attn(uint64_t *rng_state, int n_head, int n_embd, int content_dim,
                       float *harmonic_raw, float *phase_proj_w, float *phase_proj_b,
                       float *v_proj_w, float *v_proj_b, float *content_proj_w,
                       float *content_proj_b, float *out_proj_w, float *out_proj_b);

/* ---- prefill forward (attn.rs:90-305) --------------------------------- */
/* x [batch][seq_len][n_embd] -> y [batch][seq_len][n_embd]; each sequence is
 * an independent call of the reference.  att_w (nullable) receives the
 * reference's second return value [batch][n_head][seq_len][seq_len]
 * (softmax weights, -inf above the diagonal exactly as attn.rs:240 leaves
 * them); requesting it routes the scores through WB_PATH_EXACT.
 * phases_out (nullable) receives the per-head phases [batch][n_head][seq_len]
 * used for the bucket mask. */
WB_API int wb_attn_forward(wb_context *ctx, const wb_attn_layer *layer, const float *x, int batch,
                    int seq_len, int flags, float *y, float *att_w, float *phases_out);

/* ---- forward cache and backward (attn.rs:51-70, :346-430) ------------- */
/* The WaveAttnCache of attn.rs:51-70 for a batch of sequences (each array
 * stacks the reference's per-sequence arrays over the batch):
 *   phases     [batch][n_head][seq_len]            (cache.phases)
 *   phase_rs   [batch][n_head][seq_len][2]         (cache.phase_rs: (r, s))
 *   v_all      [batch][n_head][seq_len][head_dim]  (cache.v_all)
 *   content    [batch][n_head][seq_len][content_dim] or NULL without content
 *   att_w      [batch][n_head][seq_len][seq_len]   (cache.att_w, 0 above the
 *              diagonal and for masked keys)
 *   out_merged [batch][seq_len][n_embd]            (cache.out_merged)
 * cache.normed is the forward's x; cache.content_scale is 1/sqrt(C). */
typedef struct {
    float *phases;
    float *phase_rs;
    float *v_all;
    float *content;
    float *att_w;
    float *out_merged;
} wb_attn_cache_desc;

/* Weight gradients in the layouts of wb_attn_weights_desc (WaveAttnGrads,
 * attn.rs:346-430), summed over the batch; NULL entries are not computed. */
typedef struct {
    float *harmonic_raw;
    float *phase_proj_w;
    float *phase_proj_b;
    float *v_proj_w;
    float *v_proj_b;
    float *content_proj_w;
    float *content_proj_b;
    float *out_proj_w;
    float *out_proj_b;
} wb_attn_grads_desc;

/* attn.rs:90 wave_attention_forward with return_pathway_cache = true: y as
 * wb_attn_forward's WB_PATH_EXACT (all-fp32 SIMT) and the cache above.
 * flags: WB_NO_CONTENT. */
WB_API int wb_attn_forward_cache(wb_context *ctx, const wb_attn_layer *layer, const float *x, int batch,
                                 int seq_len, int flags, float *y, const wb_attn_cache_desc *cache);

/* attn.rs:346-430 wave_attention_backward_full from the cache and the output
 * gradient d_y [batch][seq_len][n_embd]: the input gradient d_x (d_normed)
 * and, when grads is non-NULL, the weight gradients summed over the batch.
 * With grads NULL this is wave_attention_backward_pathway (attn.rs:432).
 * x is the forward's input (cache.normed).  fp32 on the GPU; the sums run in
 * another order than the reference's loops (see the tests' tolerance).
 * flags: WB_NO_CONTENT (as in the forward).  head_dim <= 128. */
WB_API int wb_attn_backward(wb_context *ctx, const wb_attn_layer *layer, const float *x, const float *d_y,
                            int batch, int seq_len, int flags, const wb_attn_cache_desc *cache, float *d_x,
                            const wb_attn_grads_desc *grads);

/* Head-sharded prefill (no counterpart in the reference, which runs all
 * heads in one call): the forward of heads [head_begin, head_end) only,
 * y_partial = o[:, heads] W_out[:, heads]^T, plus out_proj's bias when
 * add_bias != 0.  Summing the y_partial of ranges that cover every head
 * exactly once, with add_bias set on exactly one of them, gives
 * wb_attn_forward's y (up to float summation order): the sharding of the
 * 4096-dim model across GPUs by heads, with one all-reduce of y_partial.
 * Tensor path only (flags: WB_NO_CONTENT); head_begin * head_dim must be a
 * multiple of 4. */
WB_API int wb_attn_forward_heads(wb_context *ctx, const wb_attn_layer *layer, const float *x, int batch,
                                 int seq_len, int head_begin, int head_end, int add_bias, int flags, float *y_partial);

/* ---- Dot-product attention (compute.rs:43, :357-414) ------------------ */
/* The legacy causal self-attention of ComputeBackend::attention
 * (compute.rs:43 -> attention_cpu, compute.rs:357-414; the same math as
 * model_forward.rs:124-180): q, k, v = c_attn(x); per head softmax(q k^T /
 * sqrt(head_dim)) over keys <= the query, times v; y = c_proj(heads).
 * Weights as AttentionWeights (model.rs:191-195): c_attn_w [3*n_embd][n_embd]
 * and c_proj_w [n_embd][n_embd] in LinearWeights' [out][in] row-major layout
 * (model.rs:177-180), biases [3*n_embd] and [n_embd]; host memory, copied.
 * head_dim <= 128. */
WB_API int wb_dot_attn_layer_create(wb_context *ctx, int n_head, int n_embd, const float *c_attn_w,
                                    const float *c_attn_b, const float *c_proj_w, const float *c_proj_b,
                                    wb_dot_attn_layer **out);
WB_API int wb_dot_attn_layer_destroy(wb_dot_attn_layer *layer);
/* x, y [batch][seq_len][n_embd], host or device.  flags: WB_PATH_EXACT runs
 * both projections as the reference's sequential fp32 sums (model.rs:144-150);
 * otherwise they run on the tensor cores in TF32 (n_embd a multiple of 4, a
 * device x 16-byte aligned).  The exact path's attention core is fp32; the
 * tensor path's runs on tcgen05 (bf16 q/sqrt(d) and k, fp16 probabilities and
 * values, features padded to 64 or 128 columns), and query tiles whose scores
 * could leave the fixed shift's range are recomputed by the fp32 core. */
WB_API int wb_dot_attn_forward(wb_context *ctx, const wb_dot_attn_layer *layer, const float *x, int batch,
                               int seq_len, int flags, float *y);

/* ---- KV cache (kv_cache.rs:36-54) ------------------------------------- */
/* One cache holds n_layers x max_seqs slots of capacity max_ctx positions,
 * each with per-head phases (f32), buckets (u8) and values (f32 [hd]). */
WB_API int wb_kv_cache_create(wb_context *ctx, int n_layers, int n_head, int head_dim, int max_seqs,
                       int max_ctx, wb_kv_cache **out);
WB_API int wb_kv_cache_destroy(wb_kv_cache *cache);
/* Number of cached positions of (layer, seq). */
WB_API int wb_kv_cache_length(wb_kv_cache *cache, int layer, int seq, int *len_out);
/* Empty a sequence slot in every layer (a new request); seq = -1 empties
 * every slot. */
WB_API int wb_kv_cache_reset_seq(wb_kv_cache *cache, int seq);

/* Paged KV cache (multi-request serving: src/serve_tier/inference.rs:44
 * creates one KvCache per request; here the requests share one pool).  Each
 * layer's storage is a pool of n_pages pages, a page holding WB_KV_PAGE
 * positions of every head; a slot's positions 128p .. 128p+127 live in the
 * page its page table maps p to.  A slot holds no positions until
 * wb_kv_seq_reserve gives it pages; a prefill or decode past a slot's
 * reserved pages fails with WB_EINVAL (host seq ids) or, with device seq
 * ids, is not written and sets bit 0x8 (bounds) of the device error word.
 * max_ctx (a slot's most positions) rounds up to whole pages.  Every other
 * call works on a paged cache as on a contiguous one, with the same results
 * bit for bit. */
#define WB_KV_PAGE 128
WB_API int wb_kv_cache_create_paged(wb_context *ctx, int n_layers, int n_head, int head_dim, int max_seqs,
                                    int max_ctx, int n_pages, wb_kv_cache **out);
/* Reserve pages so that slot seq holds n_positions (<= max_ctx) in every
 * layer; WB_ENOMEM (nothing reserved) when the pool is short.  Pages stay
 * with the slot until wb_kv_seq_release.  No-op on a contiguous cache. */
WB_API int wb_kv_seq_reserve(wb_kv_cache *cache, int seq, int n_positions);
/* Empty slot seq in every layer and return its pages to the pool
 * (synchronises the context's stream first).  On a contiguous cache:
 * wb_kv_cache_reset_seq. */
WB_API int wb_kv_seq_release(wb_kv_cache *cache, int seq);
/* Pages in the pool's free list (0 for a contiguous cache). */
WB_API int wb_kv_cache_free_pages(wb_kv_cache *cache, int *n_free);
/* Load n positions of one (layer, seq) slot from raw arrays: phases
 * [n_head][n], values [n_head][n][head_dim] (host or device).  Buckets are
 * derived from the phases exactly as kv_cache.rs:66-70.  Replaces the slot's
 * contents. */
WB_API int wb_kv_cache_load(wb_context *ctx, wb_kv_cache *cache, int layer, int seq, int n,
                     const float *phases, const float *values);
/* Read one (layer, seq) slot back: phases [n_head][len], buckets
 * [n_head][len] (u8), values [n_head][len][head_dim]; any may be NULL. */
WB_API int wb_kv_cache_read(wb_context *ctx, wb_kv_cache *cache, int layer, int seq, float *phases,
                     uint8_t *buckets, float *values);

/* kv_cache.rs:121-193: prompt attention for n_seq sequences of seq_len
 * positions each (x [n_seq][seq_len][n_embd]) into EMPTY slots seq_ids[i]
 * of `layer_idx`; writes y [n_seq][seq_len][n_embd] and fills the slots.
 * The serve copy of the math never adds the content bias. */
WB_API int wb_kv_prefill(wb_context *ctx, wb_kv_cache *cache, int layer_idx, const wb_attn_layer *layer,
                  const int32_t *seq_ids, int n_seq, const float *x, int seq_len, int flags,
                  float *y);

/* kv_cache.rs:263-335: one new position per sequence (x [n_seq][n_embd])
 * against slots seq_ids[i] of `layer_idx`; writes y [n_seq][n_embd] and
 * appends the new phase/bucket/value to each slot.
 * seq_ids in HOST memory are validated (range, duplicates, capacity) before
 * any work is queued.  seq_ids in DEVICE memory are not read by the host:
 * the call then does no host synchronisation and can be captured in a CUDA
 * graph and replayed (lengths live on the device); the kernels check range
 * and capacity and report violations through the device error word, and
 * duplicate ids are the caller's responsibility.  The same holds for
 * wb_kv_prefill, which additionally requires empty slots. */
WB_API int wb_kv_decode(wb_context *ctx, wb_kv_cache *cache, int layer_idx, const wb_attn_layer *layer,
                 const int32_t *seq_ids, int n_seq, const float *x, int flags, float *y);

/* Size of the static device array behind wb_kv_decode_noalloc (4 MiB). */
#define WB_NOALLOC_SCRATCH_BYTES (4u << 20)

/* wb_kv_decode on the tensor path without allocating any device memory.
 * No counterpart in the reference: it exists for callers that may not
 * allocate at decode time (a server that reserves its device memory at
 * start-up and forbids allocation per request; a host application whose own
 * memory pool owns the device and forbids outside cudaMalloc; a latency-
 * bound loop that cannot take cudaMalloc's implicit synchronisation or its
 * failure mid-request).  The kernels' scratch
 * lives in one static device array of WB_NOALLOC_SCRATCH_BYTES per GPU,
 * held until the process exits; a cache whose decode scratch
 * (slots x heads x splits partial rows -- one split up to max_ctx 1536,
 * else ceil(max_ctx/512) -- plus per-slot values and outputs) exceeds it is
 * rejected with WB_EINVAL.  seq_ids, x and y must be
 * DEVICE pointers (nothing is staged) and are used as with device ids in
 * wb_kv_decode.  The first call on each device resolves the array's device
 * address (cudaGetSymbolAddress) and must come before any stream capture.
 * All calls share the array: calls that overlap on the GPU race and must
 * not be issued; the counters that must start at zero are cleared by each
 * call. */
WB_API int wb_kv_decode_noalloc(wb_context *ctx, wb_kv_cache *cache, int layer_idx, const wb_attn_layer *layer,
                                const int32_t *seq_ids, int n_seq, const float *x, float *y);

/* ---- the serve-tier layer around the attention ------------------------- */
/* kv_cache.rs prefill (:93-236) and forward_one (:241-381) run, per layer,
 *   normed = layer_norm(hidden, ln); attn = attention(normed)   (wb_kv_*)
 *   normed_ffn = layer_norm(hidden, ln_ffn); ffn = FFN(normed_ffn)
 *   hidden += attn + ffn
 * and then layer_norm(hidden, ln_f) and a decoder.  The entries below are
 * those steps; with device pointers they queue on the context's stream
 * without host synchronisation, so a whole serve step stays on the GPU. */

/* KerrDualMaestroWeights of one block (model.rs, wave_model.rs:134-170) as
 * the serve tier runs it: ffn.rs:39-230 with a frozen ODE and no memory --
 * maestro_in, the AGC, the stencil Kerr ODE (fft_ode.rs:171-250; the
 * four-wave-mixing term is not part of that path), the corrector plate,
 * maestro_out and out_proj.  Arrays are host or device memory, row-major
 * [out][in] as the reference's Vec<Vec<f32>>; they are copied at creation. */
typedef struct {
    int n_embd;            /* 2 * n_bands */
    int maestro_dim;
    int rk4_steps;         /* KerrWeights::rk4_n_steps */
    int use_corrector;     /* Dims::use_corrector (the corrector plate) */
    int out_groups;        /* 1: dense out_proj; > 1: block-diagonal groups */
    const float *mi_squeeze_w, *mi_squeeze_b;   /* maestro_in: [M][E], [M] */
    const float *mi_process_w, *mi_process_b;   /*             [E][M], [E] */
    const float *mo_squeeze_w, *mo_squeeze_b;   /* maestro_out */
    const float *mo_process_w, *mo_process_b;
    const float *gamma_raw, *omega;             /* [n_bands] */
    float alpha, beta;
    const float *phase_correction;              /* [n_bands] */
    const float *rk4_weights;                   /* [4] */
    const float *out_w, *out_b;  /* dense: [E][E], [E]; block-diagonal: per group [gs][gs] then [gs],
                                    groups one after another in out_w (out_proj.rs flatten order), out_b NULL */
} wb_ffn_weights_desc;

WB_API int wb_ffn_layer_create(wb_context *ctx, const wb_ffn_weights_desc *w, wb_ffn_layer **out);
WB_API int wb_ffn_layer_destroy(wb_ffn_layer *layer);

/* agc.rs OdeAgc::from_coupling(alpha, beta) (OdeAgc::new() is 0.1, 0.1),
 * device resident.  The reference keeps one process-wide instance that every
 * FFN call updates (ffn.rs:76); pass the same wb_agc to every call to match
 * it. */
WB_API int wb_agc_create(wb_context *ctx, float alpha, float beta, wb_agc **out);
WB_API int wb_agc_destroy(wb_agc *agc);
/* state[8] = ema_mean, ema_var, headroom, decay, min_threshold,
 * max_threshold, threshold, count (synchronises the context's stream). */
WB_API int wb_agc_read(wb_agc *agc, float *state);

/* y = FFN(x), x and y [n_rows][n_embd] host or device.  The rows are
 * n_rows / rows_per_call consecutive reference calls (one request's rows
 * each): the AGC observes them one after another, in order, exactly as
 * that many ffn_forward_via_backend calls would.  flags: WB_PATH_EXACT runs
 * out_proj as the reference's sequential fp32 sums; otherwise a dense
 * out_proj (n_embd a multiple of 8) runs on the tcgen05 GEMM as a bf16x3
 * product (hi.hi + lo.hi + hi.lo, ~16 mantissa bits). */
WB_API int wb_ffn_forward(wb_context *ctx, const wb_ffn_layer *layer, wb_agc *agc, const float *x, int n_rows,
                          int rows_per_call, int flags, float *y);

/* model.rs:154 layer_norm of each row of n values; weight, bias [n]. */
WB_API int wb_layer_norm(wb_context *ctx, const float *x, int n_rows, int n, const float *weight, const float *bias,
                         float *y);

/* hidden[i] += a[i] + b[i] (kv_cache.rs:220, :352); DEVICE pointers. */
WB_API int wb_residual_add(wb_context *ctx, float *hidden, const float *a, const float *b, long long n);

/* hidden[r] = wte[tokens[r]] + wpe[wpe_index[r]] (the wpe row only when
 * wpe_index[r] < n_pos; wpe may be NULL).  kv_cache.rs prefill indexes wpe
 * by the token id (:108-110), forward_one by the position (:254-256): pass
 * the tokens or the positions as wpe_index.  wte [vocab][n_embd] and wpe
 * [n_pos][n_embd] are DEVICE pointers; tokens, wpe_index and hidden host or
 * device.  An out-of-range token sets bit 0x8 of the device error word. */
WB_API int wb_embed(wb_context *ctx, const int32_t *tokens, const int32_t *wpe_index, int n_rows, const float *wte,
                    int vocab, const float *wpe, int n_pos, int n_embd, float *hidden);

/* kv_cache.rs:18-33 phase_native_decode of each row of hidden [n_rows]
 * [n_embd]: every band rotated by corrector [n_embd/2], then logits[r][v] =
 * rotated . wte[v].  wb_lm_head (kv_cache.rs:365-378): logits = hidden .
 * lm_head[v].  The tables are DEVICE pointers; hidden and logits host or
 * device.  flags: WB_PATH_EXACT (sequential fp32 sums) or, for n_embd a
 * multiple of 8, the bf16x3 tensor-core product (the table is split into
 * bf16 hi / lo in the context's workspace on every call). */
WB_API int wb_phase_native_decode(wb_context *ctx, const float *hidden, int n_rows, int n_embd,
                                  const float *corrector, const float *wte, int vocab, int flags, float *logits);
WB_API int wb_lm_head(wb_context *ctx, const float *hidden, int n_rows, int n_embd, const float *lm_head, int vocab,
                      int flags, float *logits);

#ifdef __cplusplus
}
#endif
#endif /* WAVE_B200_H */
