"""GPU parity of the CUDA library against the CPU oracle (reference math).

Every case runs through the C ABI (wave_engine_b200 -> libwave_b200.so).
Tolerances: WB_PATH_EXACT (all-fp32 SIMT) max-abs 1e-5; WB_PATH_TENSOR
(tcgen05 bf16 scores/PV, fp32 accumulation) max-abs 2e-3.

Phases go through atan2f, whose CUDA and glibc implementations differ in the
last bits, and the tensor path computes the phase projection (r, s) with
3xTF32 tensor-core products summed in another order than the reference's
sequential loop, so a phase lying very close to a bucket boundary can land
in the neighbouring bucket.  The comparison therefore checks the phases (to
2e-6 rad on the exact path, 5e-5 rad on the tensor path), allows bucket
differences only that close to a boundary, and in that case recomputes the
oracle with the GPU's phases (mask-conditioned parity) so that the rest of
the math is still compared element by element.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import oracle
from tests.parity import EXACT_TOL, TENSOR_TOL, boundary_distance, buckets_of, check, phase_diff

pytestmark = pytest.mark.gpu

NT = os.cpu_count() or 1


def make_case(E, H, C, B, T, seed, init="gauss"):
    import wave_engine_b200 as wb
    if init == "gauss":
        w = wb.gaussian_block_attn(seed, H, E, C)
    else:
        w = wb.init_block_attn(wb.Rng(seed), H, E, C)
    x = np.random.default_rng(seed + 1).standard_normal((B, T, E)).astype(np.float32)
    return w, x


PHASE_TOL = {"exact": 2e-6, "tensor": 5e-5}


def oracle_for(wp, x, gpu_phases, use_content=True, path="tensor"):
    """Oracle outputs per sequence, conditioned on the GPU's buckets where
    (and only where) a phase sits within twice the phase tolerance of a
    bucket boundary."""
    if not use_content:
        wp = dict(wp, content_proj_w=None, content_proj_b=None)
    tol = PHASE_TOL[path]
    ys, aws, flips = [], [], 0
    for b in range(x.shape[0]):
        y, aw, ph = oracle.attn_forward(wp, x[b], want_att_w=True, n_threads=NT)
        gp = gpu_phases[b]
        assert phase_diff(gp, ph).max() <= tol, f"phase mismatch {phase_diff(gp, ph).max()}"
        diff = buckets_of(gp) != buckets_of(ph)
        if diff.any():
            assert (boundary_distance(ph)[diff] < 2 * tol).all(), "bucket differs away from a boundary"
            flips += int(diff.sum())
            y, aw, _ = oracle.attn_forward(wp, x[b], want_att_w=True, phase_override=gp, n_threads=NT)
        ys.append(y)
        aws.append(aw)
    return np.stack(ys), np.stack(aws), flips


SHAPES = [
    # E, H, C, B, T
    (168, 4, 16, 2, 64),    # 168-dim research model (head_dim 42)
    (384, 8, 16, 1, 129),   # 384-dim grammar model (head_dim 48), ragged T
    (768, 12, 16, 2, 130),  # 768-dim production model (head_dim 64)
    (768, 12, 0, 1, 17),    # --freeze-ode: no content projection
    (64, 1, 16, 3, 1),      # T = 1
    (64, 2, 16, 2, 2),      # T = 2
]


@pytest.mark.parametrize("E,H,C,B,T", SHAPES)
@pytest.mark.parametrize("init", ["gauss", "reference"])
def test_exact_path_matches_oracle(ctx, E, H, C, B, T, init):
    import wave_engine_b200 as wb
    w, x = make_case(E, H, C, B, T, seed=E + T, init=init)
    y, aw, _, ph = wb.wave_attention_forward(w, x, E // 2, path="exact", return_att_weights=True,
                                            return_phases=True, ctx=ctx)
    oy, oaw, flips = oracle_for(w.packed(), x, ph, path="exact")
    r = check("y", y, oy, EXACT_TOL)
    assert r.passed, str(r)
    r = check("att_w", aw, oaw, EXACT_TOL)
    assert r.passed, str(r)
    assert ctx.take_device_error() == 0


@pytest.mark.parametrize("E,H,C,B,T", SHAPES + [
    (768, 12, 16, 2, 1024),
    (4096, 32, 16, 1, 48),
    # head_dim 128 over several query and key tiles: the 2-stage K/V ring
    # wraps, the single P buffer is reused, diagonal tiles after j > 0
    (512, 4, 16, 2, 520),
    (4096, 32, 16, 1, 300),
    # head_dim 128 with 320 work items: the persistent CTAs take two or three
    # items each, so the single O buffer passes from item to item
    (512, 4, 16, 16, 640),
])
def test_tensor_path_matches_oracle(ctx, E, H, C, B, T):
    import wave_engine_b200 as wb
    w, x = make_case(E, H, C, B, T, seed=3 * E + T)
    y, _, _, ph = wb.wave_attention_forward(w, x, E // 2, path="tensor", return_phases=True, ctx=ctx)
    oy, _, flips = oracle_for(w.packed(), x, ph)
    r = check("y", y, oy, TENSOR_TOL)
    assert r.passed, str(r)
    assert ctx.take_device_error() == 0


def test_tensor_path_reference_init_and_no_content(ctx):
    import wave_engine_b200 as wb
    w, x = make_case(384, 8, 16, 2, 200, seed=5, init="reference")
    for use_content in (True, False):
        y, _, _, ph = wb.wave_attention_forward(w, x, 192, path="tensor", use_content=use_content,
                                                return_phases=True, ctx=ctx)
        oy, _, _ = oracle_for(w.packed(), x, ph, use_content=use_content)
        r = check(f"y content={use_content}", y, oy, TENSOR_TOL)
        assert r.passed, str(r)


def test_single_sequence_and_torch_inputs(ctx):
    import torch
    import wave_engine_b200 as wb
    w, x = make_case(168, 4, 16, 1, 33, seed=11)
    y_np, att, cache = wb.wave_attention_forward(w, x[0], 84, path="exact", ctx=ctx)
    assert y_np.shape == (33, 168) and att == [] and cache is None
    xt = torch.from_numpy(x[0]).cuda()
    y_t, _, _ = wb.wave_attention_forward(w, xt, 84, path="exact", ctx=ctx)
    torch.cuda.synchronize()
    assert y_t.is_cuda and np.array_equal(y_t.cpu().numpy(), y_np)


def test_argument_errors(ctx):
    import wave_engine_b200 as wb
    w, x = make_case(168, 4, 16, 1, 8, seed=2)
    with pytest.raises(ValueError):
        wb.wave_attention_forward(w, x, 80, ctx=ctx)  # n_bands mismatch
    with pytest.raises(ValueError):
        wb.wave_attention_forward(w, x[0, :, :100], 50, ctx=ctx)  # weights for another n_embd


# ---------------------------------------------------------------------------
# KV cache: prefill + decode (kv_cache.rs)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("path,tol", [("exact", EXACT_TOL), ("tensor", TENSOR_TOL)])
@pytest.mark.parametrize("E,H", [(168, 4), (768, 12)])
def test_kv_prefill_and_decode_match_oracle(ctx, path, tol, E, H):
    import wave_engine_b200 as wb
    n_seq, T, steps = 3, 40, 6
    w, x = make_case(E, H, 16, n_seq, T + steps, seed=E + 17)
    wp = w.packed()
    d = E // H
    cache = wb.KvCache(1, H, d, max_seqs=4, max_ctx=T + steps, ctx=ctx)
    seq_ids = np.array([2, 0, 3], np.int32)
    y = cache.prefill(0, w, x[:, :T], seq_ids, path=path)
    states = []
    for i in range(n_seq):
        oy, st = oracle.kv_prefill(wp, x[i, :T], cap=T + steps)
        states.append(st)
        ph, bk, vv = cache.read(0, int(seq_ids[i]))
        assert phase_diff(ph, st.phases[:, :T]).max() <= PHASE_TOL[path]
        same = bk == st.buckets[:, :T]
        assert (same | (boundary_distance(st.phases[:, :T]) < 2 * PHASE_TOL[path])).all()
        if not same.all():
            # a phase next to a bucket boundary landed in the neighbouring
            # bucket: the oracle reruns with the GPU's phases (the serve
            # prefill is the forward without content), and the decode state
            # continues from the GPU's phases and buckets
            oy, _, _ = oracle.attn_forward(dict(wp, content_proj_w=None, content_proj_b=None), x[i, :T],
                                           phase_override=ph, n_threads=NT)
            st.phases[:, :T] = ph
            st.buckets[:, :T] = oracle.phase_to_bucket(ph)
        r = check(f"prefill y seq{i}", y[i], oy, tol)
        assert r.passed, str(r)
        assert check("values", vv, st.values[:, :T], EXACT_TOL).passed
    for s in range(steps):
        yd = cache.forward_one(0, w, x[:, T + s].copy(), seq_ids, path=path)
        for i in range(n_seq):
            oyd = oracle.kv_decode(wp, x[i, T + s], states[i])
            r = check(f"decode step {s} seq{i}", yd[i], oyd, tol)
            assert r.passed, str(r)
    for i in range(n_seq):
        assert cache.n_cached(0, int(seq_ids[i])) == T + steps
    assert cache.n_cached(0, 1) == 0
    assert ctx.take_device_error() == 0


def test_kv_decode_equals_prefill_last_row(ctx):
    """GPU forward_one after prefill(T) agrees with prefill(T+1)'s last row."""
    import wave_engine_b200 as wb
    w, x = make_case(768, 12, 0, 2, 65, seed=9)
    c1 = wb.KvCache(1, 12, 64, max_seqs=2, max_ctx=65, ctx=ctx)
    c2 = wb.KvCache(1, 12, 64, max_seqs=2, max_ctx=65, ctx=ctx)
    y_full = c1.prefill(0, w, x, [0, 1], path="exact")
    c2.prefill(0, w, x[:, :64].copy(), [0, 1], path="exact")
    y_dec = c2.forward_one(0, w, x[:, 64].copy(), [0, 1], path="exact")
    r = check("decode vs prefill", y_dec, y_full[:, 64], (1e-6, 1e-6))
    assert r.passed, str(r)


def test_tensor_decode_rejects_head_dims_its_value_stream_cannot_split(ctx):
    """A tensor-path decode reads a value row with at most one warp's lanes,
    VEC floats each: head_dim 66 (VEC 2, 33 lanes) is refused with
    WB_ENOTSUP before any launch; the fp32 path decodes it against the
    oracle."""
    import wave_engine_b200 as wb
    from wave_engine_b200 import _lib
    w, x = make_case(132, 2, 0, 1, 9, seed=66)
    c = wb.KvCache(1, 2, 66, max_seqs=1, max_ctx=16, ctx=ctx)
    c.prefill(0, w, x[:, :8].copy(), [0], path="exact")
    with pytest.raises(wb.WaveB200Error) as e:
        c.forward_one(0, w, x[:, 8].copy(), [0], path="tensor")
    assert e.value.code == _lib.WB_ENOTSUP
    c.reset()
    c.prefill(0, w, x[:, :8].copy(), [0], path="exact")
    y = c.forward_one(0, w, x[:, 8].copy(), [0], path="exact")
    wp = w.packed()
    _, st = oracle.kv_prefill(wp, x[0, :8], cap=16)
    oy = oracle.kv_decode(wp, x[0, 8], st)
    r = check("hd 66 exact decode vs oracle", y.reshape(-1), oy.reshape(-1), EXACT_TOL)
    assert r.passed, str(r)
    assert ctx.take_device_error() == 0


def test_kv_cache_load_read_and_errors(ctx):
    import wave_engine_b200 as wb
    H, d, n = 4, 42, 50
    cache = wb.KvCache(2, H, d, max_seqs=2, max_ctx=64, ctx=ctx)
    g = np.random.default_rng(4)
    ph = np.arctan2(g.standard_normal((H, n)), g.standard_normal((H, n))).astype(np.float32)
    vv = g.standard_normal((H, n, d)).astype(np.float32)
    cache.load(1, 1, ph, vv)
    rp, rb, rv = cache.read(1, 1)
    assert np.array_equal(rp, ph) and np.array_equal(rv, vv)
    assert np.array_equal(rb, oracle.phase_to_bucket(ph).astype(np.uint8))
    w, x = make_case(168, 4, 16, 1, 70, seed=3)
    with pytest.raises(wb.WaveB200Error):
        cache.prefill(0, w, x, [0])  # seq_len > max_ctx
    with pytest.raises(wb.WaveB200Error):
        cache.prefill(1, w, x[:, :10].copy(), [1])  # slot not empty
    with pytest.raises(wb.WaveB200Error):
        cache.forward_one(0, w, x[:, 0].copy(), [5])  # seq id out of range
    cache.reset_seq(1)
    assert cache.n_cached(1, 1) == 0


@pytest.mark.parametrize("E,H,ctx_len", [(168, 4, 700), (384, 8, 1100), (768, 12, 1200), (768, 12, 1300),
                                         (4096, 32, 520)])
def test_fused_decode_long_context_matches_oracle(ctx, E, H, ctx_len):
    """Fused decode of long loaded caches, head dims 42/48/64/128.  Caches of
    up to 1536 positions take one CTA of 8, 10 or 12 warps per (sequence, head)
    (warp partials merged in shared memory); longer caches are covered by
    test_decode_stress_shape_splits_and_gemm_out_proj."""
    import wave_engine_b200 as wb
    d = E // H
    w = wb.gaussian_block_attn(E + 1, H, E, 0)
    wp = w.packed()
    g = np.random.default_rng(E)
    n_seq, steps = 3, 3
    cache = wb.KvCache(1, H, d, max_seqs=n_seq, max_ctx=ctx_len + steps, ctx=ctx)
    states = []
    for i in range(n_seq):
        n = ctx_len - 97 * i
        ph = np.arctan2(g.standard_normal((H, n)), g.standard_normal((H, n))).astype(np.float32)
        vv = g.standard_normal((H, n, d)).astype(np.float32)
        cache.load(0, i, ph, vv)
        st = oracle.KvState(H, d, ctx_len + steps)
        st.phases[:, :n] = ph
        st.values[:, :n] = vv
        st.buckets[:, :n] = oracle.phase_to_bucket(ph)
        st.n.value = n
        states.append(st)
    x = g.standard_normal((steps, n_seq, E)).astype(np.float32)
    for s in range(steps):
        y = cache.forward_one(0, w, x[s], np.arange(n_seq, dtype=np.int32))
        for i in range(n_seq):
            oy = oracle.kv_decode(wp, x[s, i], states[i])
            r = check(f"step {s} seq {i}", y[i], oy, TENSOR_TOL)
            assert r.passed, str(r)
    for i in range(n_seq):
        ph, bk, vv = cache.read(0, i)
        n = states[i].n_cached
        assert ph.shape[1] == n
        # the fused kernel sums the phase projection as a tree, not in the
        # reference's sequential order: a few ulps of (r, s), ~1e-6 rad
        assert phase_diff(ph, states[i].phases[:, :n]).max() <= 2e-5
        assert check("appended values", vv, states[i].values[:, :n], (1e-5, 1e-5)).passed
    assert ctx.take_device_error() == 0


def test_fused_decode_from_empty_cache_and_device_ids(ctx):
    """n_cached = 0 gives o = v_new (softmax over the self score only); device
    seq ids skip host validation and still advance the lengths."""
    import torch
    import wave_engine_b200 as wb
    w = wb.gaussian_block_attn(3, 12, 768, 0)
    wp = w.packed()
    cache = wb.KvCache(1, 12, 64, max_seqs=4, max_ctx=8, ctx=ctx)
    x = np.random.default_rng(1).standard_normal((2, 768)).astype(np.float32)
    ids = torch.tensor([3, 1], dtype=torch.int32, device="cuda")
    xt = torch.from_numpy(x).cuda()
    y = cache.forward_one(0, w, xt, ids)
    torch.cuda.synchronize()
    for i in range(2):
        st = oracle.KvState(12, 64, 8)
        oy = oracle.kv_decode(wp, x[i], st)
        assert check("empty-cache decode", y[i].cpu().numpy(), oy, TENSOR_TOL).passed
    assert cache.n_cached(0, 3) == 1 and cache.n_cached(0, 1) == 1 and cache.n_cached(0, 0) == 0
    assert ctx.take_device_error() == 0


def test_decode_graph_capture_replays_like_eager(ctx):
    """A decode step captured in a CUDA graph (device ids, device buffers)
    replays to the same outputs as eager calls on a twin cache."""
    import torch
    import wave_engine_b200 as wb
    H, E, T, L = 12, 768, 200, 2
    ws = [wb.gaussian_block_attn(50 + l, H, E, 16) for l in range(L)]
    layers = [wb.AttnLayer(ctx, w) for w in ws]
    g = torch.Generator(device="cuda").manual_seed(0)
    xp = torch.randn((L, 4, T, E), generator=g, device="cuda")
    xd = torch.randn((3, L, 4, E), generator=g, device="cuda")
    ids = torch.arange(4, dtype=torch.int32, device="cuda")
    caches = [wb.KvCache(L, H, 64, max_seqs=4, max_ctx=T + 3, ctx=ctx) for _ in range(2)]
    yp = torch.empty((4, T, E), device="cuda")
    for c in caches:
        for l in range(L):
            c.prefill(l, layers[l], xp[l], ids, out=yp)
    stage = torch.empty((L, 4, E), device="cuda")
    y_graph = torch.empty((L, 4, E), device="cuda")
    y_eager = torch.empty((3, L, 4, E), device="cuda")
    graph = torch.cuda.CUDAGraph()
    stage.copy_(xd[0])
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    # eager step 0 on cache 1 first (allocates the decode scratch)
    for l in range(L):
        caches[1].forward_one(l, layers[l], xd[0, l], ids, out=y_eager[0, l])
    torch.cuda.synchronize()
    with torch.cuda.graph(graph, stream=s):
        for l in range(L):
            caches[0].forward_one(l, layers[l], stage[l], ids, out=y_graph[l])
    torch.cuda.current_stream().wait_stream(s)
    for step in range(3):
        stage.copy_(xd[step])
        graph.replay()
        if step > 0:
            for l in range(L):
                caches[1].forward_one(l, layers[l], xd[step, l], ids, out=y_eager[step, l])
        torch.cuda.synchronize()
        assert torch.equal(y_graph, y_eager[step]), step
    assert caches[0].n_cached(1, 2) == T + 3
    del graph
    assert ctx.take_device_error() == 0


@pytest.mark.parametrize("L", [1, 2, 3])
def test_chained_decode_matches_unchained(ctx, L):
    """Back-to-back decode calls (layer after layer, step after step) launch
    each attention grid as a programmatic dependent of the previous layer's
    out_proj.  The same steps with a torch kernel between the calls (nothing
    chains) give bitwise the same outputs and lengths; with one layer the
    consecutive steps of that layer must not chain at all."""
    import torch
    import wave_engine_b200 as wb
    H, E, T, B, steps = 12, 768, 300, 4, 5
    layers = [wb.AttnLayer(ctx, wb.gaussian_block_attn(70 + l, H, E, 16)) for l in range(L)]
    g = torch.Generator(device="cuda").manual_seed(5)
    xp = torch.randn((L, B, T, E), generator=g, device="cuda")
    xd = torch.randn((steps, L, B, E), generator=g, device="cuda")
    ids = torch.tensor([2, 0, 3, 1], dtype=torch.int32, device="cuda")
    caches = [wb.KvCache(L, H, 64, max_seqs=B, max_ctx=T + steps, ctx=ctx) for _ in range(2)]
    yp = torch.empty((B, T, E), device="cuda")
    for c in caches:
        for l in range(L):
            c.prefill(l, layers[l], xp[l], ids, out=yp)
    ys = [torch.empty((steps, L, B, E), device="cuda") for _ in range(2)]
    bump = torch.zeros(1, device="cuda")
    for s in range(steps):
        for l in range(L):
            caches[0].forward_one(l, layers[l], xd[s, l], ids, out=ys[0][s, l])
    for s in range(steps):
        for l in range(L):
            caches[1].forward_one(l, layers[l], xd[s, l], ids, out=ys[1][s, l])
            bump.add_(1.0)
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1])
    for l in range(L):
        assert all(caches[0].n_cached(l, i) == T + steps for i in range(B))
    assert ctx.take_device_error() == 0
    # the last step against the oracle (tensor-path tolerance)
    for l in range(L):
        wp = wb.gaussian_block_attn(70 + l, H, E, 16).packed()
        xs = xp[l].cpu().numpy()
        for i in range(B):
            _, st = oracle.kv_prefill(wp, xs[i], cap=T + steps)
            for s in range(steps):
                od = oracle.kv_decode(wp, xd[s, l, i].cpu().numpy(), st)
            r = check(f"layer {l} seq {i}", ys[0][steps - 1, l, i].cpu().numpy(), od, TENSOR_TOL)
            assert r.passed, str(r)


def test_tensor_path_fallback_tiles_for_unbounded_scores(ctx):
    """Content weights 100x larger push |c_q|(max|c_k| - |c_q|)/4 past the
    fixed-shift bound; those query tiles are recomputed by the fp32 SIMT
    kernel and the result still matches the oracle."""
    import wave_engine_b200 as wb
    w, x = make_case(168, 4, 16, 2, 150, seed=77)
    for hw in w.heads:
        hw.content_proj_w = hw.content_proj_w * 100.0
    w.invalidate()
    ctx.profile("attn_simt_fallback")
    y, _, _, ph = wb.wave_attention_forward(w, x, 84, path="tensor", return_phases=True, ctx=ctx)
    rep = ctx.profile_report()
    ctx.profile(None)
    oy, _, _ = oracle_for(w.packed(), x, ph)
    r = check("y (fallback tiles)", y, oy, TENSOR_TOL)
    assert r.passed, str(r)
    assert "attn_simt_fallback" in rep
    assert ctx.take_device_error() == 0


def test_decode_batches_of_different_sizes_share_scratch(ctx):
    """Decode calls with 3, then 1, then 2 sequences on one cache: the
    scratch tickets must stay zeroed between calls of different batch."""
    import wave_engine_b200 as wb
    H, E, d = 12, 768, 64
    w = wb.gaussian_block_attn(8, H, E, 0)
    wp = w.packed()
    g = np.random.default_rng(2)
    cache = wb.KvCache(1, H, d, max_seqs=4, max_ctx=1400, ctx=ctx)
    states = {}
    for sidx in range(4):
        n = 600 + 200 * sidx
        ph = np.arctan2(g.standard_normal((H, n)), g.standard_normal((H, n))).astype(np.float32)
        vv = g.standard_normal((H, n, d)).astype(np.float32)
        cache.load(0, sidx, ph, vv)
        st = oracle.KvState(H, d, 1400)
        st.phases[:, :n] = ph
        st.values[:, :n] = vv
        st.buckets[:, :n] = oracle.phase_to_bucket(ph)
        st.n.value = n
        states[sidx] = st
    for ids in ([0, 2, 3], [1], [3, 0], [2, 1, 0, 3]):
        x = g.standard_normal((len(ids), E)).astype(np.float32)
        y = cache.forward_one(0, w, x, np.array(ids, np.int32))
        for j, sidx in enumerate(ids):
            oy = oracle.kv_decode(wp, x[j], states[sidx])
            r = check(f"ids {ids} seq {sidx}", y[j], oy, TENSOR_TOL)
            assert r.passed, str(r)
    assert ctx.take_device_error() == 0


@pytest.mark.parametrize("ids_on_device", [False, True])
def test_decode_stress_shape_splits_and_gemm_out_proj(ctx, ids_on_device):
    """A reduced decode-stress configuration (768-dim, 12 heads x 64, fp32
    cache of N(0,1) values and uniform phases): 72 sequences, so out_proj runs
    on the tcgen05 GEMM (64 rows and more) followed by the length update;
    contexts drawn from U[128, 4096] in a cache of 4099 positions, so every
    (sequence, head) is split over 4-warp CTAs of 512 keys whose partials the
    last CTA merges through the atomic ticket, with 1 to 9 active splits per
    sequence (lengths 128, 512, 513 and 4096 pin the split boundaries); three
    steps in a row reuse the tickets."""
    import torch
    import wave_engine_b200 as wb
    H, E, d = 12, 768, 64
    n_seq, steps = 72, 3
    cap = 4096 + steps
    w = wb.gaussian_block_attn(404, H, E, 0)
    wp = w.packed()
    g = np.random.default_rng(404)
    lens = g.integers(128, 4097, n_seq)
    lens[:4] = (128, 512, 513, 4096)
    cache = wb.KvCache(1, H, d, max_seqs=n_seq, max_ctx=cap, ctx=ctx)
    states = []
    for i, n in enumerate(lens):
        n = int(n)
        ph = np.arctan2(g.standard_normal((H, n)), g.standard_normal((H, n))).astype(np.float32)
        vv = g.standard_normal((H, n, d), dtype=np.float32)
        cache.load(0, i, ph, vv)
        st = oracle.KvState(H, d, n + steps)
        st.phases[:, :n] = ph
        st.values[:, :n] = vv
        st.buckets[:, :n] = oracle.phase_to_bucket(ph)
        st.n.value = n
        states.append(st)
    order = g.permutation(n_seq).astype(np.int32)  # slots in a shuffled order
    ids = torch.from_numpy(order).cuda() if ids_on_device else order
    ctx.profile("gemm_tf32")
    for s in range(steps):
        x = g.standard_normal((n_seq, E), dtype=np.float32)
        xin = torch.from_numpy(x).cuda() if ids_on_device else x
        y = cache.forward_one(0, w, xin, ids)
        if ids_on_device:
            torch.cuda.synchronize()
            y = y.cpu().numpy()
        for j, sidx in enumerate(order):
            oy = oracle.kv_decode(wp, x[j], states[sidx])
            r = check(f"step {s} slot {sidx} (context {lens[sidx] + s})", y[j], oy, TENSOR_TOL)
            assert r.passed, str(r)
    rep = ctx.profile_report()
    ctx.profile(None)
    assert "gemm_tf32" in rep  # out_proj of 72 rows ran on the tensor-core GEMM
    for sidx in (0, 3, int(order[-1])):
        assert cache.n_cached(0, sidx) == lens[sidx] + steps
        ph, bk, vv = cache.read(0, sidx)
        st = states[sidx]
        assert phase_diff(ph, st.phases[:, :st.n_cached]).max() <= 2e-5
        assert check("appended values", vv[:, -steps:], st.values[:, st.n_cached - steps:st.n_cached],
                     (1e-5, 1e-5)).passed
    assert ctx.take_device_error() == 0


# ---- the GPU against the committed oracle dumps of the benchmark
# configurations (tests/golden/configs.npz)

def _configs():
    from pathlib import Path
    return np.load(Path(__file__).resolve().parent / "golden" / "configs.npz")


@pytest.mark.parametrize("case", ["cfg1_168", "cfg2_384", "cfg3_768", "cfg5_4096"])
@pytest.mark.parametrize("path,tol", [("exact", EXACT_TOL), ("tensor", TENSOR_TOL)])
def test_config_fixture_prefill(ctx, case, path, tol):
    """Prefill of each configuration (reduced T) against the fixture; where
    a GPU phase lands in the neighbouring bucket (only next to a boundary)
    the oracle is rerun with the GPU's phases for that sequence."""
    import wave_engine_b200 as wb
    from tests.golden import config_cases as cc
    fx = _configs()
    name, E, H, C, B, T, init, seed = next(c for c in cc.PREFILL if c[0] == case)
    wp = cc.weights(init, seed, H, E, C)
    w = wb.WaveAttnWeights.from_packed(wp)
    x = cc.inputs(seed, B, T, E)
    y, _, _, ph = wb.wave_attention_forward(w, x, E // 2, path=path, return_phases=True, ctx=ctx)
    for b in range(B):
        ref_ph = fx[case + "/phases"][b]
        assert phase_diff(ph[b], ref_ph).max() <= PHASE_TOL[path]
        diff = buckets_of(ph[b]) != buckets_of(ref_ph)
        expect = fx[case + "/y"][b]
        if diff.any():
            assert (boundary_distance(ref_ph)[diff] < 2 * PHASE_TOL[path]).all()
            expect, _, _ = oracle.attn_forward(wp, x[b], phase_override=ph[b], n_threads=NT)
        r = check(f"{case} {path} seq{b}", y[b], expect, tol)
        assert r.passed, str(r)
    assert ctx.take_device_error() == 0


@pytest.mark.parametrize("case", ["cfg3_decode", "cfg4_ragged"])
@pytest.mark.parametrize("path,tol", [("exact", EXACT_TOL), ("tensor", TENSOR_TOL)])
def test_config_fixture_decode(ctx, case, path, tol):
    """Prompts of different lengths prefilled into their own slots, then
    decode steps of all sequences together, against the fixture."""
    import wave_engine_b200 as wb
    from tests.golden import config_cases as cc
    fx = _configs()
    name, E, H, lens, steps, seed = next(c for c in cc.DECODE if c[0] == case)
    w = wb.WaveAttnWeights.from_packed(cc.weights("gauss", seed, H, E, 0))
    x = cc.inputs(seed, len(lens), max(lens) + steps, E)
    cache = wb.KvCache(1, H, E // H, max_seqs=len(lens), max_ctx=max(lens) + steps, ctx=ctx)
    for b, n in enumerate(lens):
        cache.prefill(0, w, x[b:b + 1, :n].copy(), [b], path=path)
    ids = list(range(len(lens)))
    for s in range(steps):
        xs = np.stack([x[b, n + s] for b, n in enumerate(lens)])
        yd = cache.forward_one(0, w, xs, ids, path=path)
        r = check(f"{case} {path} step{s}", yd, fx[case + "/y"][s], tol)
        assert r.passed, str(r)
    assert ctx.take_device_error() == 0


@pytest.mark.parametrize("E,H,C,T,groups", [
    (768, 12, 16, 130, [(0, 4), (4, 9), (9, 12)]),
    (4096, 32, 16, 40, [(0, 8), (8, 16), (16, 24), (24, 32)]),
    # the two-GPU split of the 4096-dim model at T = 1024: 256 work items
    # per range, several per persistent CTA at head_dim 128
    (4096, 32, 16, 1024, [(0, 16), (16, 32)]),
])
def test_head_ranges_sum_to_the_full_forward(ctx, E, H, C, T, groups):
    """wb_attn_forward_heads over ranges that cover every head once (bias on
    one of them) sums to wb_attn_forward's output (the same kernels on the
    same phases; only out_proj's K is split).  The 768-dim full output is
    also checked against the oracle here; the 4096-dim forward's oracle
    parity is covered by the configuration fixture and the shape tests."""
    import wave_engine_b200 as wb
    w, x = make_case(E, H, C, 2, T, seed=E + T)
    y, _, _, ph = wb.wave_attention_forward(w, x, E // 2, path="tensor", return_phases=True, ctx=ctx)
    parts = [wb.wave_attention_forward_heads(w, x, E // 2, h0, h1, add_bias=(h0 == 0), ctx=ctx)
             for h0, h1 in groups]
    r = check("sum of head ranges vs full", np.sum(parts, axis=0), y, (2e-5, 0))
    assert r.passed, str(r)
    if E == 768:
        oy, _, _ = oracle_for(w.packed(), x, ph)
        r = check("full vs oracle", y, oy, TENSOR_TOL)
        assert r.passed, str(r)
    assert ctx.take_device_error() == 0


def test_head_range_errors(ctx):
    import wave_engine_b200 as wb
    from wave_engine_b200 import _lib
    w, x = make_case(168, 4, 16, 1, 8, seed=3)
    with pytest.raises(wb.WaveB200Error) as e:   # 1 * 42 floats is not 16-byte aligned
        wb.wave_attention_forward_heads(w, x, 84, 1, 3, add_bias=False, ctx=ctx)
    assert e.value.code == _lib.WB_ENOTSUP
    with pytest.raises(wb.WaveB200Error) as e:
        wb.wave_attention_forward_heads(w, x, 84, 2, 2, add_bias=False, ctx=ctx)
    assert e.value.code == _lib.WB_EINVAL
    y = wb.wave_attention_forward_heads(w, x, 84, 0, 4, add_bias=True, ctx=ctx)
    y_full, _, _ = wb.wave_attention_forward(w, x, 84, ctx=ctx)
    assert np.allclose(y, y_full, atol=2e-5, rtol=0)
