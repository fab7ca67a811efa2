"""Attention backward on the GPU (wb_attn_forward_cache + wb_attn_backward)
against the CPU oracle's restatement of src/common/attn.rs:346-430
wave_attention_backward_full (oracle/wave_oracle.c wo_attn_backward_full,
itself pinned by the reference's known-answer tests and by finite
differences in tests/test_oracle_backward.py).

Tolerance: the GPU sums in another order than the reference's loops (per
query, per key, per weight over positions), so each gradient is compared
with the J10 rule |a - b| <= tol_abs + tol_rel * max(|a|, |b|) at
tol_abs = 2e-5 * max|oracle| of that tensor and tol_rel = 1e-3.  The cache
arrays come from the all-fp32 forward and are held to the exact path's
1e-5.  A phase that lands in the neighbouring bucket (only next to a
boundary) would change the mask; the seeds below have none, and the test
checks that the GPU's buckets equal the oracle's before comparing."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tests.parity import EXACT_TOL, buckets_of, check, phase_diff

pytestmark = pytest.mark.gpu

NT = 8
GRADS = ("out_proj_w", "out_proj_b", "phase_proj_w", "phase_proj_b", "v_proj_w", "v_proj_b", "content_proj_w",
         "content_proj_b", "harmonic_raw")


def _case(E, H, C, B, T, seed, init="gauss"):
    import wave_engine_b200 as wb
    w = wb.gaussian_block_attn(seed, H, E, C) if init == "gauss" else wb.init_block_attn(wb.Rng(seed), H, E, C)
    g = np.random.default_rng(seed + 7)
    x = g.standard_normal((B, T, E)).astype(np.float32)
    d_y = g.standard_normal((B, T, E)).astype(np.float32)
    return w, x, d_y


def _grad_tol(ref):
    m = float(np.max(np.abs(ref))) if np.size(ref) else 0.0
    return (2e-5 * max(m, 1e-6), 1e-3)


@pytest.mark.parametrize("E,H,C,B,T,init", [
    (168, 4, 16, 2, 33, "gauss"),      # 168-dim research model, head_dim 42
    (384, 8, 16, 1, 65, "reference"),  # 384-dim, head_dim 48, the reference's init
    (768, 12, 0, 2, 40, "gauss"),      # --freeze-ode (no content), head_dim 64
    (512, 4, 16, 1, 70, "gauss"),      # head_dim 128
    (64, 2, 16, 3, 1, "gauss"),        # T = 1
])
def test_backward_full_matches_oracle(ctx, E, H, C, B, T, init):
    import wave_engine_b200 as wb
    w, x, d_y = _case(E, H, C, B, T, seed=E + T, init=init)
    wp = w.packed()
    y, att, cache = wb.wave_attention_forward(w, x, E // 2, return_pathway_cache=True, ctx=ctx)
    grads = wb.wave_attention_backward_full(w, cache, d_y, ctx=ctx)
    ref_sum = {}
    for b in range(B):
        oy, oaw, oph = oracle.attn_forward(wp, x[b], want_att_w=True, n_threads=NT)
        assert phase_diff(cache.phases[b], oph).max() <= 2e-6
        assert (buckets_of(cache.phases[b]) == buckets_of(oph)).all(), "bucket flip: pick another seed"
        assert check("y", y[b], oy, EXACT_TOL).passed
        assert check("att_w", cache.att_w[b], oaw, EXACT_TOL).passed
        g = oracle.attn_backward_full(wp, x[b], d_y[b])
        r = check(f"d_normed seq {b}", grads["d_normed"][b], g["d_x"], _grad_tol(g["d_x"]))
        assert r.passed, str(r)
        for k in GRADS:
            if g.get(k) is not None:
                ref_sum[k] = ref_sum.get(k, 0.0) + g[k]
    for k in GRADS:
        if k not in ref_sum:
            assert grads.get(k) is None
            continue
        r = check(k, grads[k], ref_sum[k], _grad_tol(ref_sum[k]))
        assert r.passed, str(r)
    assert ctx.take_device_error() == 0


def test_backward_pathway_equals_full_d_normed_and_torch_inputs(ctx):
    """wave_attention_backward_pathway (attn.rs:432) returns the full
    backward's d_normed; the same call on CUDA tensors gives the same result."""
    import torch
    import wave_engine_b200 as wb
    w, x, d_y = _case(768, 12, 16, 2, 50, seed=3)
    _, _, cache = wb.wave_attention_forward(w, x, 384, return_pathway_cache=True, ctx=ctx)
    full = wb.wave_attention_backward_full(w, cache, d_y, ctx=ctx)
    d_n = wb.wave_attention_backward_pathway(w, cache, d_y, ctx=ctx)
    assert np.array_equal(d_n, full["d_normed"])
    xt, dyt = torch.from_numpy(x).cuda(), torch.from_numpy(d_y).cuda()
    yt, _, cache_t = wb.wave_attention_forward(w, xt, 384, return_pathway_cache=True, ctx=ctx)
    full_t = wb.wave_attention_backward_full(w, cache_t, dyt, ctx=ctx)
    torch.cuda.synchronize()
    for k in ("d_normed", "out_proj_w", "phase_proj_w", "v_proj_w", "content_proj_w", "harmonic_raw"):
        assert np.allclose(full_t[k].cpu().numpy(), full[k], rtol=1e-6, atol=1e-7), k
    assert ctx.take_device_error() == 0


def test_backward_argument_errors(ctx):
    import wave_engine_b200 as wb
    w, x, d_y = _case(168, 4, 16, 1, 8, seed=2)
    _, _, cache = wb.wave_attention_forward(w, x, 84, return_pathway_cache=True, ctx=ctx)
    with pytest.raises(ValueError):
        wb.wave_attention_backward_full(w, cache, d_y[:, :4].copy(), ctx=ctx)  # wrong shape
