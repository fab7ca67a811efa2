"""The serve-tier layer around the attention on the GPU (wb_layer_norm,
wb_ffn_forward + wb_agc, wb_embed, wb_residual_add, wb_phase_native_decode,
wb_lm_head, and ServeSession composing them as kv_cache.rs prefill /
forward_one) against the CPU oracle (oracle/serve_oracle.c).

Tolerances (the J10 rule |a - b| <= tol_abs + tol_rel * max(|a|, |b|)):
the all-fp32 path keeps the reference's operation order except for the
LayerNorm and AGC reductions and the last bits of tanhf / sinf / cosf, so it
is held to (2e-5, 1e-4); the tensor path (out_proj and the vocabulary
products as bf16x3 tcgen05 products) to max-abs 2e-3, the attention tensor
path's budget."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tests.parity import TENSOR_TOL, check

pytestmark = pytest.mark.gpu

FP32_TOL = (2e-5, 1e-4)


def test_layer_norm_matches_oracle(ctx):
    import wave_engine_b200 as wb
    g = np.random.default_rng(0)
    for n in (168, 768, 4096):
        x = (g.standard_normal((37, n)) * 3 + 0.5).astype(np.float32)
        w = g.standard_normal(n).astype(np.float32)
        b = g.standard_normal(n).astype(np.float32)
        r = check(f"layer_norm {n}", wb.layer_norm(x, w, b, ctx=ctx), oracle.layer_norm(x, w, b), FP32_TOL)
        assert r.passed, str(r)


@pytest.mark.parametrize("path,tol", [("exact", FP32_TOL), ("tensor", TENSOR_TOL)])
@pytest.mark.parametrize("E,groups", [(168, 1), (512, 1), (768, 1), (768, 4)])
def test_ffn_matches_oracle_over_a_sequence_of_calls(ctx, path, tol, E, groups):
    """Twelve calls of 3 rows each (the AGC's first nine observations replace
    its state, later ones are EMA updates), then one call holding four
    requests of 2 rows (four reference calls in one launch), then two requests
    of 300 rows.  168-dim: the
    plain stencil (84 bands); 512: 256 bands, a power of two, where the
    reference's FFT convolution wraps around; 768: 384 bands padded to 512.
    Inputs of std 1.5 push magnitudes past the AGC threshold."""
    import wave_engine_b200 as wb
    w = wb.gaussian_ffn(E + groups, E, 16, out_groups=groups, phase_correction_std=0.2)
    wp = w.packed()
    g = np.random.default_rng(E)
    agc_o = oracle.agc_new()
    agc_g = wb.Agc(ctx)
    for call in range(12):
        x = (g.standard_normal((3, E)) * 1.5).astype(np.float32)
        y = wb.ffn_forward(w, agc_g, x, path=path, ctx=ctx)
        r = check(f"call {call}", y, oracle.ffn_forward(wp, agc_o, x), tol)
        assert r.passed, str(r)
    x = (g.standard_normal((8, E)) * 1.5).astype(np.float32)
    y = wb.ffn_forward(w, agc_g, x, rows_per_call=2, path=path, ctx=ctx)
    ref = np.concatenate([oracle.ffn_forward(wp, agc_o, x[2 * i:2 * i + 2]) for i in range(4)])
    r = check("four requests in one call", y, ref, tol)
    assert r.passed, str(r)
    # two requests of 300 rows: the AGC statistics over several blocks per
    # request, and (tensor path) the bf16x3 out_proj for 256 rows and more
    x = (g.standard_normal((600, E)) * 1.5).astype(np.float32)
    y = wb.ffn_forward(w, agc_g, x, rows_per_call=300, path=path, ctx=ctx)
    ref = np.concatenate([oracle.ffn_forward(wp, agc_o, x[300 * i:300 * i + 300]) for i in range(2)])
    r = check("two long requests", y, ref, tol)
    assert r.passed, str(r)
    st = agc_g.state()
    assert st["count"] == agc_o.count == 18
    for k in ("ema_mean", "ema_var", "threshold"):
        assert abs(st[k] - getattr(agc_o, k)) <= 1e-5 * max(1.0, abs(getattr(agc_o, k))), k
    assert ctx.take_device_error() == 0


@pytest.mark.parametrize("path,tol", [("exact", FP32_TOL), ("tensor", TENSOR_TOL)])
def test_decoders_and_embedding_match_oracle(ctx, path, tol):
    import torch
    import wave_engine_b200 as wb
    E, V = 768, 1003
    g = np.random.default_rng(4)
    wte = (g.standard_normal((V, E)) / np.sqrt(E)).astype(np.float32)
    wpe = (g.standard_normal((64, E)) * 0.1).astype(np.float32)
    corr = (g.standard_normal(E // 2) * 0.5).astype(np.float32)
    head = (g.standard_normal((V, E)) * 0.02).astype(np.float32)
    hidden = g.standard_normal((5, E)).astype(np.float32)
    dev = lambda a: torch.from_numpy(a).cuda()
    lp = wb.phase_native_decode(hidden, dev(corr), dev(wte), path=path, ctx=ctx)
    lh = wb.lm_head(hidden, dev(head), path=path, ctx=ctx)
    for i in range(5):
        r = check(f"phase_native row {i}", lp[i], oracle.phase_native_decode(hidden[i], corr, wte), tol)
        assert r.passed, str(r)
        r = check(f"lm_head row {i}", lh[i], oracle.lm_head(hidden[i], head), tol)
        assert r.passed, str(r)
    tok = np.array([5, 1002, 0, 63, 7], np.int32)
    idx = np.array([5, 70, 0, 63, 2], np.int32)  # 70 >= n_pos: no wpe row
    h = wb.embed(tok, idx, dev(wte), dev(wpe), ctx=ctx)
    torch.cuda.synchronize()
    assert np.array_equal(h.cpu().numpy(), oracle.embed(tok, idx, wte, wpe))
    assert ctx.take_device_error() == 0


def _model(seed, E, H, L, V, phase_native):
    import wave_engine_b200 as wb
    g = np.random.default_rng(seed)
    blocks = []
    for l in range(L):
        blocks.append(wb.ServeBlock(
            (1 + 0.1 * g.standard_normal(E)).astype(np.float32), (0.05 * g.standard_normal(E)).astype(np.float32),
            (1 + 0.1 * g.standard_normal(E)).astype(np.float32), (0.05 * g.standard_normal(E)).astype(np.float32),
            wb.gaussian_block_attn(seed + 10 * l, H, E, 0), wb.gaussian_ffn(seed + 10 * l + 1, E, 16,
                                                                            phase_correction_std=0.1)))
    wte = (g.standard_normal((V, E)) / np.sqrt(E)).astype(np.float32)
    wpe = (g.standard_normal((48, E)) * 0.1).astype(np.float32)
    return wb.ServeModel(wte, wpe, blocks, np.ones(E, np.float32), np.zeros(E, np.float32),
                         output_corrector=(g.standard_normal(E // 2) * 0.3).astype(np.float32) if phase_native else None,
                         lm_head=None if phase_native else (g.standard_normal((V, E)) * 0.05).astype(np.float32))


def _oracle_serve(m, tokens, steps_tokens, cap):
    """kv_cache.rs prefill then forward_one, for the requests in the order a
    batched session visits the process-wide AGC (layer by layer, request by
    request)."""
    n_seq, T = tokens.shape
    E = m.wte.shape[1]
    agc = oracle.agc_new()
    hid = [oracle.embed(tokens[i], tokens[i], m.wte, m.wpe) for i in range(n_seq)]
    states = [[None] * len(m.blocks) for _ in range(n_seq)]

    def run_layers(rows_of, prefill):
        for l, b in enumerate(m.blocks):
            wp = b.attn.packed()
            fp = b.ffn.packed()
            att = []
            for i in range(n_seq):
                normed = oracle.layer_norm(rows_of[i], b.ln_w, b.ln_b)
                if prefill:
                    y, st = oracle.kv_prefill(wp, normed, cap)
                    states[i][l] = st
                else:
                    y = oracle.kv_decode(wp, normed[0], states[i][l])[None]
                att.append(y)
            for i in range(n_seq):
                ffn = oracle.ffn_forward(fp, agc, oracle.layer_norm(rows_of[i], b.ln_ffn_w, b.ln_ffn_b))
                rows_of[i] = rows_of[i] + (att[i] + ffn)

    def decode(rows):
        fin = oracle.layer_norm(rows, m.ln_f_w, m.ln_f_b)
        if m.output_corrector is not None:
            return np.stack([oracle.phase_native_decode(r, m.output_corrector, m.wte) for r in fin])
        return np.stack([oracle.lm_head(r, m.lm_head) for r in fin])

    run_layers(hid, True)
    out = [decode(np.stack([h[T - 1] for h in hid]))]
    for s, tk in enumerate(steps_tokens):
        rows = [oracle.embed(tk[i:i + 1], np.array([T + s], np.int32), m.wte, m.wpe) for i in range(n_seq)]
        run_layers(rows, False)
        out.append(decode(np.concatenate(rows)))
    return out, agc


@pytest.mark.parametrize("phase_native", [True, False])
def test_serve_session_matches_oracle(ctx, phase_native):
    """Two requests through a 2-layer 168-dim model on the all-fp32 path:
    prefill of 20 tokens, then three decode steps; logits compared at every
    step, and the AGC state at the end."""
    import wave_engine_b200 as wb
    E, H, L, V, T = 168, 4, 2, 300, 20
    m = _model(7 if phase_native else 8, E, H, L, V, phase_native)
    g = np.random.default_rng(1)
    tokens = g.integers(0, V, (2, T)).astype(np.int32)
    steps = [g.integers(0, V, 2).astype(np.int32) for _ in range(3)]
    sess = wb.ServeSession(m, max_seqs=3, max_ctx=T + 8, ctx=ctx, path="exact")
    ids = np.array([2, 0], np.int32)
    got = [sess.prefill(tokens, ids).cpu().numpy()]
    for s, tk in enumerate(steps):
        got.append(sess.forward_one(tk, np.full(2, T + s, np.int32), ids).cpu().numpy())
    ref, agc = _oracle_serve(m, tokens, steps, T + 8)
    for s, (a, b) in enumerate(zip(got, ref)):
        r = check(f"logits step {s}", a, b, (1e-4, 1e-4))
        assert r.passed, str(r)
    st = sess.agc.state()
    assert st["count"] == agc.count
    assert abs(st["threshold"] - agc.threshold) <= 1e-5
    assert ctx.take_device_error() == 0


def test_serve_decode_graph_equals_eager(ctx):
    """forward_one captured in one CUDA graph (tensor path) gives the eager
    calls' logits bit for bit over four replays."""
    import wave_engine_b200 as wb
    E, H, L, V, T = 768, 12, 2, 500, 40
    m = _model(11, E, H, L, V, True)
    g = np.random.default_rng(2)
    tokens = g.integers(0, V, (3, T)).astype(np.int32)
    steps = [g.integers(0, V, 3).astype(np.int32) for _ in range(4)]
    ids = np.array([1, 0, 2], np.int32)
    outs = []
    for graph in (False, True):
        sess = wb.ServeSession(m, max_seqs=3, max_ctx=T + 8, ctx=ctx)
        sess.prefill(tokens, ids)
        if graph:
            sess.capture_decode(ids)
        got = []
        for s, tk in enumerate(steps):
            pos = np.full(3, T + s, np.int32)
            y = sess.forward_one_graph(tk, pos) if graph else sess.forward_one(tk, pos, ids)
            got.append(y.cpu().numpy().copy())
        outs.append(got)
    for a, b in zip(*outs):
        assert np.array_equal(a, b)
    assert ctx.take_device_error() == 0
