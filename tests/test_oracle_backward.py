"""CPU tests of the attention-backward restatement in the oracle
(oracle/wave_oracle.c: src/common/math/attn_backward.rs composed as
src/common/attn.rs:346-430 wave_attention_backward_full).

The primitives are pinned by the reference's own known-answer tests
(attn_backward.rs:336-430, same inputs, same expected values and
tolerances); the composition is checked against central finite differences
of a float64 statement of the forward with the bucket mask held fixed (the
mask is piecewise constant and the reference's gradient treats it so)."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle

TAU = 6.2831855


def test_out_proj_backward_known_answer():
    """attn_backward.rs:336-350: identity out_proj, 2 positions."""
    d_out, d_w, d_b = oracle.bwd_out_proj([[1, 0], [0, 1]], [[3, 4], [5, 6]], [[1, 0], [0, 1]])
    assert abs(d_out[0, 0] - 1.0) < 1e-6 and abs(d_out[0, 1]) < 1e-6
    assert abs(d_w[0, 0] - 3.0) < 1e-6
    assert abs(d_b[0] - 1.0) < 1e-6


def test_softmax_backward_known_answer():
    """attn_backward.rs:352-365."""
    d = oracle.bwd_softmax([[1, 0], [2, 4]], [[1, 0], [0.3, 0.7]])
    assert abs(d[0, 0]) < 1e-6
    assert abs(d[1, 0] + 0.42) < 1e-4
    assert abs(d[1, 1] - 0.42) < 1e-4


def test_value_aggregation_backward_known_answer():
    """attn_backward.rs:367-379."""
    d_aw, d_v = oracle.bwd_value_aggregation([[1, 0], [0, 1]], [[1, 0], [0.5, 0.5]], [[1, 2], [3, 4]])
    assert abs(d_aw[0, 0] - 1.0) < 1e-6
    assert abs(d_v[0, 0] - 1.0) < 1e-6 and abs(d_v[0, 1] - 0.5) < 1e-6


def test_phase_projection_backward_known_answer():
    """attn_backward.rs:381-395: identity projection, x = [1, 0], phase 0."""
    d_x, _, _ = oracle.bwd_phase_projection([1.0], [[1, 0]], [[1, 0], [0, 1]], [0, 0])
    assert abs(d_x[0, 0]) < 1e-6 and abs(d_x[0, 1] - 1.0) < 1e-6


def test_value_projection_backward_known_answer():
    """attn_backward.rs:397-410."""
    d_x, d_w, d_b = oracle.bwd_value_projection([[1, 0]], [[3, 4]], 0, [[1, 0], [0, 1]])
    assert abs(d_x[0, 0] - 1.0) < 1e-6 and abs(d_x[0, 1]) < 1e-6
    assert abs(d_w[0, 0] - 3.0) < 1e-6
    assert abs(d_b[0] - 1.0) < 1e-6


def test_combine_d_normed_known_answer():
    """attn_backward.rs:412-429: two heads, t = 1, n_embd = 4, no content."""
    dxp = np.array([[[1, 0, 0, 0]], [[0, 0, 0.5, 0]]], np.float32)
    dxv = np.array([[[0, 2, 0, 0]], [[0, 0, 0, 3]]], np.float32)
    r = oracle.bwd_combine(dxp, dxv)
    assert np.allclose(r[0], [1.0, 2.0, 0.5, 3.0], atol=1e-6)


# ---------------------------------------------------------------------------
# the composition against finite differences
# ---------------------------------------------------------------------------
def _bucket(th):
    n = np.fmod(np.fmod(th, TAU) + TAU, TAU)
    return np.minimum((n / (TAU / 8)).astype(np.int64), 7)


def _forward64(w, x, mask=None):
    """float64 wave attention (attn.rs:116-285) for x [T][E]; mask [H][T][T] of
    kept pairs (computed from the phases when None).  Returns (y, mask)."""
    H = w["harmonic_raw"].shape[0]
    T, E = x.shape
    hd = E // H
    cw = w.get("content_proj_w")
    Cd = 0 if cw is None or cw.size == 0 else cw.shape[1]
    merged = np.zeros((T, E))
    masks = []
    for h in range(H):
        raw = float(w["harmonic_raw"][h])
        hn = raw if raw > 20 else np.log1p(np.exp(raw))
        rs = x @ w["phase_proj_w"][h].T.astype(np.float64) + w["phase_proj_b"][h]
        th = np.arctan2(rs[:, 1], rs[:, 0])
        v = x[:, h * hd:(h + 1) * hd] @ w["v_proj_w"][h].T.astype(np.float64) + w["v_proj_b"][h]
        c = x @ w["content_proj_w"][h].T.astype(np.float64) + w["content_proj_b"][h] if Cd else None
        if mask is None:
            b = _bucket(th)
            m = np.zeros((T, T), bool)
            for q in range(T):
                for k in range(q + 1):
                    m[q, k] = ((b[k] - b[q]) % 8) in (0, 1, 7) or k == q - 1
        else:
            m = mask[h]
        masks.append(m)
        s = np.cos(hn * (th[:, None] - th[None, :]))
        if Cd:
            s = s + (c @ c.T) / np.sqrt(Cd)
        s = np.where(m, s, -np.inf)
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        merged[:, h * hd:(h + 1) * hd] = p @ v
    y = merged @ w["out_proj_w"].T.astype(np.float64) + w["out_proj_b"]
    return y, np.array(masks)


@pytest.mark.parametrize("Cd", [0, 4])
def test_backward_full_matches_finite_differences(Cd):
    import wave_engine_b200 as wb
    H, E, T = 2, 16, 6
    w = wb.init_block_attn(wb.Rng(7 + Cd), H, E, Cd).packed()
    w = {k: (None if v is None else np.asarray(v, np.float64)) for k, v in w.items()}
    rng = np.random.default_rng(11)
    x = rng.standard_normal((T, E))
    g = rng.standard_normal((T, E))
    _, mask = _forward64(w, x)

    def loss(ww=None, xx=None):
        y, _ = _forward64(ww or w, x if xx is None else xx, mask)
        return float((y * g).sum())

    grads = oracle.attn_backward_full(w, x, g)
    eps = 1e-6

    def fd_x(i, j):
        xp, xm = x.copy(), x.copy()
        xp[i, j] += eps
        xm[i, j] -= eps
        return (loss(xx=xp) - loss(xx=xm)) / (2 * eps)

    def fd_w(key, idx):
        wp = {k: (None if v is None else v.copy()) for k, v in w.items()}
        wm = {k: (None if v is None else v.copy()) for k, v in w.items()}
        wp[key][idx] += eps
        wm[key][idx] -= eps
        return (loss(ww=wp) - loss(ww=wm)) / (2 * eps)

    def close(a, b):
        return abs(a - b) <= 1e-4 + 2e-3 * max(abs(a), abs(b))

    for i in range(T):
        for j in range(E):
            assert close(grads["d_x"][i, j], fd_x(i, j)), ("d_x", i, j)
    picks = {"out_proj_w": [(0, 0), (3, 5), (15, 2)], "out_proj_b": [(1,), (9,)],
             "phase_proj_w": [(0, 0, 3), (1, 1, 7)], "phase_proj_b": [(0, 1), (1, 0)],
             "v_proj_w": [(0, 2, 3), (1, 7, 0)], "v_proj_b": [(0, 4), (1, 1)], "harmonic_raw": [(0,), (1,)]}
    if Cd:
        picks.update({"content_proj_w": [(0, 1, 5), (1, 3, 12)], "content_proj_b": [(0, 2), (1, 0)]})
    for key, idxs in picks.items():
        for idx in idxs:
            assert close(grads[key][idx], fd_w(key, idx)), (key, idx, grads[key][idx], fd_w(key, idx))
