"""CPU tests of the oracle (oracle/wave_oracle.c) against the known-answer
fixtures and the reference's invariants.  No GPU needed."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tests.parity import buckets_of, check

KAT_TOL = (2e-6, 2e-6)


@pytest.mark.parametrize("name", ["kat_t1", "kat_uniform", "kat_mask"])
def test_oracle_matches_known_answers(kat, name):
    c = kat[name]
    y, aw, _ = oracle.attn_forward(c["w"], c["x"], want_att_w=True)
    r = check(name + "/y", y, c["y"], KAT_TOL)
    assert r.passed, str(r)
    r = check(name + "/att", aw, c["att"], KAT_TOL)
    assert r.passed, str(r)


def test_oracle_mask_pattern(kat):
    """Masked keys get weight exactly 0 and keys above the diagonal -inf
    (attn.rs:187 initialises scores to -inf; :233 zeroes masked ones)."""
    c = kat["kat_mask"]
    _, aw, _ = oracle.attn_forward(c["w"], c["x"], want_att_w=True)
    exp = c["att"]
    assert np.array_equal(aw == 0.0, exp == 0.0)
    assert np.array_equal(np.isneginf(aw), np.isneginf(exp))


def test_oracle_decode_equals_prefill_last_row(kat):
    """forward_one after prefill(T) == prefill(T+1) last row (kv_cache.rs)."""
    c = kat["kat_decode"]
    x = c["x"]
    T = x.shape[0] - 1
    y_full, st_full = oracle.kv_prefill(c["w"], x, cap=T + 1)
    y_pre, st = oracle.kv_prefill(c["w"], x[:T], cap=T + 1)
    y_dec = oracle.kv_decode(c["w"], x[T], st)
    assert np.array_equal(y_pre, y_full[:T])
    assert np.array_equal(y_dec, y_full[T])
    assert st.n_cached == T + 1
    assert np.array_equal(st.phases, st_full.phases)
    assert np.array_equal(st.values, st_full.values)
    r = check("kat_decode/y", y_full, c["y"], KAT_TOL)
    assert r.passed, str(r)


def test_oracle_threads_do_not_change_results():
    w, _ = oracle.init_block_attn(42, 4, 32, 16)
    x = np.random.default_rng(0).standard_normal((40, 32)).astype(np.float32)
    y1, a1, p1 = oracle.attn_forward(w, x, want_att_w=True, n_threads=1)
    y4, a4, p4 = oracle.attn_forward(w, x, want_att_w=True, n_threads=4)
    assert np.array_equal(y1, y4) and np.array_equal(a1, a4) and np.array_equal(p1, p4)
    yb = oracle.attn_forward_batch(w, np.stack([x, x[::-1].copy()]), n_threads=3)
    assert np.array_equal(yb[0], y1)
    assert np.array_equal(yb[1], oracle.attn_forward(w, x[::-1].copy())[0])


def test_oracle_phase_override_reproduces_own_phases():
    w, _ = oracle.init_block_attn(7, 2, 16, 16)
    x = np.random.default_rng(1).standard_normal((20, 16)).astype(np.float32)
    y, aw, ph = oracle.attn_forward(w, x, want_att_w=True)
    y2, aw2, _ = oracle.attn_forward(w, x, want_att_w=True, phase_override=ph)
    assert np.array_equal(y, y2) and np.array_equal(aw, aw2)


def test_oracle_bucket_function_edges():
    tau = np.float32(6.2831855)
    w = tau / np.float32(8)
    # +pi lands in bucket 3, not 4: fmodf(pi, tau) + tau rounds 3*pi down in
    # f32, so the normalised phase is just below pi (kv_cache.rs:68).
    cases = {0.0: 0, -0.0: 0, float(np.float32(np.pi)): 3, float(-np.float32(np.pi)): 4,
             float(w * np.float32(0.999)): 0, float(w * np.float32(1.001)): 1,
             float(np.float32(-1e-6)): 7, float(np.nextafter(np.float32(0), np.float32(-1))): 0, float("nan"): 0}
    for th, b in cases.items():
        assert oracle.phase_to_bucket(th) == b, (th, oracle.phase_to_bucket(th), b)
    grid = np.random.default_rng(3).uniform(-np.pi, np.pi, 20000).astype(np.float32)
    assert np.array_equal(oracle.phase_to_bucket(grid), buckets_of(grid))


def test_oracle_softplus_and_harmonic_init():
    # math/core.rs:5 and wave_model.rs:73: n_h = softplus(ln((h+1)/2)) = ln(1 + (h+1)/2)
    for h in range(12):
        raw = np.float32(np.log(np.float32((h + 1) * 0.5)))
        assert abs(oracle.softplus(float(raw)) - np.log1p((h + 1) / 2)) < 1e-6
    assert oracle.softplus(25.0) == 25.0


def test_oracle_init_block_attn_draw_order():
    """init_linear draws U(+-1/sqrt(in)) row by row (wave_model.rs:39-46) in
    init_block_attn order (wave_model.rs:64-80); check the first draws by
    restating xorshift64 (rng.rs:24-39) in Python."""
    def xs(s):
        s ^= (s << 13) & 0xFFFFFFFFFFFFFFFF
        s ^= s >> 7
        s ^= (s << 17) & 0xFFFFFFFFFFFFFFFF
        return s
    s = 1234
    draws = []
    for _ in range(3):
        s = xs(s)
        f = np.float32(s >> 40) / np.float32(1 << 24)
        draws.append((f * np.float32(2) - np.float32(1)) * (np.float32(1) / np.sqrt(np.float32(32))))
    w, _ = oracle.init_block_attn(1234, 4, 32, 16)
    assert np.array_equal(w["phase_proj_w"][0, 0, :3], np.array(draws, np.float32))
    assert np.all(np.abs(w["out_proj_w"]) <= 1 / np.sqrt(32) + 1e-7)
    assert np.all(w["phase_proj_b"] == 0) and np.all(w["out_proj_b"] == 0)


# ---- seeded oracle dumps of the benchmark configurations at reduced size
# (tests/golden/configs.npz, written by tests/golden/make_config_golden.py)

def _configs():
    from pathlib import Path
    return np.load(Path(__file__).resolve().parent / "golden" / "configs.npz")


def _sha(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("case", ["cfg1_168", "cfg2_384", "cfg3_768", "cfg5_4096"])
def test_oracle_reproduces_config_fixture(case):
    """The oracle recomputes the committed prefill dump bit for bit (a change
    of the oracle's arithmetic or of the seeded inputs shows up here)."""
    from tests.golden import config_cases as cc
    fx = _configs()
    name, E, H, C, B, T, init, seed = next(c for c in cc.PREFILL if c[0] == case)
    w = cc.weights(init, seed, H, E, C)
    x = cc.inputs(seed, B, T, E)
    for b in range(B):
        y, _, ph = oracle.attn_forward(w, x[b])
        assert np.array_equal(y, fx[case + "/y"][b])
        assert np.array_equal(ph, fx[case + "/phases"][b])
    assert _sha(fx[case + "/y"]) == str(fx[case + "/y.sha256"])


@pytest.mark.parametrize("case", ["cfg3_decode", "cfg4_ragged"])
def test_oracle_reproduces_decode_fixture(case):
    from tests.golden import config_cases as cc
    fx = _configs()
    name, E, H, lens, steps, seed = next(c for c in cc.DECODE if c[0] == case)
    w = cc.weights("gauss", seed, H, E, 0)
    x = cc.inputs(seed, len(lens), max(lens) + steps, E)
    for b, n in enumerate(lens):
        _, st = oracle.kv_prefill(w, x[b, :n], cap=n + steps)
        for s in range(steps):
            assert np.array_equal(oracle.kv_decode(w, x[b, n + s], st), fx[case + "/y"][s, b])
    assert _sha(fx[case + "/y"]) == str(fx[case + "/y.sha256"])


# ---------------------------------------------------------------------------
# legacy dot-product attention (compute.rs:357-414)
# ---------------------------------------------------------------------------
def _dot_attn_f64(w, x):
    """Float64 statement of attention_cpu (compute.rs:357-414) for checking the oracle."""
    E = x.shape[1]
    H = w["n_head"]
    hd = E // H
    T = x.shape[0]
    qkv = x.astype(np.float64) @ w["c_attn_w"].T.astype(np.float64) + w["c_attn_b"]
    q, k, v = qkv[:, :E], qkv[:, E:2 * E], qkv[:, 2 * E:]
    o = np.zeros((T, E))
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        s = q[:, sl] @ k[:, sl].T / np.sqrt(hd)
        s[np.triu_indices(T, 1)] = -np.inf
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        o[:, sl] = p @ v[:, sl]
    return o @ w["c_proj_w"].T.astype(np.float64) + w["c_proj_b"]


def test_dot_attention_oracle_known_answers():
    """T = 1: the one key has weight 1, so y = c_proj(v) with v = c_attn's v
    rows; identical positions: every query averages identical values, so
    every output row equals the first; and a random case against float64."""
    import wave_engine_b200 as wb
    w = wb.gaussian_attention_weights(11, 4, 32, bias_std=0.1).packed()
    x1 = np.random.default_rng(0).standard_normal((1, 32)).astype(np.float32)
    v = (x1.astype(np.float64) @ w["c_attn_w"][64:].T + w["c_attn_b"][64:])
    y_kat = v @ w["c_proj_w"].T.astype(np.float64) + w["c_proj_b"]
    r = check("t1", oracle.dot_attn_forward(w, x1), y_kat, KAT_TOL)
    assert r.passed, str(r)
    xs = np.repeat(x1, 7, axis=0)
    ys = oracle.dot_attn_forward(w, xs)
    r = check("same rows", ys, np.repeat(ys[:1], 7, axis=0), (1e-6, 0.0))
    assert r.passed, str(r)
    x = np.random.default_rng(1).standard_normal((23, 32)).astype(np.float32)
    r = check("random", oracle.dot_attn_forward(w, x), _dot_attn_f64(w, x), (1e-5, 0.0))
    assert r.passed, str(r)
