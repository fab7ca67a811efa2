"""Generate the known-answer fixtures ``tests/golden/kat.npz``.

The reference (Rust crate wave-engine) ships no golden vectors for the
attention forward and cannot be built here, so these cases pin the CPU
oracle with answers derived by hand from the reference's semantics
(src/common/attn.rs:90-305, src/common/kv_cache.rs:121-193/:263-335):

  kat_t1        T = 1: softmax over one key is [1], so y = W_out v + b.
  kat_uniform   every position has the same phase and content, so every
                causal key gets the same score and the weights are
                uniform 1/(q+1): y[q] = W_out mean(v[0..=q]) + b.
  kat_mask      phases placed in buckets 0,4,0,4,2,6: a query sees only
                keys in its own or an adjacent bucket plus the previous
                position (attn.rs:212-221), every other key is masked.
  kat_decode    forward_one after a prefill of the same prompt equals the
                prefill of the longer prompt at its last row (kv_cache.rs
                scores self as 1.0 = cos(0) and appends in order).

Expected outputs are computed here in float64 with explicit index sets
(not with the oracle), then stored as float32.  Run:
    python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "kat.npz"
TAU = 2 * np.pi


def softplus(x):
    return x if x > 20 else np.log1p(np.exp(x))


def bucket_of(theta):
    t = np.mod(np.mod(theta, TAU) + TAU, TAU)
    return min(int(t / (TAU / 8)), 7)


def base_weights(E, H, C, rng):
    d = E // H
    w = {
        "harmonic_raw": np.log((np.arange(H) + 1) * 0.5).astype(np.float32),
        "phase_proj_w": np.zeros((H, 2, E), np.float32),
        "phase_proj_b": np.zeros((H, 2), np.float32),
        "v_proj_w": (rng.standard_normal((H, d, d)) * 0.3).astype(np.float32),
        "v_proj_b": (rng.standard_normal((H, d)) * 0.1).astype(np.float32),
        "content_proj_w": np.zeros((H, C, E), np.float32) if C else None,
        "content_proj_b": (rng.standard_normal((H, C)) * 0.5).astype(np.float32) if C else None,
        "out_proj_w": (rng.standard_normal((E, E)) * 0.3).astype(np.float32),
        "out_proj_b": (rng.standard_normal(E) * 0.1).astype(np.float32),
    }
    # r = x[0], s = x[1] for every head: theta = atan2(x1, x0).
    w["phase_proj_w"][:, 0, 0] = 1.0
    w["phase_proj_w"][:, 1, 1] = 1.0
    return w


def values64(w, x):
    """v[h][t][d] = Wv x_h + b in float64."""
    H, d, _ = w["v_proj_w"].shape
    T = x.shape[0]
    v = np.zeros((H, T, d))
    for h in range(H):
        xs = x[:, h * d:(h + 1) * d].astype(np.float64)
        v[h] = xs @ w["v_proj_w"][h].astype(np.float64).T + w["v_proj_b"][h]
    return v


def attention64(w, x, allowed_fn, use_content=True):
    """float64 attention with an explicit allowed-key predicate."""
    H = w["harmonic_raw"].shape[0]
    T, E = x.shape
    d = E // H
    v = values64(w, x)
    x64 = x.astype(np.float64)
    theta = np.arctan2(x64[:, 1], x64[:, 0])
    out = np.zeros((T, E))
    att = np.full((H, T, T), -np.inf)
    for h in range(H):
        n = softplus(float(w["harmonic_raw"][h]))
        c = None
        if use_content and w["content_proj_w"] is not None:
            c = x64 @ w["content_proj_w"][h].astype(np.float64).T + w["content_proj_b"][h]
        for q in range(T):
            s = np.full(q + 1, -np.inf)
            for k in range(q + 1):
                if allowed_fn(q, k, theta):
                    s[k] = np.cos(n * (theta[q] - theta[k]))
                    if c is not None:
                        s[k] += 0.25 * float(c[q] @ c[k])
            p = np.where(np.isfinite(s), np.exp(s - s.max()), 0.0)
            p /= p.sum()
            att[h, q, :q + 1] = p
            out[q, h * d:(h + 1) * d] = p @ v[h, :q + 1]
    y = out @ w["out_proj_w"].astype(np.float64).T + w["out_proj_b"]
    return y, att


def bucket_rule(q, k, theta):
    bq, bk = bucket_of(theta[q]), bucket_of(theta[k])
    return ((bk - bq) % 8 in (0, 1, 7)) or k == q - 1


def main():
    rng = np.random.default_rng(20261201)
    E, H, C = 8, 2, 16
    cases = {}

    # kat_t1
    w = base_weights(E, H, C, rng)
    x = rng.standard_normal((1, E)).astype(np.float32)
    v = values64(w, x)
    merged = np.concatenate([v[h, 0] for h in range(H)])
    y = merged @ w["out_proj_w"].astype(np.float64).T + w["out_proj_b"]
    cases["kat_t1"] = (w, x, y[None, :], np.ones((H, 1, 1)))

    # kat_uniform: x[:,0:2] fixed (same phase), content weights zero (same content)
    w = base_weights(E, H, C, rng)
    T = 6
    x = rng.standard_normal((T, E)).astype(np.float32)
    x[:, 0], x[:, 1] = 0.8, 0.3
    v = values64(w, x)
    out = np.zeros((T, E))
    for q in range(T):
        for h in range(H):
            out[q, h * (E // H):(h + 1) * (E // H)] = v[h, :q + 1].mean(axis=0)
    y = out @ w["out_proj_w"].astype(np.float64).T + w["out_proj_b"]
    att = np.full((H, T, T), -np.inf)
    for q in range(T):
        att[:, q, :q + 1] = 1.0 / (q + 1)
    cases["kat_uniform"] = (w, x, y, att)

    # kat_mask: bucket centres 0,4,0,4,2,6 (bucket b centre = (b + 0.5) * tau/8)
    w = base_weights(E, H, C, rng)
    w["content_proj_w"][:] = (rng.standard_normal(w["content_proj_w"].shape) * 0.2).astype(np.float32)
    bks = [0, 4, 0, 4, 2, 6]
    T = len(bks)
    x = rng.standard_normal((T, E)).astype(np.float32)
    for t, b in enumerate(bks):
        phi = (b + 0.5) * TAU / 8
        phi = phi if phi <= np.pi else phi - TAU
        x[t, 0], x[t, 1] = np.cos(phi) * 1.3, np.sin(phi) * 1.3
    y, att = attention64(w, x, bucket_rule)
    cases["kat_mask"] = (w, x, y, att)

    # kat_decode (no content, as kv_cache.rs): prefill T then one decode step
    w = base_weights(E, H, C, rng)
    w["content_proj_w"] = w["content_proj_b"] = None
    T = 7
    x = rng.standard_normal((T + 1, E)).astype(np.float32)
    y, att = attention64(w, x, bucket_rule, use_content=False)
    cases["kat_decode"] = (w, x, y, att)

    arrays = {}
    for name, (w, x, y, att) in cases.items():
        for k, a in w.items():
            if a is not None:
                arrays[f"{name}/w/{k}"] = a
        arrays[f"{name}/x"] = x.astype(np.float32)
        arrays[f"{name}/y"] = y.astype(np.float32)
        arrays[f"{name}/att"] = att.astype(np.float32)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({len(cases)} cases)")


if __name__ == "__main__":
    main()
