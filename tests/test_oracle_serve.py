"""The serve-layer oracle (oracle/serve_oracle.c) against an independent
float64 statement of the same reference code: model.rs:154 layer_norm,
ffn.rs:39-230 (maestro, agc.rs process/observe, fft_ode.rs kerr_ode_fft
with its stencil -- circular over next_pow2(n_bands) points from 256 bands
on -- the corrector plate, out_proj.rs) and kv_cache.rs:18-33
phase_native_decode.  The float64 statement shares no code with the C one;
agreement to fp32 rounding pins the restatement's structure (term order,
indexing, the AGC's state machine), not the reference's last bits."""
from __future__ import annotations

import numpy as np
import pytest

import wave_engine_b200 as wb
from oracle import oracle


def _gelu(v):
    return 0.5 * v * (1.0 + np.tanh(0.7978845608 * (v + 0.044715 * v ** 3)))


def _softplus(x):
    return np.where(x > 20, x, np.log1p(np.exp(x)))


class _Agc64:
    def __init__(self, alpha=0.1, beta=0.1):
        c = max(np.sqrt(np.pi / 2 / (alpha + 4 * beta)), 0.5)
        self.mean, self.var, self.head, self.decay = 1.0, 0.5, 3.0, 0.995
        self.lo, self.hi, self.thr, self.count = max(c * 0.3, 0.5), c, max(c * 0.75, 0.5), 0

    def process(self, pre, nb):
        mags = np.sqrt(pre[:, 0::2] ** 2 + pre[:, 1::2] ** 2).ravel()
        clean = mags[np.isfinite(mags) & (mags < 2 * self.hi)]
        if clean.size:
            m, v = clean.mean(), ((clean - clean.mean()) ** 2).mean()
            self.count += 1
            if self.count < 10:
                self.mean, self.var = m, v
            else:
                self.mean = self.decay * self.mean + (1 - self.decay) * m
                self.var = self.decay * self.var + (1 - self.decay) * v
            self.thr = min(max(self.mean + self.head * max(np.sqrt(self.var), 0.01), self.lo), self.hi)
        out = pre.copy()
        r, s = out[:, 0::2], out[:, 1::2]
        mag = np.sqrt(r ** 2 + s ** 2)
        t = self.thr
        sel = (mag > t) & (mag > 0.001)
        scale = np.where(sel, (t + t * np.tanh((mag - t) / t)) / np.where(sel, mag, 1), 1.0)
        out[:, 0::2], out[:, 1::2] = r * scale, s * scale
        return out


def _ffn64(f, agc, x):
    E, nb = f["n_embd"], f["n_embd"] // 2
    lin = lambda w, b, v: v @ w.astype(np.float64).T + b
    pre = x + lin(f["mi_process_w"], f["mi_process_b"], _gelu(lin(f["mi_squeeze_w"], f["mi_squeeze_b"], x)))
    pre = agc.process(pre, nb)
    g = _softplus(f["gamma_raw"].astype(np.float64))
    om, a, b = f["omega"].astype(np.float64), f["alpha"], f["beta"]
    L = 0
    if nb >= 256:
        L = 1
        while L < nb:
            L <<= 1
    idx = np.arange(nb)

    def deriv(r, s):
        m = r * r + s * s
        ns = np.zeros_like(m)
        for off in (-2, -1, 1, 2):
            j = idx + off
            if L:
                j = j % L
            ok = (j >= 0) & (j < nb)
            ns[:, ok] += m[:, j[ok]]
        phi = om + a * m + b * ns
        return -g * r - phi * s, -g * s + phi * r

    r, s = pre[:, 0::2].copy(), pre[:, 1::2].copy()
    dt, w = 1.0 / f["rk4_steps"], f["rk4_weights"].astype(np.float64)
    for _ in range(f["rk4_steps"]):
        k1 = deriv(r, s)
        k2 = deriv(r + 0.5 * dt * k1[0], s + 0.5 * dt * k1[1])
        k3 = deriv(r + 0.5 * dt * k2[0], s + 0.5 * dt * k2[1])
        k4 = deriv(r + dt * k3[0], s + dt * k3[1])
        r = r + dt * (w[0] * k1[0] + w[1] * k2[0] + w[2] * k3[0] + w[3] * k4[0])
        s = s + dt * (w[0] * k1[1] + w[1] * k2[1] + w[2] * k3[1] + w[3] * k4[1])
    if f["use_corrector"]:
        c, sn = np.cos(f["phase_correction"]), np.sin(f["phase_correction"])
        r, s = r * c - s * sn, r * sn + s * c
    ko = np.empty_like(pre)
    ko[:, 0::2], ko[:, 1::2] = r, s
    reg = ko + lin(f["mo_process_w"], f["mo_process_b"], _gelu(lin(f["mo_squeeze_w"], f["mo_squeeze_b"], ko)))
    G = f["out_groups"]
    if G == 1:
        return lin(f["out_w"], f["out_b"], reg)
    gs, y, off = E // G, np.empty_like(reg), 0
    for gi in range(G):
        gw = f["out_w"][off:off + gs * gs].reshape(gs, gs)
        gb = f["out_w"][off + gs * gs:off + gs * gs + gs]
        y[:, gi * gs:(gi + 1) * gs] = lin(gw, gb, reg[:, gi * gs:(gi + 1) * gs])
        off += gs * gs + gs
    return y


@pytest.mark.parametrize("E,groups", [(168, 1), (512, 1), (768, 2)])
def test_ffn_oracle_matches_float64_statement(E, groups):
    f = wb.gaussian_ffn(E, E, 16, out_groups=groups, phase_correction_std=0.3).packed()
    g = np.random.default_rng(E)
    a32, a64 = oracle.agc_new(), _Agc64()
    for call in range(11):
        x = (g.standard_normal((4, E)) * 1.5).astype(np.float32)
        y = oracle.ffn_forward(f, a32, x)
        ref = _ffn64(f, a64, x.astype(np.float64))
        assert np.abs(y - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max()), call
    assert a32.count == a64.count == 11
    assert abs(a32.threshold - a64.thr) < 1e-5


def test_layer_norm_and_phase_native_decode_oracle():
    g = np.random.default_rng(3)
    x = (g.standard_normal((5, 768)) * 2 + 1).astype(np.float32)
    w, b = g.standard_normal(768).astype(np.float32), g.standard_normal(768).astype(np.float32)
    x64 = x.astype(np.float64)
    ref = (x64 - x64.mean(1, keepdims=True)) / np.sqrt(x64.var(1, keepdims=True) + 1e-5) * w + b
    assert np.abs(oracle.layer_norm(x, w, b) - ref).max() < 1e-4
    wte = g.standard_normal((50, 768)).astype(np.float32)
    corr = g.standard_normal(384).astype(np.float32)
    c, s = np.cos(corr.astype(np.float64)), np.sin(corr.astype(np.float64))
    h = x64[0]
    rot = np.empty(768)
    rot[0::2], rot[1::2] = h[0::2] * c - h[1::2] * s, h[0::2] * s + h[1::2] * c
    assert np.abs(oracle.phase_native_decode(x[0], corr, wte) - wte.astype(np.float64) @ rot).max() < 1e-3
    # prefill indexes wpe by the token id, decode by the position (kv_cache.rs:108-110, :254-256)
    wpe = g.standard_normal((10, 768)).astype(np.float32)
    e = oracle.embed(np.array([3, 40]), np.array([3, 40]), wte, wpe)
    assert np.array_equal(e[0], wte[3] + wpe[3]) and np.array_equal(e[1], wte[40])
