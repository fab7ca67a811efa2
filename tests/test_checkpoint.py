"""WCHK checkpoint interop (src/common/checkpoint.rs, flatten_params_ex at
src/common/wave_model.rs:335-399): files written here in the reference's
byte layout -- the writer below follows save_checkpoint (checkpoint.rs:20-87)
field by field, with every non-attention parameter random so an offset
error cannot go unnoticed -- must give back the attention weights exactly."""
from __future__ import annotations

import struct

import numpy as np
import pytest

import wave_engine_b200 as wb
from wave_engine_b200.checkpoint import (FLAG_DYN_HARMONICS, FLAG_LEARNABLE_ATTN, FLAG_LEARNABLE_ODE,
                                         FLAG_RK4_WEIGHTS, load_wchk_attention, read_wchk_header)


def _flatten(blocks, g, E, M, groups, flags, n_bands, content_dim, tail):
    """flatten_params_ex for attention blocks `blocks` (WaveAttnWeights),
    random everything else; `tail` extra model-level floats at the end."""
    out = []
    r = lambda *s: g.standard_normal(s).astype(np.float32).ravel()
    gs = E // groups
    for w in blocks:
        p = w.packed()
        out += [r(E), r(E), r(E), r(E)]                      # ln, ln_ffn
        for _ in range(2):                                   # maestro_in, maestro_out
            out += [r(M, E), r(M), r(E, M), r(E)]
        for _ in range(groups):                              # ffn out_proj
            out += [r(gs, gs), r(gs)]
        if flags & FLAG_LEARNABLE_ODE:
            out += [r(n_bands), r(1), r(1), r(n_bands)]
            if flags & FLAG_RK4_WEIGHTS:
                out += [r(4)]
        if flags & FLAG_DYN_HARMONICS:
            out += [p["harmonic_raw"]]
        for h in range(w.n_head):
            out += [p["phase_proj_w"][h].ravel(), p["phase_proj_b"][h], p["v_proj_w"][h].ravel(), p["v_proj_b"][h]]
            if content_dim:
                out += [p["content_proj_w"][h].ravel(), p["content_proj_b"][h]]
        out += [p["out_proj_w"].ravel(), p["out_proj_b"]]
    out += [r(tail)]
    return np.concatenate(out).astype("<f4")


def _write(path, version, params, n_bands, n_head, n_layers, maestro, groups, flags):
    with open(path, "wb") as f:
        f.write(b"WCHK")
        f.write(struct.pack("<I", version))
        f.write(struct.pack("<6I", n_bands, n_head, n_layers, maestro, 64, 8))
        if version >= 2:
            f.write(struct.pack("<I", groups))
        if version >= 3:
            f.write(struct.pack("<I", flags))
        if version >= 4:
            f.write(struct.pack("<f", 0.25))
        f.write(struct.pack("<QQ", 50257, 1234))
        f.write(struct.pack("<f", 3e-4))
        f.write(struct.pack("<Q", 0xDEADBEEF))
        f.write(struct.pack("<Q", 77))
        n = params.size
        f.write(np.full(n, 0.5, "<f4").tobytes())   # Adam m
        f.write(np.full(n, 0.25, "<f4").tobytes())  # Adam v
        f.write(params.tobytes())


@pytest.mark.parametrize("version,flags,groups,content_dim", [
    (4, FLAG_LEARNABLE_ATTN | FLAG_LEARNABLE_ODE | FLAG_RK4_WEIGHTS | FLAG_DYN_HARMONICS, 1, 16),
    (4, FLAG_LEARNABLE_ATTN | FLAG_LEARNABLE_ODE, 4, 16),
    (3, FLAG_LEARNABLE_ATTN | FLAG_DYN_HARMONICS, 2, 0),     # --freeze-ode: no content projection
])
def test_wchk_attention_round_trip(tmp_path, version, flags, groups, content_dim):
    E, H, L, M = 64, 4, 3, 24
    g = np.random.default_rng(version * 10 + groups)
    blocks = [wb.init_block_attn(wb.Rng(100 + l), H, E, content_dim) for l in range(L)]
    if flags & FLAG_DYN_HARMONICS:
        for w in blocks:
            for hw in w.heads:
                hw.harmonic_raw = float(g.standard_normal())
    params = _flatten(blocks, g, E, M, groups, flags, E // 2, content_dim, tail=2 * E + E // 2)
    path = str(tmp_path / "model.wchk")
    _write(path, version, params, E // 2, H, L, M, groups, flags)
    h = read_wchk_header(path)
    assert (h.version, h.n_bands, h.n_head, h.n_layers, h.maestro_dim, h.out_proj_groups, h.flags) == \
        (version, E // 2, H, L, M, groups, flags)
    assert h.n_params == params.size and h.adam_t == 77 and h.vocab_size == 50257
    hdr, got = load_wchk_attention(path, content_dim=content_dim)
    assert len(got) == L
    for a, b in zip(got, blocks):
        pa, pb = a.packed(), b.packed()
        for k in pb:
            if pb[k] is None:
                assert pa[k] is None
            else:
                assert np.array_equal(pa[k], pb[k]), k


def test_wchk_defaults_and_errors(tmp_path):
    E, H, L, M = 32, 2, 2, 8
    g = np.random.default_rng(5)
    blocks = [wb.init_block_attn(wb.Rng(7 + l), H, E, 16) for l in range(L)]
    # legacy: learnable attention saved without bit 4 (checkpoint.rs:199-203)
    params = _flatten(blocks, g, E, M, 1, 0, E // 2, 16, tail=2 * E)
    path = str(tmp_path / "legacy.wchk")
    _write(path, 2, params, E // 2, H, L, M, 1, 0)
    with pytest.raises(ValueError):
        load_wchk_attention(path)                           # bit 4 unset
    _, got = load_wchk_attention(path, learnable_attn=True)
    for a, b in zip(got, blocks):
        assert np.array_equal(a.packed()["v_proj_w"], b.packed()["v_proj_w"])
        # no dynamic harmonics in the file: the initialiser's ln((h+1)/2)
        assert np.array_equal(a.packed()["harmonic_raw"], b.packed()["harmonic_raw"])
    with pytest.raises(ValueError):
        load_wchk_attention(path, content_dim=64, learnable_attn=True)  # does not fit the file
    bad = tmp_path / "bad.wchk"
    bad.write_bytes(b"WCHX" + bytes(100))
    with pytest.raises(ValueError):
        read_wchk_header(str(bad))
