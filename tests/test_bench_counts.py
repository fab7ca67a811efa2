"""The algorithmic counts behind bench.py's roofline numbers, checked on CPU
against direct enumeration of the wave mask (attn.rs:185-220 for prefill,
kv_cache.rs:285-298 for decode): a key is scored when its bucket is the
query's or adjacent (mod 8) or when it is the previous position."""
from __future__ import annotations

import numpy as np


def _kept(bq: int, bk: int, k: int, q: int) -> bool:
    return ((bk - bq) % 8) in (0, 1, 7) or k == q - 1


def test_prefill_unmasked_pairs_matches_enumeration():
    import bench
    rng = np.random.default_rng(3)
    bk = rng.integers(0, 8, (2, 3, 2, 41)).astype(np.uint8)
    T = 37
    unmasked, dense = bench.prefill_unmasked_pairs(bk, T)
    count = 0
    for l, b, h in np.ndindex(2, 3, 2):
        for q in range(T):
            for k in range(q + 1):
                count += _kept(int(bk[l, b, h, q]), int(bk[l, b, h, k]), k, q)
    assert unmasked == count
    assert dense == 2 * 3 * 2 * T * (T + 1) // 2


def test_decode_bytes_exact_matches_enumeration():
    """Decode step p reads the phase + bucket (5 B) of every cached key and the
    fp32 value row (4*hd B) of every kept key; the new position itself is the
    self term, not a cached key."""
    import bench
    rng = np.random.default_rng(4)
    T0, S, hd = 19, 6, 8
    bk = rng.integers(0, 8, (2, 2, 3, T0 + S)).astype(np.uint8)
    for first in (0, 2):
        byts, unmasked, keys = bench.decode_bytes_exact(bk, T0, S, 3, hd, first=first)
        kept = total = 0
        for l, b, h in np.ndindex(2, 2, 3):
            for p in range(T0 + first, T0 + S):
                total += p
                kept += sum(_kept(int(bk[l, b, h, p]), int(bk[l, b, h, k]), k, p) for k in range(p))
        assert (unmasked, keys) == (kept, total)
        assert byts == 5 * total + 4 * hd * kept


def test_flop_formulas_match_the_configuration_table():
    """The attention kernel is credited only with its own work, 2*P*(2+C+hd)
    over the dense causal pairs; the whole layer adds the projections and
    out_proj.  Figures of the 768-dim configuration (B 32, T 1024, 12 x 64,
    C 16): 33.05 GFLOP of pairs inside 85.8 GFLOP per layer."""
    import bench
    core = bench.attn_core_flops(32, 1024, 12, 64, 16)
    layer = bench.prefill_flops_per_layer(32, 1024, 768, 12, 64, 16)
    assert core == 32 * 12 * 1024 * 1025 // 2 * 2 * (2 + 16 + 64)
    assert abs(core / 1e9 - 33.05) < 0.01
    assert abs(layer / 1e9 - 85.8) < 0.1
    assert layer - core == 2 * 32 * 1024 * 768 * (12 * 18 + 64 + 768)
