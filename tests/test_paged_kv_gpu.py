"""Paged KV cache (wb_kv_cache_create_paged): the same prefill and decode
calls as on a contiguous cache give bit-identical outputs and cache
contents, with each sequence's pages scattered over the pool; reservation
and release keep the pool's accounting; positions past a slot's reserved
pages are refused (host ids) or flagged and skipped (device ids)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(ctx, w, x_pre, x_dec, ids, path, paged, max_ctx, reserve_order=None):
    import wave_engine_b200 as wb
    n_seq, T, E = x_pre.shape
    H = w.n_head
    kw = {"n_pages": 64} if paged else {}
    cache = wb.KvCache(2, H, E // H, max_seqs=6, max_ctx=max_ctx, ctx=ctx, **kw)
    if paged:
        # interleaved reservations: every sequence's pages are scattered
        for seq, n in reserve_order:
            cache.reserve(seq, n)
    outs = []
    for layer in range(2):
        outs.append(cache.prefill(layer, w, x_pre + layer, ids, path=path))
    for s in range(x_dec.shape[0]):
        for layer in range(2):
            outs.append(cache.forward_one(layer, w, x_dec[s] - layer, ids, path=path))
    contents = [cache.read(layer, int(i)) for layer in range(2) for i in ids]
    return cache, outs, contents


@pytest.mark.parametrize("path", ["tensor", "exact"])
@pytest.mark.parametrize("T,steps,max_ctx", [(200, 60, 300), (1600, 3, 1700)])
def test_paged_equals_contiguous(ctx, path, T, steps, max_ctx):
    import wave_engine_b200 as wb
    E, H = 768, 12
    w = wb.gaussian_block_attn(21, H, E, 0)
    g = np.random.default_rng(T)
    ids = np.array([4, 1, 3], np.int32)
    x_pre = g.standard_normal((3, T, E)).astype(np.float32)
    x_dec = g.standard_normal((steps, 3, E)).astype(np.float32)
    order = []
    for n in range(128, T + steps + 128, 128):
        for seq in (1, 3, 4):
            order.append((seq, min(n, T + steps)))
    _, ref, ref_c = _run(ctx, w, x_pre, x_dec, ids, path, False, max_ctx)
    cache, got, got_c = _run(ctx, w, x_pre, x_dec, ids, path, True, max_ctx, order)
    for i, (a, b) in enumerate(zip(got, ref)):
        assert np.array_equal(a, b), f"output {i}"
    for a, b in zip(got_c, ref_c):
        for u, v in zip(a, b):
            assert np.array_equal(u, v)
    assert ctx.take_device_error() == 0
    used = sum(-(-(T + steps) // 128) for _ in range(3))
    assert cache.free_pages() == 64 - used
    for seq in (1, 3, 4):
        cache.release(seq)
    assert cache.free_pages() == 64
    assert cache.n_cached(0, 1) == 0


def test_paged_reservation_limits(ctx):
    import torch
    import wave_engine_b200 as wb
    E, H = 256, 4
    w = wb.gaussian_block_attn(3, H, E, 0)
    cache = wb.KvCache(1, H, E // H, max_seqs=3, max_ctx=512, ctx=ctx, n_pages=5)
    g = np.random.default_rng(0)
    x = g.standard_normal((1, 130, E)).astype(np.float32)
    with pytest.raises(wb.WaveB200Error):
        cache.prefill(0, w, x, [0])                 # nothing reserved
    cache.reserve(0, 130)                            # 2 pages
    assert cache.free_pages() == 3
    with pytest.raises(wb.WaveB200Error):
        cache.reserve(1, 512)                        # needs 4, 3 free
    assert cache.free_pages() == 3
    with pytest.raises(wb.WaveB200Error):
        cache.reserve(1, 513)                        # beyond max_ctx
    cache.prefill(0, w, x, [0])
    for _ in range(126):                             # fills the 2 pages: 256 positions
        cache.forward_one(0, w, g.standard_normal((1, E)).astype(np.float32), [0])
    assert cache.n_cached(0, 0) == 256
    with pytest.raises(wb.WaveB200Error):
        cache.forward_one(0, w, g.standard_normal((1, E)).astype(np.float32), [0])
    # device seq ids past the reservation: flagged, nothing appended
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = cache.forward_one(0, w, torch.randn(1, E, device="cuda"), ids)
    torch.cuda.synchronize()
    assert ctx.take_device_error() & 0x8
    assert cache.n_cached(0, 0) == 256
    assert np.isfinite(y.cpu().numpy()).all()
    cache.release(0)
    assert cache.free_pages() == 5 and cache.n_cached(0, 0) == 0
