"""Host-buffer calls (the reference's shape: Vec<f32> in, Vec<f32> out)
against the same calls on device tensors.

Host x / y go through the library's own staging: prefill and the
uncached forward run in sequence chunks whose copies overlap the compute
(several chunks at these sizes: 2 MB per chunk minimum, 786 KB per
sequence), decode uploads a seq-id list only when it changes, and a decode
with pinned host y (fewer than 64 rows) stores y from the out_proj kernel
directly.  Per-row math is identical in every mode, so results must be
bit-identical to the device-tensor run."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _modes():
    import torch
    return {
        "device": lambda a: torch.from_numpy(a).cuda(),
        "pageable": lambda a: a.copy(),
        "pinned": lambda a: torch.from_numpy(a).pin_memory(),
    }


def _np(t):
    import torch
    if isinstance(t, torch.Tensor):
        torch.cuda.synchronize()
        return t.cpu().numpy()
    return t


def test_forward_host_chunks_equal_device(ctx):
    import wave_engine_b200 as wb
    E, H, B, T = 768, 12, 8, 256
    w = wb.gaussian_block_attn(5, H, E, 16)
    x = np.random.default_rng(1).standard_normal((B, T, E)).astype(np.float32)
    outs = {}
    for name, mk in _modes().items():
        y, _, _ = wb.wave_attention_forward(w, mk(x), E // 2, ctx=ctx)
        outs[name] = _np(y)
    assert np.isfinite(outs["device"]).all()
    for name in ("pageable", "pinned"):
        assert np.array_equal(outs[name], outs["device"]), name
    assert ctx.take_device_error() == 0


@pytest.mark.parametrize("path", ["tensor", "exact"])
def test_kv_host_buffers_equal_device(ctx, path):
    import torch
    import wave_engine_b200 as wb
    E, H, B, T, steps = 768, 12, 8, 256, 4
    w = wb.gaussian_block_attn(9, H, E, 16)
    g = np.random.default_rng(2)
    x = g.standard_normal((B, T, E)).astype(np.float32)
    xs = g.standard_normal((steps, B, E)).astype(np.float32)
    ids = np.array([5, 0, 7, 2, 1, 6, 3, 4], np.int32)
    cache = wb.KvCache(1, H, E // H, max_seqs=8, max_ctx=T + 2 * steps + 2, ctx=ctx)
    res = {}
    for name, mk in _modes().items():
        cache.reset()
        yp = cache.prefill(0, w, mk(x), ids, path=path)
        dec = []
        for s in range(steps):
            # the full list, then one sequence (the reference's shape), then
            # the full list again: the id upload follows each change
            y = mk(np.zeros((B, E), np.float32))
            cache.forward_one(0, w, mk(xs[s]), ids, path=path, out=y)
            dec.append(_np(y).copy())
            y1 = mk(np.zeros((1, E), np.float32))
            cache.forward_one(0, w, mk(xs[s, 3:4]), ids[3:4], path=path, out=y1)
            dec.append(_np(y1).copy())
        res[name] = (_np(yp), dec)
        torch.cuda.synchronize()
    ref_p, ref_d = res["device"]
    assert np.isfinite(ref_p).all()
    for name in ("pageable", "pinned"):
        assert np.array_equal(res[name][0], ref_p), f"{name} prefill"
        for i, (a, b) in enumerate(zip(res[name][1], ref_d)):
            assert np.array_equal(a, b), f"{name} decode call {i}"
    assert ctx.take_device_error() == 0
