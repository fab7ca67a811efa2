"""wb_kv_decode_noalloc: the decode step that allocates no device memory.

Some callers cannot allocate at decode time -- a server that reserves all
of its device memory when it starts and forbids allocation per request, a
host application whose own memory pool owns the device, or a latency-bound
loop that cannot take cudaMalloc's implicit synchronisation.  For them the
library keeps the decode kernels' scratch in one static device array
(WB_NOALLOC_SCRATCH_BYTES per GPU).  These tests call
that entry point through the C ABI and check it against the ordinary
wb_kv_decode on a twin cache, for two decode calls in a row.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.  It creates its own context, so
it passes alone in a fresh process as well as after the other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from tests.parity import TENSOR_TOL, check

pytestmark = pytest.mark.gpu

H, HD, E, SLOTS, CAP, N0 = 12, 64, 768, 8, 1400, 1100


def _twin_caches(ctx, w, rng):
    import wave_engine_b200 as wb
    caches = [wb.KvCache(1, H, HD, max_seqs=SLOTS, max_ctx=CAP, ctx=ctx) for _ in range(2)]
    for s in range(SLOTS):
        n = N0 - 37 * s
        ph = np.arctan2(rng.standard_normal((H, n)), rng.standard_normal((H, n))).astype(np.float32)
        vv = rng.standard_normal((H, n, HD)).astype(np.float32)
        for c in caches:
            c.load(0, s, ph, vv)
    return caches


def test_noalloc_decode_matches_wb_kv_decode_twice():
    import torch
    import wave_engine_b200 as wb
    from wave_engine_b200 import _lib

    ctx = wb.Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    w = wb.gaussian_block_attn(21, H, E, 16)
    layer = wb.AttnLayer(ctx, w)
    rng = np.random.default_rng(5)
    ref_cache, na_cache = _twin_caches(ctx, w, rng)
    ids = torch.tensor([5, 0, 3, 7, 2], dtype=torch.int32, device="cuda")
    n0 = {int(s): na_cache.n_cached(0, int(s)) for s in ids.tolist()}
    torch.cuda.synchronize()
    free_after_first = None
    for step in range(2):
        x = torch.from_numpy(rng.standard_normal((ids.numel(), E)).astype(np.float32)).cuda()
        y_ref = torch.empty_like(x)
        y_na = torch.full_like(x, float("nan"))
        ref_cache.forward_one(0, layer, x, ids, out=y_ref)
        _lib.call("wb_kv_decode_noalloc", ctx.handle, na_cache.handle, 0, layer.handle, ids.data_ptr(),
                  ids.numel(), x.data_ptr(), y_na.data_ptr())
        torch.cuda.synchronize()
        r = check(f"noalloc decode step {step}", y_na.cpu().numpy(), y_ref.cpu().numpy(), TENSOR_TOL)
        assert r.passed, str(r)
        if step == 0:
            free_after_first = torch.cuda.mem_get_info()[0]
    # the second call allocated nothing on the device
    assert torch.cuda.mem_get_info()[0] == free_after_first
    for s in ids.tolist():
        assert na_cache.n_cached(0, s) == n0[s] + 2
        ph_a, bk_a, v_a = na_cache.read(0, s)
        ph_b, bk_b, v_b = ref_cache.read(0, s)
        assert np.array_equal(bk_a, bk_b) and np.allclose(v_a, v_b, atol=1e-6) and np.allclose(ph_a, ph_b, atol=1e-6)
    assert ctx.take_device_error() == 0
    ctx.close()


def test_noalloc_decode_rejects_oversize_and_host_buffers():
    import torch
    import wave_engine_b200 as wb
    from wave_engine_b200 import _lib

    ctx = wb.Context(0)
    w = wb.gaussian_block_attn(3, 1, 64, 0)
    layer = wb.AttnLayer(ctx, w)
    # 8192 one-position slots: a ~2 MB cache whose decode scratch (~6.4 MB:
    # the partial row, new value and output row of every slot) exceeds 4 MiB
    big = wb.KvCache(1, 1, 64, max_seqs=8192, max_ctx=1, ctx=ctx)
    ids = torch.zeros(1, dtype=torch.int32, device="cuda")
    x = torch.zeros((1, 64), device="cuda")
    y = torch.zeros((1, 64), device="cuda")
    rc = _lib.lib().wb_kv_decode_noalloc(ctx.handle, big.handle, 0, layer.handle, ids.data_ptr(), 1,
                                         x.data_ptr(), y.data_ptr())
    assert rc == _lib.WB_EINVAL
    assert b"static limit" in _lib.lib().wb_last_error()
    small = wb.KvCache(1, 1, 64, max_seqs=2, max_ctx=16, ctx=ctx)
    xh = np.zeros((1, 64), np.float32)
    rc = _lib.lib().wb_kv_decode_noalloc(ctx.handle, small.handle, 0, layer.handle, ids.data_ptr(), 1,
                                         xh.ctypes.data, y.data_ptr())
    assert rc == _lib.WB_EINVAL
    assert b"device pointers" in _lib.lib().wb_last_error()
    ctx.close()
