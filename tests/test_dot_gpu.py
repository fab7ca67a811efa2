"""GPU parity of the legacy dot-product attention (compute.rs:357-414,
ComputeBackend::attention) against the CPU oracle, through the C ABI.

Tolerances: WB_PATH_EXACT (sequential fp32 projections, fp32 attention core)
max-abs 1e-5; WB_PATH_TENSOR (TF32 tensor-core projections, fp32 core)
max-abs 2e-3."""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tests.parity import EXACT_TOL, TENSOR_TOL, check

pytestmark = pytest.mark.gpu

SHAPES = [
    # E, H, B, T
    (16, 2, 1, 1),      # T = 1: one key
    (168, 4, 2, 64),    # head_dim 42 (odd halves)
    (384, 8, 1, 129),   # head_dim 48, ragged T
    (768, 12, 2, 130),  # head_dim 64
    (256, 2, 1, 70),    # head_dim 128
]


@pytest.mark.parametrize("path,tol", [("exact", EXACT_TOL), ("tensor", TENSOR_TOL)])
@pytest.mark.parametrize("E,H,B,T", SHAPES)
def test_dot_attention_matches_oracle(ctx, path, tol, E, H, B, T):
    import wave_engine_b200 as wb
    w = wb.gaussian_attention_weights(E + T, H, E, bias_std=0.05)
    x = np.random.default_rng(E * 7 + T).standard_normal((B, T, E)).astype(np.float32)
    y = wb.attention(w, x, path=path, ctx=ctx)
    for b in range(B):
        r = check(f"{path} seq {b}", y[b], oracle.dot_attn_forward(w.packed(), x[b]), tol)
        assert r.passed, str(r)
    assert ctx.take_device_error() == 0


def test_dot_attention_torch_inputs_and_errors(ctx):
    import torch
    import wave_engine_b200 as wb
    w = wb.gaussian_attention_weights(3, 4, 64, bias_std=0.05)
    x = np.random.default_rng(2).standard_normal((40, 64)).astype(np.float32)
    y_np = wb.attention(w, x, ctx=ctx)
    y_t = wb.attention(w, torch.from_numpy(x).cuda(), ctx=ctx)
    torch.cuda.synchronize()
    assert y_t.is_cuda and np.array_equal(y_t.cpu().numpy(), y_np)
    with pytest.raises(ValueError):
        wb.attention(w, x[:, :32], ctx=ctx)  # weights for another n_embd
    with pytest.raises(wb.WaveB200Error):
        wb.DotAttnLayer(ctx, wb.gaussian_attention_weights(1, 1, 132))  # head_dim 132 > 128
