"""The tcgen05 bf16 GEMM behind out_proj, against torch in fp32."""
from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


# fewer than 148 tiles of 128 x 128 take the 128 x 32 tiles; (2048, 1536, 512)
# and (4096, 768, 768) are 192 wide tiles
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 768, 768), (300, 168, 168), (1000, 384, 384),
                                   (129, 4096, 4096), (2048, 1536, 512)])
def test_gemm_bf16_matches_torch(ctx, M, N, K):
    import torch
    from wave_engine_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    B = torch.randn(N, K, device="cuda", generator=g).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda", generator=g)
    C = torch.full((M, N), float("nan"), device="cuda")
    torch.cuda.synchronize()
    _lib.call("wb_test_gemm_bf16", ctx.handle, A.data_ptr(), B.data_ptr(), bias.data_ptr(), C.data_ptr(), M, N, K)
    ctx.synchronize()
    ref = A.float() @ B.float().T + bias
    err = (C - ref).abs().max().item()
    assert err <= 1e-3 * max(1.0, K ** 0.5), err
    assert ctx.take_device_error() == 0


@pytest.mark.parametrize("M,N,K", [(128, 128, 32), (300, 4096, 4096), (1000, 1536, 1536), (4096, 768, 768),
                                   (256, 720, 768)])
def test_gemm_tf32_matches_torch(ctx, M, N, K):
    import torch
    from wave_engine_b200 import _lib
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g)
    B = torch.randn(N, K, device="cuda", generator=g)
    bias = torch.randn(N, device="cuda", generator=g)
    C = torch.full((M, N), float("nan"), device="cuda")
    torch.cuda.synchronize()
    _lib.call("wb_test_gemm_tf32", ctx.handle, A.data_ptr(), B.data_ptr(), bias.data_ptr(), C.data_ptr(), M, N, K)
    ctx.synchronize()
    ref = A.double() @ B.double().T + bias.double()
    d = C.double() - ref
    # tf32 keeps 10 explicit mantissa bits (unit roundoff 2^-11): the relative
    # RMS error of a random dot product is ~1e-3; an operand layout error
    # would give O(1).
    rel_rms = (d.pow(2).mean().sqrt() / ref.pow(2).mean().sqrt()).item()
    assert rel_rms <= 3e-3, rel_rms
    assert d.abs().max().item() <= 8 * 3e-3 * ref.pow(2).mean().sqrt().item()
    assert ctx.take_device_error() == 0
