"""CPU tests of the C ABI library: it loads without a GPU, exports every
symbol include/wave_b200.h declares, and its host-only entry points work.
No compute kernels are launched here."""
from __future__ import annotations

import ctypes as C
import re
import subprocess

import numpy as np
import pytest

from tests.conftest import ROOT

HEADER = ROOT / "include" / "wave_b200.h"


def declared_symbols():
    syms = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        syms |= set(re.findall(r"^WB_API\s+[\w\s\*]*?\b(wb_\w+)\s*\(", h.read_text(), flags=re.M))
    return sorted(syms)


def test_header_declares_the_boundary():
    syms = declared_symbols()
    for s in ("wb_attn_forward", "wb_kv_prefill", "wb_kv_decode", "wb_attn_layer_create", "wb_kv_cache_create",
              "wb_last_error", "wb_context_create"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    from wave_engine_b200 import _lib
    lib = _lib.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (wb_\w+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    assert set(_lib.SIGNATURES) == set(declared_symbols())
    for s in declared_symbols():
        assert getattr(lib, s) is not None
    assert lib.wb_abi_version() == 1


def test_context_create_reports_missing_device_without_crashing():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from wave_engine_b200 import _lib
    h = C.c_void_p()
    rc = _lib.lib().wb_context_create(0, C.byref(h))
    assert rc == _lib.WB_ENODEV
    assert b"device" in _lib.lib().wb_last_error()


def test_null_arguments_are_rejected():
    from wave_engine_b200 import _lib
    l = _lib.lib()
    assert l.wb_context_create(0, None) == _lib.WB_EINVAL
    assert l.wb_attn_forward(None, None, None, 1, 1, 0, None, None, None) == _lib.WB_EINVAL
    assert l.wb_kv_decode(None, None, 0, None, None, 1, None, 0, None) == _lib.WB_EINVAL
    assert l.wb_attn_layer_destroy(None) == _lib.WB_OK
    assert l.wb_dot_attn_layer_create(None, 4, 64, None, None, None, None, None) == _lib.WB_EINVAL
    assert l.wb_dot_attn_forward(None, None, None, 1, 1, 0, None) == _lib.WB_EINVAL
    assert l.wb_dot_attn_layer_destroy(None) == _lib.WB_OK
    assert l.wb_context_destroy(None) == _lib.WB_OK


@pytest.mark.parametrize("H,E,Cd", [(4, 168, 16), (8, 384, 0), (12, 768, 16)])
def test_native_init_block_attn_matches_oracle(H, E, Cd):
    """wb_init_block_attn (product) and the oracle's restatement of
    wave_model.rs:57-81 draw the same weights and leave the same state."""
    from oracle import oracle
    import wave_engine_b200 as wb
    rng = wb.Rng(99)
    w = wb.init_block_attn(rng, H, E, Cd).packed()
    ow, ostate = oracle.init_block_attn(99, H, E, Cd)
    assert rng.state == ostate
    for k, v in ow.items():
        if v is None:
            assert w[k] is None
        else:
            assert np.array_equal(w[k], v), k


def test_weights_pack_roundtrip_and_shape_errors():
    import wave_engine_b200 as wb
    w = wb.gaussian_block_attn(1, 4, 32, 16)
    p = w.packed()
    w2 = wb.WaveAttnWeights.from_packed(p)
    for k, v in w2.packed().items():
        assert np.array_equal(v, p[k])
    assert w.n_head == 4 and w.n_embd == 32 and w.head_dim == 8 and w.content_dim == 16
    w.heads[1].v_proj_w = np.zeros((3, 3), np.float32)
    with pytest.raises(ValueError):
        w.packed()
