"""ctypes binding of the in-tree CUDA library (``libwave_b200.so``).

The library is the product: there is no Python or CPU fallback.  Importing
this module fails loudly when the shared object is missing; build it with
``python -m wave_engine_b200.build``.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libwave_b200.so"

WB_OK = 0
WB_EINVAL = -1
WB_ENOMEM = -2
WB_ECUDA = -3
WB_ENOTSUP = -4
WB_ETIMEOUT = -5
WB_ENODEV = -6

WB_PATH_TENSOR = 0x0
WB_PATH_EXACT = 0x1
WB_NO_CONTENT = 0x2
WB_RETURN_PATHWAY = 0x4

_F = C.POINTER(C.c_float)
_VP = C.c_void_p

# Every symbol the C ABI (include/wave_b200.h) declares, with its signature.
SIGNATURES = {
    "wb_abi_version": (C.c_int, []),
    "wb_last_error": (C.c_char_p, []),
    "wb_context_create": (C.c_int, [C.c_int, C.POINTER(_VP)]),
    "wb_context_destroy": (C.c_int, [_VP]),
    "wb_context_set_stream": (C.c_int, [_VP, _VP]),
    "wb_context_own_stream": (_VP, [_VP]),
    "wb_context_synchronize": (C.c_int, [_VP]),
    "wb_context_take_device_error": (C.c_int, [_VP, C.POINTER(C.c_uint32)]),
    "wb_context_profile": (C.c_int, [_VP, C.c_char_p]),
    "wb_context_profile_report": (C.c_int, [_VP, C.c_char_p, C.c_size_t]),
    "wb_attn_layer_create": (C.c_int, [_VP, _VP, C.POINTER(_VP)]),
    "wb_attn_layer_destroy": (C.c_int, [_VP]),
    "wb_init_block_attn": (C.c_int, [C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_int] + [_VP] * 9),
    "wb_attn_forward": (C.c_int, [_VP, _VP, _VP, C.c_int, C.c_int, C.c_int, _VP, _VP, _VP]),
    "wb_attn_forward_heads": (C.c_int, [_VP, _VP, _VP, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _VP]),
    "wb_dot_attn_layer_create": (C.c_int, [_VP, C.c_int, C.c_int, _VP, _VP, _VP, _VP, C.POINTER(_VP)]),
    "wb_dot_attn_layer_destroy": (C.c_int, [_VP]),
    "wb_dot_attn_forward": (C.c_int, [_VP, _VP, _VP, C.c_int, C.c_int, C.c_int, _VP]),
    "wb_kv_cache_create": (C.c_int, [_VP, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_VP)]),
    "wb_kv_cache_destroy": (C.c_int, [_VP]),
    "wb_kv_cache_length": (C.c_int, [_VP, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "wb_kv_cache_reset_seq": (C.c_int, [_VP, C.c_int]),
    "wb_kv_cache_create_paged": (C.c_int, [_VP, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_VP)]),
    "wb_kv_seq_reserve": (C.c_int, [_VP, C.c_int, C.c_int]),
    "wb_kv_seq_release": (C.c_int, [_VP, C.c_int]),
    "wb_kv_cache_free_pages": (C.c_int, [_VP, C.POINTER(C.c_int)]),
    "wb_kv_cache_load": (C.c_int, [_VP, _VP, C.c_int, C.c_int, C.c_int, _VP, _VP]),
    "wb_kv_cache_read": (C.c_int, [_VP, _VP, C.c_int, C.c_int, _VP, _VP, _VP]),
    "wb_kv_prefill": (C.c_int, [_VP, _VP, C.c_int, _VP, _VP, C.c_int, _VP, C.c_int, C.c_int, _VP]),
    "wb_kv_decode": (C.c_int, [_VP, _VP, C.c_int, _VP, _VP, C.c_int, _VP, C.c_int, _VP]),
    "wb_kv_decode_noalloc": (C.c_int, [_VP, _VP, C.c_int, _VP, _VP, C.c_int, _VP, _VP]),
    "wb_attn_forward_cache": (C.c_int, [_VP, _VP, _VP, C.c_int, C.c_int, C.c_int, _VP, _VP]),
    "wb_attn_backward": (C.c_int, [_VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int, _VP, _VP, _VP]),
    "wb_ffn_layer_create": (C.c_int, [_VP, _VP, C.POINTER(_VP)]),
    "wb_ffn_layer_destroy": (C.c_int, [_VP]),
    "wb_agc_create": (C.c_int, [_VP, C.c_float, C.c_float, C.POINTER(_VP)]),
    "wb_agc_destroy": (C.c_int, [_VP]),
    "wb_agc_read": (C.c_int, [_VP, _VP]),
    "wb_ffn_forward": (C.c_int, [_VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int, _VP]),
    "wb_layer_norm": (C.c_int, [_VP, _VP, C.c_int, C.c_int, _VP, _VP, _VP]),
    "wb_residual_add": (C.c_int, [_VP, _VP, _VP, _VP, C.c_longlong]),
    "wb_embed": (C.c_int, [_VP, _VP, _VP, C.c_int, _VP, C.c_int, _VP, C.c_int, C.c_int, _VP]),
    "wb_phase_native_decode": (C.c_int, [_VP, _VP, C.c_int, C.c_int, _VP, _VP, C.c_int, C.c_int, _VP]),
    "wb_lm_head": (C.c_int, [_VP, _VP, C.c_int, C.c_int, _VP, C.c_int, C.c_int, _VP]),
    # include/wave_b200_testing.h
    "wb_test_gemm_bf16": (C.c_int, [_VP, _VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int]),
    "wb_test_gemm_tf32": (C.c_int, [_VP, _VP, _VP, _VP, _VP, C.c_int, C.c_int, C.c_int]),
    "wb_test_dot_core": (C.c_int, [_VP, _VP, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _VP]),
}


class WeightsDesc(C.Structure):
    """wb_attn_weights_desc (include/wave_b200.h)."""
    _fields_ = [
        ("n_embd", C.c_int32), ("n_head", C.c_int32), ("content_dim", C.c_int32),
        ("harmonic_raw", _VP), ("phase_proj_w", _VP), ("phase_proj_b", _VP),
        ("v_proj_w", _VP), ("v_proj_b", _VP), ("content_proj_w", _VP), ("content_proj_b", _VP),
        ("out_proj_w", _VP), ("out_proj_b", _VP),
    ]


class CacheDesc(C.Structure):
    """wb_attn_cache_desc (include/wave_b200.h)."""
    _fields_ = [("phases", _VP), ("phase_rs", _VP), ("v_all", _VP), ("content", _VP), ("att_w", _VP),
                ("out_merged", _VP)]


class GradsDesc(C.Structure):
    """wb_attn_grads_desc (include/wave_b200.h)."""
    _fields_ = [("harmonic_raw", _VP), ("phase_proj_w", _VP), ("phase_proj_b", _VP), ("v_proj_w", _VP),
                ("v_proj_b", _VP), ("content_proj_w", _VP), ("content_proj_b", _VP), ("out_proj_w", _VP),
                ("out_proj_b", _VP)]


class FfnWeightsDesc(C.Structure):
    """wb_ffn_weights_desc (include/wave_b200.h)."""
    _fields_ = [("n_embd", C.c_int32), ("maestro_dim", C.c_int32), ("rk4_steps", C.c_int32),
                ("use_corrector", C.c_int32), ("out_groups", C.c_int32),
                ("mi_squeeze_w", _VP), ("mi_squeeze_b", _VP), ("mi_process_w", _VP), ("mi_process_b", _VP),
                ("mo_squeeze_w", _VP), ("mo_squeeze_b", _VP), ("mo_process_w", _VP), ("mo_process_b", _VP),
                ("gamma_raw", _VP), ("omega", _VP), ("alpha", C.c_float), ("beta", C.c_float),
                ("phase_correction", _VP), ("rk4_weights", _VP), ("out_w", _VP), ("out_b", _VP)]


class WaveB200Error(RuntimeError):
    """A non-zero status from the C ABI, with wb_last_error()'s message."""

    def __init__(self, code: int, func: str, msg: str):
        super().__init__(f"{func} failed with status {code}: {msg}")
        self.code = code


_lib = None


def lib() -> C.CDLL:
    """Load the shared library (once) and declare every ABI signature."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: the CUDA extension of wave_engine_b200 has not been built "
                "(run `python -m wave_engine_b200.build`); there is no CPU fallback")
        l = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def check(rc: int, func: str) -> None:
    if rc != WB_OK:
        msg = lib().wb_last_error()
        raise WaveB200Error(rc, func, msg.decode() if msg else "")


def call(func: str, *args) -> None:
    check(getattr(lib(), func)(*args), func)
