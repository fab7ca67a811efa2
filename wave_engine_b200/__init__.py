"""B200-native (sm_100a) wave attention: prefill and KV-cache decode.

The hot path of wave-engine's causal multi-head wave attention forward
(src/common/attn.rs:90, src/common/kv_cache.rs:93/:241) behind a C ABI
(include/wave_b200.h) implemented by the in-tree CUDA library
``libwave_b200.so``.  This package is the host-side mirror of the
reference's interface for that path, plus the legacy dot-product attention
of ComputeBackend::attention (src/common/compute.rs:43, :357-414).
"""
from .weights import CONTENT_DIM, Rng, WaveAttnHeadWeights, WaveAttnWeights, gaussian_block_attn, init_block_attn
from .runtime import AttnLayer, Context, default_context
from .attn import (WaveAttnCache, wave_attention_backward_full, wave_attention_backward_pathway,
                   wave_attention_forward, wave_attention_forward_heads)
from .kv_cache import KvCache
from .dot_attn import AttentionWeights, DotAttnLayer, attention, gaussian_attention_weights
from ._lib import WaveB200Error
from .checkpoint import WchkHeader, load_wchk_attention, read_wchk_header
from .serve import (Agc, FfnLayer, KerrFfnWeights, ServeBlock, ServeModel, ServeSession, embed, ffn_forward,
                    gaussian_ffn, layer_norm, lm_head, phase_native_decode, residual_add)

__all__ = [
    "CONTENT_DIM", "Rng", "WaveAttnHeadWeights", "WaveAttnWeights", "gaussian_block_attn", "init_block_attn",
    "AttnLayer", "Context", "default_context", "wave_attention_forward", "wave_attention_forward_heads", "KvCache",
    "WaveAttnCache", "wave_attention_backward_full", "wave_attention_backward_pathway",
    "Agc", "FfnLayer", "KerrFfnWeights", "ServeBlock", "ServeModel", "ServeSession", "embed", "ffn_forward",
    "gaussian_ffn", "layer_norm", "lm_head", "phase_native_decode", "residual_add",
    "WaveB200Error", "WchkHeader", "load_wchk_attention", "read_wchk_header", "AttentionWeights", "DotAttnLayer", "attention", "gaussian_attention_weights",
]
