"""Host-side mirror of the legacy dot-product attention:
``ComputeBackend::attention(weights, x)`` (src/common/compute.rs:43, CPU
implementation ``attention_cpu`` at compute.rs:357-414).

    weights = AttentionWeights(c_attn_w, c_attn_b, c_proj_w, c_proj_b, n_head)
    y = attention(weights, x)

``AttentionWeights`` follows src/common/model.rs:191-195 (``c_attn`` a
LinearWeights [3*n_embd][n_embd] plus bias, ``c_proj`` [n_embd][n_embd] plus
bias, ``n_head``); ``x`` is ``[T][n_embd]`` as the reference or
``[B][T][n_embd]`` (independent sequences).  The work runs in the CUDA
library through ``wb_dot_attn_forward``; there is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .attn import PATHS, _empty_like_input
from .runtime import Context, default_context, is_torch, ptr_of

try:
    import torch
except Exception:  # pragma: no cover
    torch = None


class AttentionWeights:
    """model.rs:191-195: c_attn (w [3E][E], b [3E]), c_proj (w [E][E], b [E]), n_head."""

    def __init__(self, c_attn_w, c_attn_b, c_proj_w, c_proj_b, n_head: int):
        self.c_attn_w = np.ascontiguousarray(c_attn_w, dtype=np.float32)
        self.c_attn_b = np.ascontiguousarray(c_attn_b, dtype=np.float32)
        self.c_proj_w = np.ascontiguousarray(c_proj_w, dtype=np.float32)
        self.c_proj_b = np.ascontiguousarray(c_proj_b, dtype=np.float32)
        self.n_head = int(n_head)
        E = self.c_proj_w.shape[0]
        if (self.c_attn_w.shape != (3 * E, E) or self.c_attn_b.shape != (3 * E,) or self.c_proj_w.shape != (E, E)
                or self.c_proj_b.shape != (E,)):
            raise ValueError("AttentionWeights: c_attn [3E][E] + [3E], c_proj [E][E] + [E]")
        if E % self.n_head:
            raise ValueError("n_embd must be a multiple of n_head")
        self.n_embd = E
        self._device = {}

    def packed(self) -> dict:
        return {"c_attn_w": self.c_attn_w, "c_attn_b": self.c_attn_b, "c_proj_w": self.c_proj_w,
                "c_proj_b": self.c_proj_b, "n_head": self.n_head}


def gaussian_attention_weights(seed: int, n_head: int, n_embd: int, std: float = 0.02,
                               bias_std: float = 0.0) -> AttentionWeights:
    """Seeded N(0, std) weights and N(0, bias_std) biases: the synthetic stand-in used by the tests and the
    benchmark (the measurement weights of the wave path are N(0, 0.02) too; the reference's own init_linear,
    wave_model.rs:39-46, draws uniform(+-1/sqrt(in)) with zero biases)."""
    g = np.random.default_rng(seed)
    E = n_embd
    return AttentionWeights(g.normal(0, std, (3 * E, E)), g.normal(0, bias_std, 3 * E) if bias_std else np.zeros(3 * E),
                            g.normal(0, std, (E, E)), g.normal(0, bias_std, E) if bias_std else np.zeros(E), n_head)


class DotAttnLayer:
    """wb_dot_attn_layer: AttentionWeights uploaded to one context's device."""

    def __init__(self, ctx: Context, weights: AttentionWeights):
        self.ctx = ctx
        self.n_embd, self.n_head = weights.n_embd, weights.n_head
        h = C.c_void_p()
        _lib.call("wb_dot_attn_layer_create", ctx.handle, self.n_head, self.n_embd, weights.c_attn_w.ctypes.data,
                  weights.c_attn_b.ctypes.data, weights.c_proj_w.ctypes.data, weights.c_proj_b.ctypes.data,
                  C.byref(h))
        self.handle = h
        ctx.adopt(self)

    def close(self) -> None:
        if self.handle:
            _lib.lib().wb_dot_attn_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _device_layer(weights, ctx: Context) -> DotAttnLayer:
    if isinstance(weights, DotAttnLayer):
        if weights.ctx is not ctx:
            raise ValueError("DotAttnLayer belongs to another context")
        return weights
    lay = weights._device.get(id(ctx))
    if lay is None or lay.ctx is not ctx or not lay.handle:
        lay = weights._device[id(ctx)] = DotAttnLayer(ctx, weights)
    return lay


def attention(weights, x, *, path: str = "tensor", ctx: Context | None = None):
    """Causal dot-product self-attention (compute.rs:357-414): ``y`` shaped like ``x``."""
    if path not in PATHS:
        raise ValueError(f"path must be one of {sorted(PATHS)}")
    if not is_torch(x):
        x = np.ascontiguousarray(x, dtype=np.float32)
    elif x.dtype != torch.float32 or not x.is_contiguous():
        x = x.contiguous().float()
    if x.ndim not in (2, 3):
        raise ValueError("x must be [T][n_embd] or [B][T][n_embd]")
    B, T, E = (1, *x.shape) if x.ndim == 2 else tuple(x.shape)
    if ctx is None:
        dev = x.device.index if (is_torch(x) and x.is_cuda) else 0
        ctx = default_context(dev or 0)
    layer = _device_layer(weights, ctx)
    if layer.n_embd != E:
        raise ValueError(f"weights are for n_embd={layer.n_embd}, input has {E}")
    y = _empty_like_input(x, tuple(x.shape))
    ctx.use_torch_stream(x, y)
    _lib.call("wb_dot_attn_forward", ctx.handle, layer.handle, ptr_of(x), B, T, PATHS[path], ptr_of(y))
    return y
