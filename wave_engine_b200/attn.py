"""Host-side mirror of src/common/attn.rs:90 ``wave_attention_forward``.

Same name, argument meaning and return shape as the reference:

    y, att_weights, cache = wave_attention_forward(weights, x, n_bands,
                                                   backend=None,
                                                   return_pathway_cache=False)

``x`` is ``[T][n_embd]`` (one sequence, as the reference) or ``[B][T][n_embd]``
(a batch of independent sequences, the batched form of the reference's
thread-per-sequence loop in src/cpu/train_loop.rs:320).  The work runs in the
CUDA library through ``wb_attn_forward``; there is no CPU path.

Differences that the reference's own callers never observe:
  * ``att_weights`` ([H][T][T], -inf above the diagonal as attn.rs:240
    leaves them) is only computed when ``return_att_weights=True``; it
    otherwise comes back as an empty list, because materialising T x T per
    head is what the B200 path exists to avoid.  Its one consumer is the
    attention monitor (src/monitors/attn_monitor.rs:26).
  * ``backend`` is accepted and ignored: the reference only uses it to run
    the out_proj on wgpu (attn.rs:273-274); here out_proj is on the GPU.
  * ``return_pathway_cache=True`` (the backward's WaveAttnCache) raises
    NotImplementedError: backward is not part of this library.
Shape errors raise ValueError where the reference panics.
"""
from __future__ import annotations

import numpy as np

from . import _lib
from .runtime import Context, default_context, device_layer, is_torch, ptr_of

try:
    import torch
except Exception:  # pragma: no cover
    torch = None

PATHS = {"tensor": _lib.WB_PATH_TENSOR, "exact": _lib.WB_PATH_EXACT}


def _empty_like_input(x, shape):
    if is_torch(x):
        return torch.empty(shape, dtype=torch.float32, device=x.device)
    return np.empty(shape, np.float32)


def wave_attention_forward(weights, x, n_bands: int, backend=None, return_pathway_cache: bool = False, *,
                           path: str = "tensor", use_content: bool = True, return_att_weights: bool = False,
                           return_phases: bool = False, ctx: Context | None = None):
    """Causal multi-head wave attention forward (attn.rs:90-305) on the B200.

    Returns ``(y, att_weights, None)`` (plus ``phases`` [.., H, T] when
    ``return_phases``), with ``y`` shaped like ``x``."""
    if return_pathway_cache:
        raise NotImplementedError("return_pathway_cache (WaveAttnCache for backward) is not supported")
    if path not in PATHS:
        raise ValueError(f"path must be one of {sorted(PATHS)}")
    if not is_torch(x):
        x = np.ascontiguousarray(x, dtype=np.float32)
    elif x.dtype != torch.float32 or not x.is_contiguous():
        x = x.contiguous().float()
    if x.ndim not in (2, 3):
        raise ValueError("x must be [T][n_embd] or [B][T][n_embd]")
    single = x.ndim == 2
    B, T, E = (1, *x.shape) if single else tuple(x.shape)
    if E != 2 * n_bands:
        raise ValueError(f"n_embd mismatch: n_bands*2 = {2 * n_bands}, input has {E}")
    if isinstance(weights, type(None)):
        raise ValueError("weights is None")
    if ctx is None:
        dev = x.device.index if (is_torch(x) and x.is_cuda) else 0
        ctx = default_context(dev or 0)
    layer = device_layer(weights, ctx)
    if layer.n_embd != E:
        raise ValueError(f"weights are for n_embd={layer.n_embd}, input has {E}")
    H = layer.n_head
    y = _empty_like_input(x, tuple(x.shape))
    aw = _empty_like_input(x, (B, H, T, T)) if return_att_weights else None
    ph = _empty_like_input(x, (B, H, T)) if return_phases else None
    flags = PATHS[path] | (0 if use_content else _lib.WB_NO_CONTENT)
    ctx.use_torch_stream(x, y)
    _lib.call("wb_attn_forward", ctx.handle, layer.handle, ptr_of(x), B, T, flags, ptr_of(y), ptr_of(aw),
              ptr_of(ph))
    if single:
        aw = aw[0] if aw is not None else None
        ph = ph[0] if ph is not None else None
    att = aw if aw is not None else []
    if return_phases:
        return y, att, None, ph
    return y, att, None


def wave_attention_forward_heads(weights, x, n_bands: int, head_begin: int, head_end: int, *, add_bias: bool,
                                 use_content: bool = True, ctx: Context | None = None):
    """Heads [head_begin, head_end) of the prefill forward (tensor path):
    ``y_partial = o[:, heads] W_out[:, heads]^T`` (+ the out_proj bias when
    ``add_bias``).  The sum over ranges that cover every head once, with the
    bias added once, is ``wave_attention_forward``'s ``y``: the head-sharded
    4096-dim model runs one range per GPU and all-reduces ``y_partial``.
    No counterpart in the reference (attn.rs:90 runs every head)."""
    if not is_torch(x):
        x = np.ascontiguousarray(x, dtype=np.float32)
    elif x.dtype != torch.float32 or not x.is_contiguous():
        x = x.contiguous().float()
    if x.ndim not in (2, 3):
        raise ValueError("x must be [T][n_embd] or [B][T][n_embd]")
    B, T, E = (1, *x.shape) if x.ndim == 2 else tuple(x.shape)
    if E != 2 * n_bands:
        raise ValueError(f"n_embd mismatch: n_bands*2 = {2 * n_bands}, input has {E}")
    if ctx is None:
        dev = x.device.index if (is_torch(x) and x.is_cuda) else 0
        ctx = default_context(dev or 0)
    layer = device_layer(weights, ctx)
    y = _empty_like_input(x, tuple(x.shape))
    ctx.use_torch_stream(x, y)
    _lib.call("wb_attn_forward_heads", ctx.handle, layer.handle, ptr_of(x), B, T, int(head_begin), int(head_end),
              1 if add_bias else 0, 0 if use_content else _lib.WB_NO_CONTENT, ptr_of(y))
    return y
