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
  * ``return_pathway_cache=True`` returns the backward's ``WaveAttnCache``
    (attn.rs:51-70) computed by the all-fp32 SIMT kernels
    (``wb_attn_forward_cache``); ``wave_attention_backward_full`` /
    ``wave_attention_backward_pathway`` (attn.rs:346, :432) consume it.
Shape errors raise ValueError where the reference panics.
"""
from __future__ import annotations

from dataclasses import dataclass

import ctypes as C
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


@dataclass
class WaveAttnCache:
    """The forward intermediates of attn.rs:51-70 (batched: a leading batch
    axis on every array when the forward ran on [B][T][n_embd])."""
    phases: object          # [.., H, T]
    phase_rs: object        # [.., H, T, 2]  (r, s)
    v_all: object           # [.., H, T, head_dim]
    content_vecs: object    # [.., H, T, C] or None
    content_scale: list     # [H]
    att_w: object           # [.., H, T, T]
    out_merged: object      # [.., T, n_embd]
    normed: object          # [.., T, n_embd] (the forward's x)
    n_bands: int
    use_content: bool = True


def _cache_desc(cache: WaveAttnCache) -> "_lib.CacheDesc":
    return _lib.CacheDesc(ptr_of(cache.phases), ptr_of(cache.phase_rs), ptr_of(cache.v_all),
                          ptr_of(cache.content_vecs), ptr_of(cache.att_w), ptr_of(cache.out_merged))


def wave_attention_forward(weights, x, n_bands: int, backend=None, return_pathway_cache: bool = False, *,
                           path: str = "tensor", use_content: bool = True, return_att_weights: bool = False,
                           return_phases: bool = False, ctx: Context | None = None):
    """Causal multi-head wave attention forward (attn.rs:90-305) on the B200.

    Returns ``(y, att_weights, None)`` (plus ``phases`` [.., H, T] when
    ``return_phases``), with ``y`` shaped like ``x``; with
    ``return_pathway_cache`` the third value is the ``WaveAttnCache`` (and
    the forward runs the all-fp32 path)."""
    if return_pathway_cache:
        return _forward_with_cache(weights, x, n_bands, use_content=use_content, ctx=ctx)
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


def _prep(x, n_bands, ctx):
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
    return x, B, T, E, ctx


def _forward_with_cache(weights, x, n_bands, *, use_content, ctx):
    x, B, T, E, ctx = _prep(x, n_bands, ctx)
    layer = device_layer(weights, ctx)
    if layer.n_embd != E:
        raise ValueError(f"weights are for n_embd={layer.n_embd}, input has {E}")
    H, hd, Cd = layer.n_head, E // layer.n_head, layer.content_dim
    uc = use_content and Cd > 0
    lead = () if x.ndim == 2 else (B,)
    y = _empty_like_input(x, tuple(x.shape))
    cache = WaveAttnCache(
        phases=_empty_like_input(x, lead + (H, T)), phase_rs=_empty_like_input(x, lead + (H, T, 2)),
        v_all=_empty_like_input(x, lead + (H, T, hd)),
        content_vecs=_empty_like_input(x, lead + (H, T, Cd)) if uc else None,
        content_scale=[1.0 / float(np.sqrt(Cd)) if uc else 0.0] * H,
        att_w=_empty_like_input(x, lead + (H, T, T)), out_merged=_empty_like_input(x, tuple(x.shape)),
        normed=x, n_bands=n_bands, use_content=uc)
    ctx.use_torch_stream(x, y)
    desc = _cache_desc(cache)
    _lib.call("wb_attn_forward_cache", ctx.handle, layer.handle, ptr_of(x), B, T, 0 if uc else _lib.WB_NO_CONTENT,
              ptr_of(y), C.byref(desc))
    return y, cache.att_w, cache


GRAD_FIELDS = ("harmonic_raw", "phase_proj_w", "phase_proj_b", "v_proj_w", "v_proj_b", "content_proj_w",
               "content_proj_b", "out_proj_w", "out_proj_b")


def _backward(weights, cache: WaveAttnCache, d_attn_out, want_grads: bool, ctx):
    x = cache.normed
    x, B, T, E, ctx = _prep(x, cache.n_bands, ctx)
    layer = device_layer(weights, ctx)
    H, hd, Cd = layer.n_head, E // layer.n_head, layer.content_dim
    if is_torch(x) != is_torch(d_attn_out):
        raise ValueError("d_attn_out must live where the cache does (numpy or torch)")
    d_y = d_attn_out.contiguous().float() if is_torch(d_attn_out) else np.ascontiguousarray(d_attn_out, np.float32)
    if tuple(d_y.shape) != tuple(x.shape):
        raise ValueError("d_attn_out must have the forward input's shape")
    d_x = _empty_like_input(x, tuple(x.shape))
    grads = None
    gdesc = None
    if want_grads:
        uc = cache.use_content
        shapes = {"harmonic_raw": (H,), "phase_proj_w": (H, 2, E), "phase_proj_b": (H, 2), "v_proj_w": (H, hd, hd),
                  "v_proj_b": (H, hd), "content_proj_w": (H, Cd, E) if uc else None,
                  "content_proj_b": (H, Cd) if uc else None, "out_proj_w": (E, E), "out_proj_b": (E,)}
        grads = {k: (_empty_like_input(x, s) if s else None) for k, s in shapes.items()}
        gdesc = _lib.GradsDesc(*[ptr_of(grads[k]) for k in GRAD_FIELDS])
    ctx.use_torch_stream(x, d_x)
    desc = _cache_desc(cache)
    _lib.call("wb_attn_backward", ctx.handle, layer.handle, ptr_of(x), ptr_of(d_y), B, T,
              0 if cache.use_content else _lib.WB_NO_CONTENT, C.byref(desc), ptr_of(d_x),
              C.byref(gdesc) if gdesc is not None else None)
    return d_x, grads


def wave_attention_backward_full(weights, cache: WaveAttnCache, d_attn_out, *, ctx: Context | None = None):
    """attn.rs:346 wave_attention_backward_full on the GPU: returns the
    reference's WaveAttnGrads as a dict -- the weight gradients (summed over
    the batch) under the wb_attn_weights_desc names, and ``d_normed``."""
    d_x, grads = _backward(weights, cache, d_attn_out, True, ctx)
    grads["d_normed"] = d_x
    return grads


def wave_attention_backward_pathway(weights, cache: WaveAttnCache, d_attn_out, *, ctx: Context | None = None):
    """attn.rs:432 wave_attention_backward_pathway on the GPU: d_normed only."""
    d_x, _ = _backward(weights, cache, d_attn_out, False, ctx)
    return d_x
