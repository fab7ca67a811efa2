"""Contexts and device-resident weights over the C ABI.

A ``Context`` is one device plus one stream (``wb_context``); an
``AttnLayer`` is one block's attention weights uploaded to that device
(``wb_attn_layer``).  Buffers passed to the entry points may be numpy arrays
(host memory) or torch tensors (host or CUDA); the library detects which.
"""
from __future__ import annotations

import ctypes as C
import threading
import weakref

import numpy as np

from . import _lib
from .weights import WaveAttnWeights

try:  # torch is optional plumbing (device buffers and streams)
    import torch
except Exception:  # pragma: no cover
    torch = None


def is_torch(a) -> bool:
    return torch is not None and isinstance(a, torch.Tensor)


def ptr_of(a, dtype=np.float32):
    """Raw pointer of a contiguous numpy array / torch tensor (None stays None)."""
    if a is None:
        return None
    if is_torch(a):
        want = {np.float32: torch.float32, np.int32: torch.int32, np.uint8: torch.uint8}[dtype]
        if a.dtype != want or not a.is_contiguous():
            raise ValueError(f"tensor must be contiguous {want}")
        return a.data_ptr()
    if not isinstance(a, np.ndarray) or a.dtype != dtype or not a.flags.c_contiguous:
        raise ValueError(f"array must be a C-contiguous {np.dtype(dtype).name} numpy array")
    return a.ctypes.data


class Context:
    """wb_context: one device, one stream.  Not thread-safe (one per thread)."""

    def __init__(self, device: int = 0):
        self.device = device
        h = C.c_void_p()
        _lib.call("wb_context_create", device, C.byref(h))
        self.handle = h
        self._children = weakref.WeakSet()  # layers / caches to release first

    def adopt(self, obj) -> None:
        self._children.add(obj)

    def close(self) -> None:
        """Release every layer and cache of this context, then the context."""
        if self.handle:
            for ch in list(self._children):
                ch.close()
            _lib.lib().wb_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, cuda_stream: int | None) -> None:
        """Run later calls on this cudaStream_t handle; 0/None is CUDA's legacy
        default stream (torch's default stream)."""
        _lib.call("wb_context_set_stream", self.handle, cuda_stream or None)

    def use_own_stream(self) -> None:
        """Back to the context's private stream."""
        _lib.call("wb_context_set_stream", self.handle, _lib.lib().wb_context_own_stream(self.handle))

    def synchronize(self) -> None:
        _lib.call("wb_context_synchronize", self.handle)

    def take_device_error(self) -> int:
        v = C.c_uint32(0)
        _lib.call("wb_context_take_device_error", self.handle, C.byref(v))
        return int(v.value)

    def profile(self, name_filter: str | None = "") -> None:
        """Time named kernels with CUDA events ("" = all, None = off)."""
        _lib.call("wb_context_profile", self.handle, None if name_filter is None else name_filter.encode())

    def profile_report(self) -> dict:
        """{kernel: (launches, total_ms)} since the last report (synchronises)."""
        buf = C.create_string_buffer(1 << 16)
        _lib.call("wb_context_profile_report", self.handle, buf, len(buf))
        out = {}
        for line in buf.value.decode().splitlines():
            name, n, ms = line.split("\t")
            out[name] = (int(n), float(ms))
        return out

    def use_torch_stream(self, *tensors):
        """Run on torch's current stream when any argument is a CUDA tensor
        (host-only calls keep the context's current stream)."""
        for t in tensors:
            if is_torch(t) and t.is_cuda:
                self.set_stream(torch.cuda.current_stream(t.device).cuda_stream)
                return


_tls = threading.local()


def default_context(device: int = 0) -> Context:
    """One lazily created context per (thread, device)."""
    d = getattr(_tls, "ctx", None)
    if d is None:
        d = _tls.ctx = {}
    if device not in d:
        d[device] = Context(device)
    return d[device]


class AttnLayer:
    """wb_attn_layer: a WaveAttnWeights uploaded to one context's device."""

    def __init__(self, ctx: Context, weights: WaveAttnWeights):
        p = weights.packed()
        self._keep = p  # host arrays only need to live during create, kept for clarity
        self.ctx = ctx
        self.n_embd, self.n_head, self.content_dim = weights.n_embd, weights.n_head, weights.content_dim
        self.head_dim = self.n_embd // self.n_head
        g = lambda k: None if p[k] is None else p[k].ctypes.data
        desc = _lib.WeightsDesc(self.n_embd, self.n_head, self.content_dim,
                                g("harmonic_raw"), g("phase_proj_w"), g("phase_proj_b"), g("v_proj_w"),
                                g("v_proj_b"), g("content_proj_w"), g("content_proj_b"), g("out_proj_w"),
                                g("out_proj_b"))
        h = C.c_void_p()
        _lib.call("wb_attn_layer_create", ctx.handle, C.byref(desc), C.byref(h))
        self.handle = h
        self._keep = None
        ctx.adopt(self)

    def close(self) -> None:
        if self.handle:
            _lib.lib().wb_attn_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def device_layer(weights, ctx: Context) -> AttnLayer:
    """The AttnLayer for (weights, ctx), uploading on first use."""
    if isinstance(weights, AttnLayer):
        if weights.ctx is not ctx:
            raise ValueError("AttnLayer belongs to another context")
        return weights
    key = id(ctx)
    lay = weights._device.get(key)
    if lay is None or lay.ctx is not ctx or not lay.handle:
        lay = weights._device[key] = AttnLayer(ctx, weights)
    return lay
