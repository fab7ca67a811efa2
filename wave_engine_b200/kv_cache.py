"""Host-side mirror of src/common/kv_cache.rs's attention cache.

``KvCache`` holds, per layer and sequence slot, the per-head phases,
buckets and values that kv_cache.rs:36-54 keeps in ``HeadCache`` vectors,
resident on the GPU.  ``prefill`` and ``forward_one`` run the attention part
of kv_cache.rs:121-193 and :263-335 for one layer over a batch of sequences
(the reference handles one request per call; several slots make the batched
serve loop).  The LN / FFN / lm_head around attention stay with the caller.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from .attn import PATHS, _empty_like_input
from .runtime import Context, default_context, device_layer, is_torch, ptr_of


PAGE = 128  # positions per page of a paged cache (WB_KV_PAGE)


class KvCache:
    """Device-resident cache: n_layers x max_seqs slots of max_ctx positions.

    With ``n_pages`` the cache is paged: each layer's storage is a pool of
    ``n_pages`` pages of 128 positions (all heads) that slots take as they
    grow -- ``reserve(seq, n_positions)`` before a prefill or decode needs
    them, ``release(seq)`` when the request ends.  Results are identical to
    the contiguous cache's."""

    def __init__(self, n_layers: int, n_head: int, head_dim: int, max_seqs: int = 1, max_ctx: int = 256,
                 ctx: Context | None = None, n_pages: int | None = None):
        self.ctx = ctx or default_context(0)
        self.n_layers, self.n_head, self.head_dim = n_layers, n_head, head_dim
        self.max_seqs, self.max_ctx = max_seqs, max_ctx
        self.paged = n_pages is not None
        h = C.c_void_p()
        if self.paged:
            _lib.call("wb_kv_cache_create_paged", self.ctx.handle, n_layers, n_head, head_dim, max_seqs, max_ctx,
                      int(n_pages), C.byref(h))
        else:
            _lib.call("wb_kv_cache_create", self.ctx.handle, n_layers, n_head, head_dim, max_seqs, max_ctx,
                      C.byref(h))
        self.handle = h
        self.ctx.adopt(self)

    def reserve(self, seq: int, n_positions: int) -> None:
        """Paged cache: pages so that slot ``seq`` holds ``n_positions``
        (WaveB200Error when the pool is short).  No-op when contiguous."""
        _lib.call("wb_kv_seq_reserve", self.handle, int(seq), int(n_positions))

    def release(self, seq: int) -> None:
        """Empty slot ``seq`` and return its pages to the pool."""
        _lib.call("wb_kv_seq_release", self.handle, int(seq))

    def free_pages(self) -> int:
        v = C.c_int(0)
        _lib.call("wb_kv_cache_free_pages", self.handle, C.byref(v))
        return int(v.value)

    def close(self) -> None:
        if self.handle:
            _lib.lib().wb_kv_cache_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def n_cached(self, layer: int = 0, seq: int = 0) -> int:
        v = C.c_int(0)
        _lib.call("wb_kv_cache_length", self.handle, layer, seq, C.byref(v))
        return int(v.value)

    def reset_seq(self, seq: int) -> None:
        _lib.call("wb_kv_cache_reset_seq", self.handle, seq)

    def reset(self) -> None:
        """Empty every slot (every sequence, every layer)."""
        _lib.call("wb_kv_cache_reset_seq", self.handle, -1)

    def load(self, layer: int, seq: int, phases, values) -> None:
        """Fill one slot from phases [H][n] and values [H][n][hd]."""
        if not is_torch(phases):
            phases = np.ascontiguousarray(phases, np.float32)
            values = np.ascontiguousarray(values, np.float32)
        n = int(phases.shape[1])
        if tuple(phases.shape) != (self.n_head, n) or tuple(values.shape) != (self.n_head, n, self.head_dim):
            raise ValueError("phases must be [H][n] and values [H][n][head_dim]")
        _lib.call("wb_kv_cache_load", self.ctx.handle, self.handle, layer, seq, n, ptr_of(phases),
                  ptr_of(values))

    def read(self, layer: int, seq: int):
        """(phases [H][n], buckets [H][n] u8, values [H][n][hd]) of one slot."""
        n = self.n_cached(layer, seq)
        ph = np.empty((self.n_head, n), np.float32)
        bk = np.empty((self.n_head, n), np.uint8)
        vv = np.empty((self.n_head, n, self.head_dim), np.float32)
        _lib.call("wb_kv_cache_read", self.ctx.handle, self.handle, layer, seq, ph.ctypes.data, bk.ctypes.data,
                  vv.ctypes.data)
        return ph, bk, vv

    @staticmethod
    def _ids(seq_ids):
        if is_torch(seq_ids):
            return seq_ids
        return np.ascontiguousarray(np.atleast_1d(np.asarray(seq_ids)), dtype=np.int32)

    def prefill(self, layer_idx: int, weights, x, seq_ids=(0,), *, path: str = "tensor", out=None):
        """Prompt attention (kv_cache.rs:121-193) of x [n_seq][T][E] (or
        [T][E] for one sequence) into empty slots; returns y shaped like x."""
        if not is_torch(x):
            x = np.ascontiguousarray(x, np.float32)
        single = x.ndim == 2
        n_seq, T, E = (1, *x.shape) if single else tuple(x.shape)
        ids = self._ids(seq_ids)
        if int(ids.shape[0]) != n_seq:
            raise ValueError("one seq id per sequence")
        layer = device_layer(weights, self.ctx)
        y = _empty_like_input(x, tuple(x.shape)) if out is None else out
        self.ctx.use_torch_stream(x, y)
        _lib.call("wb_kv_prefill", self.ctx.handle, self.handle, layer_idx, layer.handle, ptr_of(ids, np.int32),
                  n_seq, ptr_of(x), T, PATHS[path], ptr_of(y))
        return y

    def forward_one(self, layer_idx: int, weights, x, seq_ids=(0,), *, path: str = "tensor", out=None):
        """One new position per sequence (kv_cache.rs:263-335): x [n_seq][E]
        (or [E]); appends to each slot and returns y shaped like x."""
        if not is_torch(x):
            x = np.ascontiguousarray(x, np.float32)
        single = x.ndim == 1
        n_seq = 1 if single else int(x.shape[0])
        ids = self._ids(seq_ids)
        if int(ids.shape[0]) != n_seq:
            raise ValueError("one seq id per sequence")
        layer = device_layer(weights, self.ctx)
        y = _empty_like_input(x, tuple(x.shape)) if out is None else out
        self.ctx.use_torch_stream(x, y)
        _lib.call("wb_kv_decode", self.ctx.handle, self.handle, layer_idx, layer.handle, ptr_of(ids, np.int32),
                  n_seq, ptr_of(x), PATHS[path], ptr_of(y))
        return y
