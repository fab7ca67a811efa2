"""Attention weights: the reference's structs and their initialisers.

``WaveAttnHeadWeights`` / ``WaveAttnWeights`` mirror
src/common/attn.rs:19-46 field for field (``Vec<Vec<f32>>`` becomes a 2-D
float32 array).  ``Rng`` and ``init_block_attn`` mirror
src/common/rng.rs:24-39 and src/common/wave_model.rs:39-81; the draws are
made by the native library (``wb_init_block_attn``).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib

CONTENT_DIM = 16  # src/common/attn.rs:15


@dataclass
class WaveAttnHeadWeights:
    """One head (attn.rs:19-37)."""
    harmonic_raw: float
    phase_proj_w: np.ndarray   # [2][n_embd]
    phase_proj_b: np.ndarray   # [2]
    v_proj_w: np.ndarray       # [head_dim][head_dim]
    v_proj_b: np.ndarray       # [head_dim]
    content_proj_w: np.ndarray  # [CONTENT_DIM][n_embd], or shape (0, n_embd) when empty
    content_proj_b: np.ndarray  # [CONTENT_DIM] or empty


@dataclass
class WaveAttnWeights:
    """All heads plus the combined output projection (attn.rs:40-46)."""
    heads: list
    out_proj_w: np.ndarray  # [n_embd][n_embd]
    out_proj_b: np.ndarray  # [n_embd]
    _device: dict = field(default_factory=dict, repr=False, compare=False)

    @property
    def n_head(self) -> int:
        return len(self.heads)

    @property
    def n_embd(self) -> int:
        return int(self.out_proj_w.shape[0])

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def content_dim(self) -> int:
        cw = self.heads[0].content_proj_w
        return 0 if cw is None or np.size(cw) == 0 else int(np.shape(cw)[0])

    def packed(self) -> dict:
        """Stacked float32 arrays in the C ABI layouts (include/wave_b200.h)."""
        f = lambda a: np.ascontiguousarray(a, dtype=np.float32)
        H, E, Cd = self.n_head, self.n_embd, self.content_dim
        for h in self.heads:
            cw = np.asarray(h.content_proj_w)
            if (0 if cw.size == 0 else cw.shape[0]) != Cd:
                raise ValueError("all heads must have the same content_dim")
        out = {
            "harmonic_raw": f([h.harmonic_raw for h in self.heads]),
            "phase_proj_w": f(np.stack([np.asarray(h.phase_proj_w) for h in self.heads])),
            "phase_proj_b": f(np.stack([np.asarray(h.phase_proj_b) for h in self.heads])),
            "v_proj_w": f(np.stack([np.asarray(h.v_proj_w) for h in self.heads])),
            "v_proj_b": f(np.stack([np.asarray(h.v_proj_b) for h in self.heads])),
            "content_proj_w": f(np.stack([np.asarray(h.content_proj_w) for h in self.heads])) if Cd else None,
            "content_proj_b": f(np.stack([np.asarray(h.content_proj_b) for h in self.heads])) if Cd else None,
            "out_proj_w": f(self.out_proj_w),
            "out_proj_b": f(self.out_proj_b),
        }
        d = E // H
        shapes = {"phase_proj_w": (H, 2, E), "phase_proj_b": (H, 2), "v_proj_w": (H, d, d), "v_proj_b": (H, d),
                  "out_proj_w": (E, E), "out_proj_b": (E,)}
        if Cd:
            shapes.update(content_proj_w=(H, Cd, E), content_proj_b=(H, Cd))
        for k, s in shapes.items():
            if out[k].shape != s:
                raise ValueError(f"{k} has shape {out[k].shape}, expected {s}")
        return out

    def invalidate(self) -> None:
        """Drop device copies (call after mutating the arrays)."""
        self._device.clear()

    @classmethod
    def from_packed(cls, p: dict) -> "WaveAttnWeights":
        H = p["harmonic_raw"].shape[0]
        E = p["out_proj_w"].shape[0]
        heads = []
        for h in range(H):
            cw = p.get("content_proj_w")
            heads.append(WaveAttnHeadWeights(
                float(p["harmonic_raw"][h]), p["phase_proj_w"][h], p["phase_proj_b"][h],
                p["v_proj_w"][h], p["v_proj_b"][h],
                cw[h] if cw is not None else np.zeros((0, E), np.float32),
                p["content_proj_b"][h] if cw is not None else np.zeros((0,), np.float32)))
        return cls(heads, p["out_proj_w"], p["out_proj_b"])


class Rng:
    """xorshift64 state of src/common/rng.rs:5-12 (seed used as the state)."""

    def __init__(self, seed: int):
        self.state = int(seed) & 0xFFFFFFFFFFFFFFFF


def init_block_attn(rng: Rng, n_head: int, n_embd: int, content_dim: int) -> WaveAttnWeights:
    """src/common/wave_model.rs:57-81: the reference's attention initialiser,
    consuming ``rng`` in the reference's draw order."""
    if n_embd % n_head:
        raise ValueError("n_embd must be a multiple of n_head")
    d = n_embd // n_head
    p = {
        "harmonic_raw": np.empty(n_head, np.float32),
        "phase_proj_w": np.empty((n_head, 2, n_embd), np.float32),
        "phase_proj_b": np.empty((n_head, 2), np.float32),
        "v_proj_w": np.empty((n_head, d, d), np.float32),
        "v_proj_b": np.empty((n_head, d), np.float32),
        "content_proj_w": np.empty((n_head, content_dim, n_embd), np.float32) if content_dim else None,
        "content_proj_b": np.empty((n_head, content_dim), np.float32) if content_dim else None,
        "out_proj_w": np.empty((n_embd, n_embd), np.float32),
        "out_proj_b": np.empty(n_embd, np.float32),
    }
    st = C.c_uint64(rng.state)
    ptr = lambda a: None if a is None else a.ctypes.data
    _lib.call("wb_init_block_attn", C.byref(st), n_head, n_embd, content_dim,
              *[ptr(p[k]) for k in ("harmonic_raw", "phase_proj_w", "phase_proj_b", "v_proj_w", "v_proj_b",
                                    "content_proj_w", "content_proj_b", "out_proj_w", "out_proj_b")])
    rng.state = st.value
    return WaveAttnWeights.from_packed(p)


def gaussian_block_attn(seed: int, n_head: int, n_embd: int, content_dim: int = CONTENT_DIM,
                        std: float = 0.02) -> WaveAttnWeights:
    """Seeded N(0, std) weights with zero biases and the reference's harmonic
    init ln((h+1)/2) (wave_model.rs:73): the synthetic weights of the
    benchmark configurations."""
    g = np.random.default_rng(seed)
    d = n_embd // n_head
    n = lambda *s: (g.standard_normal(s, dtype=np.float32) * np.float32(std)).astype(np.float32)
    p = {
        "harmonic_raw": np.log((np.arange(n_head, dtype=np.float32) + 1) * np.float32(0.5)).astype(np.float32),
        "phase_proj_w": n(n_head, 2, n_embd),
        "phase_proj_b": np.zeros((n_head, 2), np.float32),
        "v_proj_w": n(n_head, d, d),
        "v_proj_b": np.zeros((n_head, d), np.float32),
        "content_proj_w": n(n_head, content_dim, n_embd) if content_dim else None,
        "content_proj_b": np.zeros((n_head, content_dim), np.float32) if content_dim else None,
        "out_proj_w": n(n_embd, n_embd),
        "out_proj_b": np.zeros(n_embd, np.float32),
    }
    return WaveAttnWeights.from_packed(p)
