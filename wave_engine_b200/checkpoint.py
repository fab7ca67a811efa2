"""Attention weights out of the reference's WCHK checkpoints.

The file format is src/common/checkpoint.rs:20-87 (writer) / :89-260
(reader): "WCHK", a u32 version (1-4), the config u32s (n_bands, n_head,
n_layers, maestro_dim, block_size, rk4_steps, and from v2 out_proj_groups),
from v3 a u32 feature-flag word, from v4 the f32 chi, then vocab_size u64,
iter u64, lr f32, rng_state u64, adam_t u64 and three f32 arrays of N
(Adam m, Adam v, the parameters), N following from the file size.

The parameter vector is src/common/wave_model.rs:335-399
``flatten_params_ex``: per block the two LayerNorms, the two maestros, the
FFN out_proj (dense or block-diagonal by ``out_proj_groups``), the ODE
fields (feature bit 0, with the RK4 weights under bit 2), one
``harmonic_raw`` per head (bit 3) and, under bit 4 (``learnable_attn``), each
head's phase / value / content projections followed by the block's
attention out_proj; the model-level tail (layer scales, ln_f, the decoder)
comes after the last block and is not read here.

``content_dim`` is not stored in the file (the reference rebuilds the model
from its CLI flags and ``unflatten_params_ex``s into it): pass the one the
model was trained with (16, or 0 for --freeze-ode).  Without bit 3 the
harmonics are the initialiser's ln((h+1)/2) (wave_model.rs:73).
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass

import numpy as np

from .weights import CONTENT_DIM, WaveAttnWeights

FLAG_LEARNABLE_ODE = 1 << 0
FLAG_LAYER_SCALE = 1 << 1
FLAG_RK4_WEIGHTS = 1 << 2
FLAG_DYN_HARMONICS = 1 << 3
FLAG_LEARNABLE_ATTN = 1 << 4


@dataclass
class WchkHeader:
    version: int
    n_bands: int
    n_head: int
    n_layers: int
    maestro_dim: int
    block_size: int
    rk4_steps: int
    out_proj_groups: int
    flags: int
    chi: float
    vocab_size: int
    iter: int
    lr: float
    rng_state: int
    adam_t: int
    n_params: int
    params_offset: int  # byte offset of the parameter array in the file

    @property
    def n_embd(self) -> int:
        return 2 * self.n_bands


def read_wchk_header(path: str) -> WchkHeader:
    """checkpoint.rs:89-227: the header fields and where the parameters are."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        if f.read(4) != b"WCHK":
            raise ValueError(f"{path}: not a WCHK checkpoint")
        (version,) = struct.unpack("<I", f.read(4))
        if not 1 <= version <= 4:
            raise ValueError(f"{path}: unknown WCHK version {version}")
        cfg = struct.unpack("<6I", f.read(24))
        groups = struct.unpack("<I", f.read(4))[0] if version >= 2 else 1
        flags = struct.unpack("<I", f.read(4))[0] if version >= 3 else 0
        chi = struct.unpack("<f", f.read(4))[0] if version >= 4 else 0.0
        vocab, it = struct.unpack("<QQ", f.read(16))
        (lr,) = struct.unpack("<f", f.read(4))
        (rng_state,) = struct.unpack("<Q", f.read(8))
        (adam_t,) = struct.unpack("<Q", f.read(8))
        data_off = f.tell()
    data = size - data_off
    if data < 0 or data % 12:
        raise ValueError(f"{path}: {data} data bytes is not 3 arrays of f32")
    n = data // 12
    return WchkHeader(version, *cfg, groups, flags, chi, vocab, it, lr, rng_state, adam_t, n, data_off + 8 * n)


def _block_fields(h: WchkHeader, content_dim: int, learnable_attn: bool):
    """(name, shape) of one block's slice of flatten_params_ex, in order."""
    E, M, H, nb = h.n_embd, h.maestro_dim, h.n_head, h.n_bands
    if E % H:
        raise ValueError("n_embd is not a multiple of n_head")
    if h.out_proj_groups < 1 or E % h.out_proj_groups:
        raise ValueError("n_embd is not a multiple of out_proj_groups")
    d, gs = E // H, E // h.out_proj_groups
    f = [("ln.weight", (E,)), ("ln.bias", (E,)), ("ln_ffn.weight", (E,)), ("ln_ffn.bias", (E,))]
    for m in ("maestro_in", "maestro_out"):
        f += [(f"{m}.squeeze.w", (M, E)), (f"{m}.squeeze.b", (M,)),
              (f"{m}.process_1.w", (E, M)), (f"{m}.process_1.b", (E,))]
    for g in range(h.out_proj_groups):  # out_proj.rs:53-66 (Dense is the one-group case)
        f += [(f"ffn.out_proj.{g}.w", (gs, gs)), (f"ffn.out_proj.{g}.b", (gs,))]
    if h.flags & FLAG_LEARNABLE_ODE:
        f += [("kerr.gamma_raw", (nb,)), ("kerr.alpha", ()), ("kerr.beta", ()), ("kerr.phase_correction", (nb,))]
        if h.flags & FLAG_RK4_WEIGHTS:
            f += [("kerr.rk4_weights", (4,))]
    if h.flags & FLAG_DYN_HARMONICS:
        f += [("attn.harmonic_raw", (H,))]
    if learnable_attn:
        for hh in range(H):
            f += [(f"attn.{hh}.phase_proj_w", (2, E)), (f"attn.{hh}.phase_proj_b", (2,)),
                  (f"attn.{hh}.v_proj_w", (d, d)), (f"attn.{hh}.v_proj_b", (d,)),
                  (f"attn.{hh}.content_proj_w", (content_dim, E)), (f"attn.{hh}.content_proj_b", (content_dim,))]
        f += [("attn.out_proj_w", (E, E)), ("attn.out_proj_b", (E,))]
    return f


def load_wchk_attention(path: str, content_dim: int = CONTENT_DIM, learnable_attn: bool | None = None):
    """The attention weights of every block of a WCHK checkpoint:
    ``(header, [WaveAttnWeights per block])``.

    ``learnable_attn`` defaults to the file's flag bit 4; pass True for
    checkpoints written with learnable attention before that bit existed
    (checkpoint.rs:199-203).  Checkpoints without learnable attention hold
    no attention weights (the model keeps its initialiser's), which raises
    ValueError."""
    h = read_wchk_header(path)
    la = bool(h.flags & FLAG_LEARNABLE_ATTN) if learnable_attn is None else learnable_attn
    if not la:
        raise ValueError(f"{path}: no learnable attention in this checkpoint (feature bit 4 unset)")
    fields = _block_fields(h, content_dim, True)
    per_block = sum(int(np.prod(s)) for _, s in fields)
    tail_min = 2 * h.n_embd  # ln_f at least follows the blocks
    if h.n_layers * per_block + tail_min > h.n_params:
        raise ValueError(f"{path}: {h.n_params} parameters cannot hold {h.n_layers} blocks of {per_block} "
                         f"(content_dim {content_dim}?)")
    params = np.fromfile(path, dtype="<f4", count=h.n_layers * per_block, offset=h.params_offset)
    H, E = h.n_head, h.n_embd
    out = []
    off = 0
    for _ in range(h.n_layers):
        blk = {}
        for name, shape in fields:
            k = int(np.prod(shape))
            blk[name] = params[off:off + k].reshape(shape).astype(np.float32)
            off += k
        harm = (blk["attn.harmonic_raw"] if "attn.harmonic_raw" in blk else
                np.log((np.arange(H, dtype=np.float32) + 1) * np.float32(0.5)).astype(np.float32))
        p = {
            "harmonic_raw": np.ascontiguousarray(harm, np.float32),
            "phase_proj_w": np.stack([blk[f"attn.{i}.phase_proj_w"] for i in range(H)]),
            "phase_proj_b": np.stack([blk[f"attn.{i}.phase_proj_b"] for i in range(H)]),
            "v_proj_w": np.stack([blk[f"attn.{i}.v_proj_w"] for i in range(H)]),
            "v_proj_b": np.stack([blk[f"attn.{i}.v_proj_b"] for i in range(H)]),
            "content_proj_w": np.stack([blk[f"attn.{i}.content_proj_w"] for i in range(H)]) if content_dim else None,
            "content_proj_b": np.stack([blk[f"attn.{i}.content_proj_b"] for i in range(H)]) if content_dim else None,
            "out_proj_w": blk["attn.out_proj_w"],
            "out_proj_b": blk["attn.out_proj_b"],
        }
        w = WaveAttnWeights.from_packed(p)
        if w.n_embd != E:
            raise ValueError("inconsistent n_embd")
        out.append(w)
    return h, out
