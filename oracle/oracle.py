"""ctypes wrapper of the CPU oracle (``oracle/wave_oracle.c``).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, by
``__graft_entry__.smoke()`` and by the CPU-baseline leg of ``bench.py``, as
the checker and the timed CPU restatement of the reference.  The product
path (``wave_engine_b200``) never imports it.

Parity status: unpinned by reference outputs (the Rust reference cannot be
built here and ships no forward golden vectors); pinned by hand-derived
known-answer cases, see ``tests/golden/make_golden.py``.

Weights are a dict of numpy float32 arrays in the reference layouts:
    harmonic_raw [H]; phase_proj_w [H,2,E]; phase_proj_b [H,2];
    v_proj_w [H,d,d]; v_proj_b [H,d]; content_proj_w [H,C,E] or None;
    content_proj_b [H,C] or None; out_proj_w [E,E]; out_proj_b [E].
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build as _build

_F = C.POINTER(C.c_float)
_I = C.POINTER(C.c_int)


class _Weights(C.Structure):
    _fields_ = [
        ("n_embd", C.c_int), ("n_head", C.c_int), ("content_dim", C.c_int),
        ("harmonic_raw", _F), ("phase_w", _F), ("phase_b", _F), ("v_w", _F), ("v_b", _F),
        ("content_w", _F), ("content_b", _F), ("out_w", _F), ("out_b", _F),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        l = C.CDLL(str(path))
        l.wo_attn_forward.argtypes = [C.POINTER(_Weights), _F, C.c_int, _F, _F, _F, _F, C.c_int]
        l.wo_attn_forward_batch.argtypes = [C.POINTER(_Weights), _F, C.c_int, C.c_int, _F, C.c_int]
        l.wo_kv_prefill.argtypes = [C.POINTER(_Weights), _F, C.c_int, _F, _F, _I, _F, C.c_int, _I]
        l.wo_kv_decode.argtypes = [C.POINTER(_Weights), _F, _F, _F, _I, _F, C.c_int, _I]
        l.wo_phase_to_bucket.argtypes = [C.c_float]
        l.wo_phase_to_bucket.restype = C.c_int
        l.wo_softplus.argtypes = [C.c_float]
        l.wo_softplus.restype = C.c_float
        l.wo_init_block_attn.argtypes = [C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_int] + [_F] * 9
        l.wo_dot_attn_forward.argtypes = [C.c_int, C.c_int, _F, _F, _F, _F, _F, C.c_int, _F]
        l.wo_attn_backward_full.argtypes = [C.POINTER(_Weights), _F, C.c_int, _F] + [_F] * 10
        l.wo_bwd_out_proj.argtypes = [_F, _F, _F, C.c_int, C.c_int, _F, _F, _F]
        l.wo_bwd_value_aggregation.argtypes = [_F, _F, _F, C.c_int, C.c_int, _F, _F]
        l.wo_bwd_softmax.argtypes = [_F, _F, C.c_int, _F]
        l.wo_bwd_phase_projection.argtypes = [_F, _F, _F, _F, C.c_int, C.c_int, _F, _F, _F]
        l.wo_bwd_value_projection.argtypes = [_F, _F, C.c_int, C.c_int, C.c_int, C.c_int, _F, _F, _F, _F]
        l.wo_bwd_combine.argtypes = [_F, _F, _F, C.c_int, C.c_int, C.c_int, _F]
        _lib = l
    return _lib


def _fp(a):
    return None if a is None else a.ctypes.data_as(_F)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


class _Packed:
    """Keeps contiguous float32 copies alive while the C struct points at them."""

    def __init__(self, w: dict):
        self.arrs = {k: _f32(w.get(k)) for k in (
            "harmonic_raw", "phase_proj_w", "phase_proj_b", "v_proj_w", "v_proj_b",
            "content_proj_w", "content_proj_b", "out_proj_w", "out_proj_b")}
        a = self.arrs
        H = a["harmonic_raw"].shape[0]
        E = a["out_proj_w"].shape[0]
        cw = a["content_proj_w"]
        Cd = 0 if cw is None or cw.size == 0 else cw.shape[1]
        if Cd == 0:
            a["content_proj_w"] = a["content_proj_b"] = None
        self.H, self.E, self.C = H, E, Cd
        self.s = _Weights(E, H, Cd, _fp(a["harmonic_raw"]), _fp(a["phase_proj_w"]), _fp(a["phase_proj_b"]),
                          _fp(a["v_proj_w"]), _fp(a["v_proj_b"]), _fp(a["content_proj_w"]),
                          _fp(a["content_proj_b"]), _fp(a["out_proj_w"]), _fp(a["out_proj_b"]))


def softplus(x: float) -> float:
    return float(lib().wo_softplus(C.c_float(x)))


def phase_to_bucket(theta) -> np.ndarray:
    t = np.asarray(theta, dtype=np.float32)
    f = np.vectorize(lambda v: lib().wo_phase_to_bucket(C.c_float(v)), otypes=[np.int32])
    return f(t)


def attn_forward(w: dict, x: np.ndarray, *, want_att_w: bool = False, phase_override=None,
                 n_threads: int = 1):
    """wave_attention_forward for one sequence x [T,E] (attn.rs:90-305).

    Returns (y [T,E], att_w [H,T,T] or None, phases [H,T])."""
    p = _Packed(w)
    x = _f32(x)
    T = x.shape[0]
    y = np.empty((T, p.E), np.float32)
    aw = np.empty((p.H, T, T), np.float32) if want_att_w else None
    ph = np.empty((p.H, T), np.float32)
    po = _f32(phase_override)
    rc = lib().wo_attn_forward(C.byref(p.s), _fp(x), T, _fp(y), _fp(aw), _fp(po), _fp(ph), n_threads)
    if rc != 0:
        raise RuntimeError("oracle wo_attn_forward failed")
    return y, aw, ph


def attn_forward_batch(w: dict, x: np.ndarray, n_threads: int | None = None) -> np.ndarray:
    """x [B,T,E] -> y [B,T,E]; (sequence, head) items on n_threads threads."""
    p = _Packed(w)
    x = _f32(x)
    B, T, _ = x.shape
    y = np.empty_like(x)
    nt = n_threads or os.cpu_count() or 1
    if lib().wo_attn_forward_batch(C.byref(p.s), _fp(x), B, T, _fp(y), nt) != 0:
        raise RuntimeError("oracle wo_attn_forward_batch failed")
    return y


class KvState:
    """One layer's cache of one sequence (kv_cache.rs:36-41 HeadCache per head)."""

    def __init__(self, n_head: int, head_dim: int, cap: int):
        self.cap = cap
        self.phases = np.zeros((n_head, cap), np.float32)
        self.buckets = np.zeros((n_head, cap), np.int32)
        self.values = np.zeros((n_head, cap, head_dim), np.float32)
        self.n = C.c_int(0)

    @property
    def n_cached(self) -> int:
        return self.n.value


def kv_prefill(w: dict, x: np.ndarray, cap: int) -> tuple[np.ndarray, KvState]:
    """Attention part of kv_cache.rs:121-193 for one prompt x [T,E]."""
    p = _Packed(w)
    x = _f32(x)
    T = x.shape[0]
    st = KvState(p.H, p.E // p.H, cap)
    y = np.empty((T, p.E), np.float32)
    rc = lib().wo_kv_prefill(C.byref(p.s), _fp(x), T, _fp(y), _fp(st.phases),
                             st.buckets.ctypes.data_as(_I), _fp(st.values), cap, C.byref(st.n))
    if rc != 0:
        raise RuntimeError("oracle wo_kv_prefill failed")
    return y, st


def kv_decode(w: dict, x: np.ndarray, st: KvState) -> np.ndarray:
    """Attention part of kv_cache.rs:263-335 for one new position x [E]."""
    p = _Packed(w)
    x = _f32(x)
    y = np.empty((p.E,), np.float32)
    rc = lib().wo_kv_decode(C.byref(p.s), _fp(x), _fp(y), _fp(st.phases), st.buckets.ctypes.data_as(_I),
                            _fp(st.values), st.cap, C.byref(st.n))
    if rc != 0:
        raise RuntimeError("oracle wo_kv_decode failed")
    return y


def init_block_attn(state: int, n_head: int, n_embd: int, content_dim: int) -> tuple[dict, int]:
    """wave_model.rs:57-81 on the xorshift64 stream; returns (weights, new state)."""
    d = n_embd // n_head
    w = {
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
    s = C.c_uint64(state)
    lib().wo_init_block_attn(C.byref(s), n_head, n_embd, content_dim,
                             *[_fp(w[k]) for k in ("harmonic_raw", "phase_proj_w", "phase_proj_b", "v_proj_w",
                                                   "v_proj_b", "content_proj_w", "content_proj_b",
                                                   "out_proj_w", "out_proj_b")])
    return w, s.value


def dot_attn_forward(w: dict, x: np.ndarray) -> np.ndarray:
    """Legacy dot-product attention (compute.rs:357-414) for one sequence x [T,E]; w as
    AttentionWeights.packed() (c_attn_w [3E][E], c_attn_b, c_proj_w [E][E], c_proj_b, n_head)."""
    x = _f32(x)
    T, E = x.shape
    y = np.empty((T, E), np.float32)
    ws = [_f32(w[k]) for k in ("c_attn_w", "c_attn_b", "c_proj_w", "c_proj_b")]
    if lib().wo_dot_attn_forward(int(w["n_head"]), E, *[_fp(a) for a in ws], _fp(x), T, _fp(y)) != 0:
        raise RuntimeError("oracle wo_dot_attn_forward failed")
    return y


# ---------------------------------------------------------------------------
# attention backward (attn_backward.rs, attn.rs:346-430)
# ---------------------------------------------------------------------------
def attn_backward_full(w: dict, x: np.ndarray, d_y: np.ndarray) -> dict:
    """wave_attention_backward_full (attn.rs:346-430) for one sequence x [T,E] and
    the output gradient d_y [T,E]: d_normed (the input gradient) and every weight
    gradient, in the layouts of WaveAttnWeights.packed()."""
    p = _Packed(w)
    x, d_y = _f32(x), _f32(d_y)
    T, E = x.shape
    H, Cd = p.H, p.C
    hd = E // H
    g = {"d_x": np.empty((T, E), np.float32), "out_proj_w": np.empty((E, E), np.float32),
         "out_proj_b": np.empty(E, np.float32), "phase_proj_w": np.empty((H, 2, E), np.float32),
         "phase_proj_b": np.empty((H, 2), np.float32), "v_proj_w": np.empty((H, hd, hd), np.float32),
         "v_proj_b": np.empty((H, hd), np.float32),
         "content_proj_w": np.empty((H, Cd, E), np.float32) if Cd else None,
         "content_proj_b": np.empty((H, Cd), np.float32) if Cd else None,
         "harmonic_raw": np.empty(H, np.float32)}
    rc = lib().wo_attn_backward_full(C.byref(p.s), _fp(x), T, _fp(d_y), _fp(g["d_x"]), _fp(g["out_proj_w"]),
                                     _fp(g["out_proj_b"]), _fp(g["phase_proj_w"]), _fp(g["phase_proj_b"]),
                                     _fp(g["v_proj_w"]), _fp(g["v_proj_b"]), _fp(g["content_proj_w"]),
                                     _fp(g["content_proj_b"]), _fp(g["harmonic_raw"]))
    if rc != 0:
        raise RuntimeError("oracle wo_attn_backward_full failed")
    return g


def bwd_out_proj(d_y, merged, w):
    """attn_backward.rs:17-53 -> (d_out, d_w, d_b)."""
    d_y, merged, w = _f32(d_y), _f32(merged), _f32(w)
    t, n = d_y.shape
    out = (np.empty((t, n), np.float32), np.empty((n, n), np.float32), np.empty(n, np.float32))
    lib().wo_bwd_out_proj(_fp(d_y), _fp(merged), _fp(w), n, t, *[_fp(a) for a in out])
    return out


def bwd_value_aggregation(d_head, att_w, v):
    """attn_backward.rs:72-105 -> (d_att_w, d_v)."""
    d_head, att_w, v = _f32(d_head), _f32(att_w), _f32(v)
    t, hd = d_head.shape
    out = (np.empty((t, t), np.float32), np.empty((t, hd), np.float32))
    lib().wo_bwd_value_aggregation(_fp(d_head), _fp(att_w), _fp(v), t, hd, *[_fp(a) for a in out])
    return out


def bwd_softmax(d_att_w, att_w):
    """attn_backward.rs:109-122 -> d_scores."""
    d_att_w, att_w = _f32(d_att_w), _f32(att_w)
    t = att_w.shape[0]
    out = np.empty((t, t), np.float32)
    lib().wo_bwd_softmax(_fp(d_att_w), _fp(att_w), t, _fp(out))
    return out


def bwd_phase_projection(d_phases, x, pw, pb):
    """attn_backward.rs:190-231 -> (d_x, d_w [2][n], d_b [2])."""
    d_phases, x, pw, pb = _f32(d_phases), _f32(x), _f32(pw), _f32(pb)
    t, n = x.shape
    out = (np.empty((t, n), np.float32), np.empty((2, n), np.float32), np.empty(2, np.float32))
    lib().wo_bwd_phase_projection(_fp(d_phases), _fp(x), _fp(pw), _fp(pb), n, t, *[_fp(a) for a in out])
    return out


def bwd_value_projection(d_v, x, offset, vw):
    """attn_backward.rs:237-263 -> (d_x, d_w [hd][hd], d_b [hd])."""
    d_v, x, vw = _f32(d_v), _f32(x), _f32(vw)
    t, hd = d_v.shape
    n = x.shape[1]
    out = (np.empty((t, n), np.float32), np.empty((hd, hd), np.float32), np.empty(hd, np.float32))
    lib().wo_bwd_value_projection(_fp(d_v), _fp(x), offset, hd, n, t, _fp(vw), *[_fp(a) for a in out])
    return out


def bwd_combine(dxp, dxv, dxc=None):
    """attn_backward.rs:299-326: [H][t][n] input gradients -> d_normed [t][n]."""
    dxp, dxv, dxc = _f32(dxp), _f32(dxv), _f32(dxc)
    H, t, n = dxp.shape
    out = np.empty((t, n), np.float32)
    lib().wo_bwd_combine(_fp(dxp), _fp(dxv), _fp(dxc), H, t, n, _fp(out))
    return out


# ---------------------------------------------------------------------------
# serve-tier layer around the attention (serve_oracle.c): LayerNorm, the
# dual-maestro Kerr-ODE FFN with its AGC, phase_native_decode / lm_head and
# the embedding, composed as kv_cache.rs prefill / forward_one
# ---------------------------------------------------------------------------
class AgcState(C.Structure):
    """agc.rs OdeAgc (the reference keeps one process-wide instance)."""
    _fields_ = [("ema_mean", C.c_float), ("ema_var", C.c_float), ("headroom", C.c_float), ("decay", C.c_float),
                ("min_threshold", C.c_float), ("max_threshold", C.c_float), ("threshold", C.c_float),
                ("count", C.c_int64)]


class _Ffn(C.Structure):
    _fields_ = [("n_embd", C.c_int), ("maestro_dim", C.c_int), ("out_groups", C.c_int), ("rk4_steps", C.c_int),
                ("use_corrector", C.c_int),
                ("mi_sq_w", _F), ("mi_sq_b", _F), ("mi_pr_w", _F), ("mi_pr_b", _F),
                ("mo_sq_w", _F), ("mo_sq_b", _F), ("mo_pr_w", _F), ("mo_pr_b", _F),
                ("gamma_raw", _F), ("omega", _F), ("alpha", C.c_float), ("beta", C.c_float),
                ("phase_correction", _F), ("rk4_w", _F), ("op_w", _F), ("op_b", _F)]


def _serve_lib():
    l = lib()
    if not getattr(l, "_serve_ready", False):
        l.wo_layer_norm.argtypes = [_F, C.c_int, _F, _F, _F]
        l.wo_agc_init.argtypes = [C.POINTER(AgcState), C.c_float, C.c_float]
        l.wo_ffn_forward.argtypes = [C.POINTER(_Ffn), C.POINTER(AgcState), _F, C.c_int, _F]
        l.wo_phase_native_decode.argtypes = [_F, _F, _F, C.c_int, C.c_int, _F]
        l.wo_lm_head.argtypes = [_F, _F, C.c_int, C.c_int, _F]
        l.wo_embed.argtypes = [_I, _I, C.c_int, _F, _F, C.c_int, C.c_int, _F]
        l._serve_ready = True
    return l


def agc_new(alpha: float = 0.1, beta: float = 0.1) -> AgcState:
    """agc.rs OdeAgc::new() (from_coupling(0.1, 0.1)) or from_coupling(alpha, beta)."""
    a = AgcState()
    _serve_lib().wo_agc_init(C.byref(a), alpha, beta)
    return a


def layer_norm(x: np.ndarray, w: np.ndarray, b: np.ndarray) -> np.ndarray:
    """model.rs:154 over the last axis."""
    x = _f32(x)
    w, b = _f32(w), _f32(b)
    n = x.shape[-1]
    xs = np.ascontiguousarray(x.reshape(-1, n))
    y = np.empty_like(xs)
    l = _serve_lib()
    for i in range(xs.shape[0]):
        l.wo_layer_norm(_fp(xs[i]), n, _fp(w), _fp(b), _fp(y[i]))
    return y.reshape(x.shape)


def ffn_forward(f: dict, agc: AgcState, x: np.ndarray) -> np.ndarray:
    """ffn.rs:39-230 as kv_cache.rs runs it (freeze_ode, stencil ODE, no
    memory) for ONE reference call over the rows of x [t][E] -> y [t][E];
    ``agc`` is updated in place.  ``f`` is KerrFfnWeights.packed()."""
    keep = {k: _f32(v) for k, v in f.items() if isinstance(v, np.ndarray)}
    E = int(f["n_embd"])
    s = _Ffn(E, int(f["maestro_dim"]), int(f["out_groups"]), int(f["rk4_steps"]), int(f["use_corrector"]),
             *[_fp(keep[k]) for k in ("mi_squeeze_w", "mi_squeeze_b", "mi_process_w", "mi_process_b",
                                      "mo_squeeze_w", "mo_squeeze_b", "mo_process_w", "mo_process_b",
                                      "gamma_raw", "omega")],
             float(f["alpha"]), float(f["beta"]), _fp(keep["phase_correction"]), _fp(keep["rk4_weights"]),
             _fp(keep["out_w"]), _fp(keep.get("out_b")))
    x = _f32(x)
    t = x.shape[0]
    y = np.empty((t, E), np.float32)
    if _serve_lib().wo_ffn_forward(C.byref(s), C.byref(agc), _fp(x), t, _fp(y)) != 0:
        raise RuntimeError("oracle wo_ffn_forward failed")
    return y


def phase_native_decode(hidden: np.ndarray, corrector: np.ndarray, wte: np.ndarray) -> np.ndarray:
    """kv_cache.rs:18-33 for one hidden row [E] -> logits [vocab]."""
    hidden, corrector, wte = _f32(hidden), _f32(corrector), _f32(wte)
    V, E = wte.shape
    out = np.empty(V, np.float32)
    _serve_lib().wo_phase_native_decode(_fp(hidden), _fp(corrector), _fp(wte), V, E // 2, _fp(out))
    return out


def lm_head(hidden: np.ndarray, w: np.ndarray) -> np.ndarray:
    """kv_cache.rs:365-378 for one hidden row."""
    hidden, w = _f32(hidden), _f32(w)
    V, E = w.shape
    out = np.empty(V, np.float32)
    _serve_lib().wo_lm_head(_fp(hidden), _fp(w), V, E, _fp(out))
    return out


def embed(tokens, wpe_index, wte: np.ndarray, wpe) -> np.ndarray:
    """kv_cache.rs:106-113 (prefill: the wpe row is the token id) and :252-256
    (forward_one: the position)."""
    tok = np.ascontiguousarray(tokens, np.int32)
    idx = np.ascontiguousarray(wpe_index, np.int32)
    wte = _f32(wte)
    wpe = _f32(wpe) if wpe is not None and np.size(wpe) else None
    E = wte.shape[1]
    out = np.empty((tok.shape[0], E), np.float32)
    _serve_lib().wo_embed(tok.ctypes.data_as(_I), idx.ctypes.data_as(_I), tok.shape[0], _fp(wte), _fp(wpe),
                          0 if wpe is None else wpe.shape[0], E, _fp(out))
    return out
