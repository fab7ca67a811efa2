"""The serve-tier layer around the attention, on the GPU.

Host-side mirror of src/common/kv_cache.rs ``prefill`` (:93-236) and
``forward_one`` (:241-381): per layer LayerNorm -> wave attention (the KV
cache of ``kv_cache.py``) and LayerNorm -> the dual-maestro Kerr-ODE FFN
(ffn.rs:39-230 as those functions call it: frozen ODE, no memory), the
parallel residual ``hidden += attn + ffn``, then the final LayerNorm and
``phase_native_decode`` or the lm_head.  Every step runs in the CUDA
library (``wb_layer_norm``, ``wb_ffn_forward``, ``wb_embed``,
``wb_residual_add``, ``wb_phase_native_decode`` / ``wb_lm_head``); torch
only holds the device tensors.

``KerrFfnWeights`` mirrors ``KerrDualMaestroWeights`` (model.rs; the
initialiser's shapes at wave_model.rs:134-170).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from .attn import PATHS
from .runtime import Context, default_context, is_torch, ptr_of
from .weights import WaveAttnWeights

try:
    import torch
except Exception:  # pragma: no cover
    torch = None


@dataclass
class KerrFfnWeights:
    """One block's FFN: maestro_in / maestro_out (squeeze [M][E] + [M],
    process_1 [E][M] + [E]), the Kerr ODE (KerrWeights: gamma_raw, omega,
    alpha, beta, rk4_n_steps, phase_correction, rk4_weights) and out_proj
    (dense [E][E] + [E], or ``out_groups`` block-diagonal groups)."""
    mi_squeeze_w: np.ndarray
    mi_squeeze_b: np.ndarray
    mi_process_w: np.ndarray
    mi_process_b: np.ndarray
    mo_squeeze_w: np.ndarray
    mo_squeeze_b: np.ndarray
    mo_process_w: np.ndarray
    mo_process_b: np.ndarray
    gamma_raw: np.ndarray
    omega: np.ndarray
    alpha: float
    beta: float
    rk4_steps: int
    phase_correction: np.ndarray
    rk4_weights: np.ndarray
    out_w: np.ndarray          # dense [E][E]; block-diagonal: the groups' [gs][gs] + [gs] packed in order
    out_b: np.ndarray | None   # dense [E]; None for block-diagonal
    out_groups: int = 1
    use_corrector: bool = True
    _device: dict = field(default_factory=dict, repr=False, compare=False)

    @property
    def n_embd(self) -> int:
        return int(np.shape(self.mi_process_b)[0])

    @property
    def maestro_dim(self) -> int:
        return int(np.shape(self.mi_squeeze_b)[0])

    def packed(self) -> dict:
        f = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
        d = {k: f(getattr(self, k)) for k in (
            "mi_squeeze_w", "mi_squeeze_b", "mi_process_w", "mi_process_b", "mo_squeeze_w", "mo_squeeze_b",
            "mo_process_w", "mo_process_b", "gamma_raw", "omega", "phase_correction", "rk4_weights", "out_w",
            "out_b")}
        d.update(n_embd=self.n_embd, maestro_dim=self.maestro_dim, rk4_steps=int(self.rk4_steps),
                 use_corrector=int(bool(self.use_corrector)), out_groups=int(self.out_groups),
                 alpha=float(self.alpha), beta=float(self.beta))
        return d


def gaussian_ffn(seed: int, n_embd: int, maestro_dim: int = 16, *, out_groups: int = 1, rk4_steps: int = 16,
                 alpha: float = 0.1, beta: float = 0.2, std: float = 0.02, use_corrector: bool = True,
                 phase_correction_std: float = 0.0) -> KerrFfnWeights:
    """Seeded synthetic FFN weights: N(0, std) linear weights and biases of
    0.02 std, the reference initialiser's ODE constants (wave_model.rs:
    134-145: gamma_raw = ln(e^0.1 - 1), omega = (k+1)/n_bands, RK4 weights
    1/6, 1/3, 1/3, 1/6) and an optional random corrector plate."""
    g = np.random.default_rng(seed)
    E, M, nb = n_embd, maestro_dim, n_embd // 2
    n = lambda *s: (g.standard_normal(s) * std).astype(np.float32)
    gs = E // out_groups
    if out_groups == 1:
        out_w, out_b = n(E, E), n(E)
    else:
        out_w, out_b = np.concatenate([np.concatenate([n(gs, gs).ravel(), n(gs)]) for _ in range(out_groups)]), None
    return KerrFfnWeights(
        n(M, E), n(M), n(E, M), n(E), n(M, E), n(M), n(E, M), n(E),
        np.full(nb, np.log(np.expm1(np.float32(0.1))), np.float32),
        ((np.arange(nb, dtype=np.float32) + 1) / np.float32(nb)).astype(np.float32),
        alpha, beta, rk4_steps,
        (g.standard_normal(nb) * phase_correction_std).astype(np.float32),
        np.array([1 / 6, 1 / 3, 1 / 3, 1 / 6], np.float32), out_w, out_b, out_groups, use_corrector)


class FfnLayer:
    """wb_ffn_layer: a KerrFfnWeights uploaded to one context's device."""

    def __init__(self, ctx: Context, w: KerrFfnWeights):
        p = w.packed()
        g = lambda k: None if p[k] is None else p[k].ctypes.data
        desc = _lib.FfnWeightsDesc(p["n_embd"], p["maestro_dim"], p["rk4_steps"], p["use_corrector"],
                                   p["out_groups"], *[g(k) for k in (
                                       "mi_squeeze_w", "mi_squeeze_b", "mi_process_w", "mi_process_b",
                                       "mo_squeeze_w", "mo_squeeze_b", "mo_process_w", "mo_process_b",
                                       "gamma_raw", "omega")],
                                   p["alpha"], p["beta"], g("phase_correction"), g("rk4_weights"), g("out_w"),
                                   g("out_b"))
        h = C.c_void_p()
        _lib.call("wb_ffn_layer_create", ctx.handle, C.byref(desc), C.byref(h))
        self.ctx, self.handle, self.n_embd = ctx, h, p["n_embd"]
        ctx.adopt(self)

    def close(self) -> None:
        if self.handle:
            _lib.lib().wb_ffn_layer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def device_ffn(w, ctx: Context) -> FfnLayer:
    if isinstance(w, FfnLayer):
        return w
    lay = w._device.get(id(ctx))
    if lay is None or lay.ctx is not ctx or not lay.handle:
        lay = w._device[id(ctx)] = FfnLayer(ctx, w)
    return lay


class Agc:
    """agc.rs OdeAgc on the device (OdeAgc::new() is alpha = beta = 0.1).
    The reference keeps one process-wide instance that every FFN call
    updates; share one Agc between the calls that should see each other."""

    def __init__(self, ctx: Context | None = None, alpha: float = 0.1, beta: float = 0.1):
        self.ctx = ctx or default_context(0)
        h = C.c_void_p()
        _lib.call("wb_agc_create", self.ctx.handle, C.c_float(alpha), C.c_float(beta), C.byref(h))
        self.handle = h
        self.ctx.adopt(self)

    def state(self) -> dict:
        v = np.empty(8, np.float32)
        _lib.call("wb_agc_read", self.handle, v.ctypes.data)
        keys = ("ema_mean", "ema_var", "headroom", "decay", "min_threshold", "max_threshold", "threshold", "count")
        return dict(zip(keys, (float(x) for x in v)))

    def close(self) -> None:
        if self.handle:
            _lib.lib().wb_agc_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _arr(x):
    if is_torch(x):
        return x if (x.dtype == torch.float32 and x.is_contiguous()) else x.contiguous().float()
    return np.ascontiguousarray(x, np.float32)


def _like(x, shape):
    if is_torch(x):
        return torch.empty(shape, dtype=torch.float32, device=x.device)
    return np.empty(shape, np.float32)


def _ctx_for(x, ctx):
    if ctx is None:
        dev = x.device.index if (is_torch(x) and x.is_cuda) else 0
        ctx = default_context(dev or 0)
    return ctx


def ffn_forward(ffn, agc: Agc, x, *, rows_per_call: int | None = None, path: str = "tensor",
                ctx: Context | None = None, out=None):
    """ffn.rs:39-230 on rows x [..., E]: ``rows_per_call`` rows per reference
    call (default: all rows are one call), observed by ``agc`` in order."""
    x = _arr(x)
    ctx = _ctx_for(x, ctx)
    lay = device_ffn(ffn, ctx)
    E = lay.n_embd
    if x.shape[-1] != E:
        raise ValueError(f"x has {x.shape[-1]} features, the FFN {E}")
    rows = int(np.prod(x.shape[:-1])) if x.ndim > 1 else 1
    y = _like(x, tuple(x.shape)) if out is None else out
    ctx.use_torch_stream(x, y)
    _lib.call("wb_ffn_forward", ctx.handle, lay.handle, agc.handle, ptr_of(x), rows, int(rows_per_call or rows),
              PATHS[path], ptr_of(y))
    return y


def layer_norm(x, weight, bias, *, ctx: Context | None = None, out=None):
    """model.rs:154 over the last axis."""
    x = _arr(x)
    ctx = _ctx_for(x, ctx)
    n = int(x.shape[-1])
    w, b = _arr(weight), _arr(bias)
    y = _like(x, tuple(x.shape)) if out is None else out
    ctx.use_torch_stream(x, y)
    _lib.call("wb_layer_norm", ctx.handle, ptr_of(x), int(np.prod(x.shape[:-1])) if x.ndim > 1 else 1, n,
              ptr_of(w), ptr_of(b), ptr_of(y))
    return y


def residual_add(hidden, a, b, *, ctx: Context | None = None):
    """hidden += a + b (kv_cache.rs:220); device tensors."""
    ctx = _ctx_for(hidden, ctx)
    ctx.use_torch_stream(hidden)
    _lib.call("wb_residual_add", ctx.handle, ptr_of(hidden), ptr_of(a), ptr_of(b), int(hidden.numel()))
    return hidden


def embed(tokens, wpe_index, wte, wpe=None, *, ctx: Context | None = None, out=None):
    """hidden = wte[tokens] + wpe[wpe_index] (wpe row only below its length);
    wte / wpe device tensors.  Prefill passes the token ids as wpe_index
    (kv_cache.rs:108-110), forward_one the positions (:254-256)."""
    ctx = _ctx_for(wte, ctx)
    tok = tokens if is_torch(tokens) else np.ascontiguousarray(tokens, np.int32)
    idx = wpe_index if is_torch(wpe_index) else np.ascontiguousarray(wpe_index, np.int32)
    n = int(tok.shape[0])
    V, E = int(wte.shape[0]), int(wte.shape[1])
    y = torch.empty((n, E), dtype=torch.float32, device=wte.device) if out is None else out
    ctx.use_torch_stream(wte, y)
    _lib.call("wb_embed", ctx.handle, ptr_of(tok, np.int32), ptr_of(idx, np.int32), n, ptr_of(wte), V,
              ptr_of(wpe), 0 if wpe is None else int(wpe.shape[0]), E, ptr_of(y))
    return y


def phase_native_decode(hidden, corrector, wte, *, path: str = "tensor", ctx: Context | None = None):
    """kv_cache.rs:18-33 for rows hidden [n][E] -> logits [n][vocab]."""
    ctx = _ctx_for(wte, ctx)
    hidden = _arr(hidden)
    n, E = (1, int(hidden.shape[0])) if hidden.ndim == 1 else (int(hidden.shape[0]), int(hidden.shape[1]))
    V = int(wte.shape[0])
    y = _like(hidden, (n, V))
    ctx.use_torch_stream(wte, y)
    _lib.call("wb_phase_native_decode", ctx.handle, ptr_of(hidden), n, E, ptr_of(corrector), ptr_of(wte), V,
              PATHS[path], ptr_of(y))
    return y


def lm_head(hidden, w, *, path: str = "tensor", ctx: Context | None = None):
    """kv_cache.rs:365-378 for rows hidden [n][E] -> logits [n][vocab]."""
    ctx = _ctx_for(w, ctx)
    hidden = _arr(hidden)
    n, E = (1, int(hidden.shape[0])) if hidden.ndim == 1 else (int(hidden.shape[0]), int(hidden.shape[1]))
    V = int(w.shape[0])
    y = _like(hidden, (n, V))
    ctx.use_torch_stream(w, y)
    _lib.call("wb_lm_head", ctx.handle, ptr_of(hidden), n, E, ptr_of(w), V, PATHS[path], ptr_of(y))
    return y


@dataclass
class ServeBlock:
    """WaveBlockWeights (block.rs:17-27): ln, ln_ffn, attention, FFN."""
    ln_w: np.ndarray
    ln_b: np.ndarray
    ln_ffn_w: np.ndarray
    ln_ffn_b: np.ndarray
    attn: WaveAttnWeights
    ffn: KerrFfnWeights


@dataclass
class ServeModel:
    """The parts of WavePacketModel the serve loop reads (wave_model.rs:
    110-230): wte [vocab][E], wpe [n_pos][E] (may be empty), the blocks,
    ln_f, and either the output corrector (phase_native) or lm_head."""
    wte: np.ndarray
    wpe: np.ndarray | None
    blocks: list
    ln_f_w: np.ndarray
    ln_f_b: np.ndarray
    output_corrector: np.ndarray | None = None  # phase_native when set
    lm_head: np.ndarray | None = None


class ServeSession:
    """kv_cache.rs prefill / forward_one for a batch of requests on one GPU:
    a KV cache slot per request, one Agc for all FFN calls (the reference's
    process-wide AGC; a batch visits it layer by layer, request by request,
    which is one of the orders concurrent reference requests can take)."""

    def __init__(self, model: ServeModel, *, max_seqs: int, max_ctx: int, ctx: Context | None = None,
                 path: str = "tensor", n_pages: int | None = None):
        from .kv_cache import KvCache
        from .runtime import AttnLayer
        if torch is None:
            raise ImportError("the serve session keeps its tables in torch device tensors")
        self.ctx = ctx or default_context(0)
        self.path = path
        dev = torch.device("cuda", self.ctx.device)
        t = lambda a: None if a is None or np.size(a) == 0 else torch.as_tensor(np.ascontiguousarray(a, np.float32), device=dev)
        self.wte, self.wpe = t(model.wte), t(model.wpe)
        self.ln_f = (t(model.ln_f_w), t(model.ln_f_b))
        self.corrector, self.lm_head = t(model.output_corrector), t(model.lm_head)
        self.blocks = [(t(b.ln_w), t(b.ln_b), t(b.ln_ffn_w), t(b.ln_ffn_b), AttnLayer(self.ctx, b.attn),
                        FfnLayer(self.ctx, b.ffn)) for b in model.blocks]
        a0 = model.blocks[0].attn
        self.E, self.H = a0.n_embd, a0.n_head
        self.cache = KvCache(len(model.blocks), self.H, self.E // self.H, max_seqs=max_seqs, max_ctx=max_ctx,
                             ctx=self.ctx, n_pages=n_pages)
        self.agc = Agc(self.ctx)
        self.dev = dev

    def _layers(self, hidden, n_seq, T, seq_ids, prefill: bool):
        E = self.E
        for l, (lnw, lnb, lfw, lfb, attn, ffn) in enumerate(self.blocks):
            normed = layer_norm(hidden, lnw, lnb, ctx=self.ctx)
            if prefill:
                a = self.cache.prefill(l, attn, normed.view(n_seq, T, E), seq_ids, path=self.path).view(-1, E)
            else:
                a = self.cache.forward_one(l, attn, normed, seq_ids, path=self.path)
            normed_ffn = layer_norm(hidden, lfw, lfb, ctx=self.ctx)
            f = ffn_forward(ffn, self.agc, normed_ffn, rows_per_call=T, path=self.path, ctx=self.ctx)
            residual_add(hidden, a, f, ctx=self.ctx)
        return hidden

    def _decode(self, rows):
        normed = layer_norm(rows, *self.ln_f, ctx=self.ctx)
        if self.corrector is not None:
            return phase_native_decode(normed, self.corrector, self.wte, path=self.path, ctx=self.ctx)
        return lm_head(normed, self.lm_head, path=self.path, ctx=self.ctx)

    def prefill(self, tokens, seq_ids):
        """kv_cache.rs:93-236 for each request (rows of tokens [n_seq][T]):
        logits of every request's last position [n_seq][vocab]."""
        tok = torch.as_tensor(np.ascontiguousarray(tokens, np.int32), device=self.dev)
        n_seq, T = tok.shape
        flat = tok.reshape(-1).contiguous()
        hidden = embed(flat, flat, self.wte, self.wpe, ctx=self.ctx)  # prefill: wpe row = token id
        ids = np.ascontiguousarray(seq_ids, np.int32)
        self._layers(hidden, n_seq, T, ids, True)
        return self._decode(hidden.view(n_seq, T, self.E)[:, T - 1].contiguous())

    def capture_decode(self, seq_ids):
        """Capture one forward_one step for the slots ``seq_ids`` in a CUDA
        graph (every launch of every layer; tokens and positions through
        static device buffers).  Call after a prefill has sized the context's
        workspaces; then ``forward_one_graph`` replays it."""
        ids = torch.as_tensor(np.ascontiguousarray(seq_ids, np.int32), device=self.dev)
        n = int(ids.shape[0])
        self._g_tok = torch.zeros(n, dtype=torch.int32, device=self.dev)
        self._g_pos = torch.zeros(n, dtype=torch.int32, device=self.dev)
        self._g_ids = ids
        prev = torch.cuda.current_stream(self.dev)
        torch.cuda.synchronize(self.dev)
        self._graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(self._graph):
                hidden = embed(self._g_tok, self._g_pos, self.wte, self.wpe, ctx=self.ctx)
                self._layers(hidden, n, 1, self._g_ids, False)
                self._g_logits = self._decode(hidden)
        finally:
            self.ctx.set_stream(prev.cuda_stream)

    def forward_one_graph(self, tokens, positions):
        """forward_one through the captured graph: logits [n][vocab] (the
        graph's static output tensor, overwritten by the next replay)."""
        self._g_tok.copy_(torch.as_tensor(np.ascontiguousarray(tokens, np.int32)))
        self._g_pos.copy_(torch.as_tensor(np.ascontiguousarray(positions, np.int32)))
        self._graph.replay()
        return self._g_logits

    def forward_one(self, tokens, positions, seq_ids):
        """kv_cache.rs:241-381: one new token per request -> logits [n][vocab]."""
        tok = torch.as_tensor(np.ascontiguousarray(tokens, np.int32), device=self.dev)
        pos = torch.as_tensor(np.ascontiguousarray(positions, np.int32), device=self.dev)
        hidden = embed(tok, pos, self.wte, self.wpe, ctx=self.ctx)
        ids = np.ascontiguousarray(seq_ids, np.int32)
        self._layers(hidden, int(tok.shape[0]), 1, ids, False)
        return self._decode(hidden)
