#!/usr/bin/env python3
"""Benchmark of the B200 wave-attention hot path (prefill + KV-cache decode).

Workload (the configuration the headline metric is quoted on): the 768-dim
production model -- n_embd 768, 12 heads of 64, 24 attention
layers -- with batch 32: a 1024-token prefill through all 24 layers, then 256
greedy decode steps, each one new position per sequence through all 24
layers.  One bench step is that whole job.  Weights are seeded N(0, 0.02)
(the reference's harmonic init for n_h), the per-layer attention inputs are
seeded N(0, 1) rows standing in for the LayerNorm output (synthetic data: no
datasets here).  Every per-layer input is 100 MB (prefill) and all inputs
(3 GB) are resident in HBM, larger than the 126 MB L2.

``value`` = (prefill + decode tokens of all ranks) / device time of a step
(CUDA events, max over ranks).  ``e2e`` = the same through the public API
with pinned HOST buffers (host->device copies of every layer's input and
device->host copies of every output inside the timed region).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Under torchrun each rank runs the full batch-32 job on its own GPU (the
attention forward shards by sequence with no data-path collective): weak
scaling.  ``--impl reference`` times the reference algorithm on the host CPU
(the C restatement in oracle/, the Rust reference cannot be built here) on a
bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "attn prefill tok/s + decode tok/s @768-dim, 1/2/4/8 GPU; % TC/HBM roofline"
CFG = dict(n_embd=768, n_head=12, head_dim=64, content_dim=16, n_layers=24, batch=32, seq_len=1024,
           decode_steps=256)
WORKLOAD = ("768-dim production model (12 heads x 64, 24 layers): batch 32, 1024-token prefill "
            "then 256 greedy KV-cache decode steps")


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def max_over_ranks(value: float, world: int, device=None) -> float:
    """Max of a per-rank number over all ranks (the step time of the slowest
    rank); the identity on one rank."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_output_stats(tensors, world: int, device=None):
    """Per-rank statistics of the rank's outputs -- [sum, sum of |y|, max |y|,
    count of non-finite values] over the given tensors -- gathered from every
    rank (all_gather: over NCCL on the GPUs, the only collective of the job
    besides the timing reduction).  Returns one list per rank, rank order."""
    import torch
    st = torch.zeros(4, dtype=torch.float64, device=device)
    for t in tensors:
        td = t.detach().to(torch.float64)
        fin = torch.isfinite(td)
        tf = torch.where(fin, td, torch.zeros_like(td))
        st[0] += tf.sum()
        st[1] += tf.abs().sum()
        if tf.numel():
            st[2] = torch.maximum(st[2], tf.abs().max())
        st[3] += (~fin).sum().to(torch.float64)
    if world == 1:
        return [[float(v) for v in st.tolist()]]
    import torch.distributed as dist
    out = [torch.zeros_like(st) for _ in range(world)]
    dist.all_gather(out, st)
    return [[float(v) for v in o.tolist()] for o in out]


def shard_sequences(ctx_lens, world: int):
    """Split sequences over ranks so every rank gets about the same number of
    cached keys (greedy: longest sequence to the least loaded rank).  Returns
    one sorted index list per rank; every index appears exactly once."""
    loads = [0] * world
    shards = [[] for _ in range(world)]
    for i in sorted(range(len(ctx_lens)), key=lambda j: (-ctx_lens[j], j)):
        r = min(range(world), key=lambda q: (loads[q], q))
        shards[r].append(i)
        loads[r] += ctx_lens[i]
    return [sorted(s) for s in shards]


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class Clocks:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and parts[1].isdigit():
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = sorted(int(r[1]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace('.', '').isdigit())}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# algorithmic work of the hot path (FLOP and byte formulas)
# ---------------------------------------------------------------------------
def decode_bytes_exact(bucket_slots, T0, S, H, hd, first=0):
    """Algorithmic HBM bytes of the decode attention launches of steps
    first..S-1: for each new position p (p = T0+first..T0+S-1) of each
    (layer, seq, head), the phase+bucket of all p cached keys (5 B each) plus
    the fp32 value row (4*hd B) of each key the mask lets through (bucket
    b-1..b+1 or the previous position).  bucket_slots is a numpy u8 array
    [L][B][H][T0+S] of the cache's buckets after the step."""
    import numpy as np
    b = bucket_slots.astype(np.int64)
    L, B, Hh, n = b.shape
    onehot = np.zeros((L, B, Hh, n + 1, 8), np.int32)
    onehot[:, :, :, 1:, :] = (b[..., None] == np.arange(8)).astype(np.int32)
    cnt = np.cumsum(onehot, axis=3)  # cnt[..., p, k] = #keys < p in bucket k
    total_keys = 0
    unmasked = 0
    for p in range(T0 + first, T0 + S):
        qb = b[:, :, :, p]
        c = cnt[:, :, :, p, :]
        adj = sum(np.take_along_axis(c, ((qb + d) % 8)[..., None], axis=3)[..., 0] for d in (-1, 0, 1))
        prev_b = b[:, :, :, p - 1]
        prev_masked = ((prev_b - qb) % 8)
        prev_masked = ~np.isin(prev_masked, (0, 1, 7))
        unmasked += int(adj.sum() + prev_masked.sum())
        total_keys += L * B * Hh * p
    return total_keys * 5 + unmasked * hd * 4, unmasked, total_keys


def prefill_unmasked_pairs(bucket_slots, T):
    """Causal pairs (q, k <= q) of a prefill of T positions that the wave
    mask lets through: key bucket within one of the query's (attn.rs:185-
    210; the query's own position included) or k = q - 1 (attn.rs:211-220).
    bucket_slots: u8 [L][B][H][>= T] from the cache.  Returns (unmasked,
    dense) summed over all layers, sequences and heads."""
    import numpy as np
    b = bucket_slots[..., :T].astype(np.int64)
    cnt = np.cumsum(b[..., None] == np.arange(8), axis=3, dtype=np.int32)  # keys <= q per bucket
    adj = sum(np.take_along_axis(cnt, ((b + d) % 8)[..., None], axis=4)[..., 0] for d in (-1, 0, 1))
    prev_masked = ~np.isin((b[..., :-1] - b[..., 1:]) % 8, (0, 1, 7))
    L, B, H = b.shape[:3]
    return int(adj.sum() + prev_masked.sum()), L * B * H * T * (T + 1) // 2


# dram__bytes_read.sum + dram__bytes_write.sum of decode_attn over its
# algorithmic bytes, measured by ncu on `bench.py --profile-case decode`
# (values kept with the capture's summary under profiles/).
DECODE_ATTN_TRAFFIC_RATIO = 1.0024  # 43.268 MB measured / 43.166 MB algorithmic


def prefill_flops_per_layer(B, T, E, H, hd, C):
    """2*B*T*E*H*(2+C) + 2*B*T*E*hd + P*2*(2+C+hd) + 2*B*T*E^2 with the dense
    causal pair count P = B*H*T(T+1)/2."""
    P = B * H * T * (T + 1) // 2
    return 2 * B * T * E * H * (2 + C) + 2 * B * T * E * hd + P * 2 * (2 + C + hd) + 2 * B * T * E * E


def attn_core_flops(B, T, H, hd, C):
    """The attention kernel's own algorithmic work: 2*P*(2+C+hd) over the
    dense causal pairs P = B*H*T(T+1)/2 (scores over the 2+C feature columns,
    PV over hd).  Projections and out_proj run in other kernels."""
    P = B * H * T * (T + 1) // 2
    return 2 * P * (2 + C + hd)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import numpy as np
    import torch
    import wave_engine_b200 as wb

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    E, H, hd, C, L = CFG["n_embd"], CFG["n_head"], CFG["head_dim"], CFG["content_dim"], CFG["n_layers"]
    B, T, S = CFG["batch"], CFG["seq_len"], args.decode_steps
    ctx = wb.Context(local)
    stream = torch.cuda.current_stream(dev)
    ctx.set_stream(stream.cuda_stream)
    layers = [wb.AttnLayer(ctx, wb.gaussian_block_attn(1000 + l, H, E, C)) for l in range(L)]
    if args.kv == "paged":
        # one pool of 128-position pages, every sequence's T + S reserved up front
        cache = wb.KvCache(L, H, hd, max_seqs=B, max_ctx=T + S, ctx=ctx, n_pages=B * (-(-(T + S) // 128)))
        for i in range(B):
            cache.reserve(i, T + S)
    else:
        cache = wb.KvCache(L, H, hd, max_seqs=B, max_ctx=T + S, ctx=ctx)
    g = torch.Generator(device=dev).manual_seed(1234 + 7919 * rank)
    x_pre = torch.randn((L, B, T, E), generator=g, device=dev)
    x_dec = torch.randn((S, L, B, E), generator=g, device=dev)
    y_pre = torch.empty((B, T, E), device=dev)
    x_stage = torch.empty((L, B, E), device=dev)   # one decode step's per-layer inputs
    y_stage = torch.empty((L, B, E), device=dev)
    ids_dev = torch.arange(B, dtype=torch.int32, device=dev)
    ids_host = np.arange(B, dtype=np.int32)

    def prefill(xp, yp, ids):
        cache.reset()
        for l in range(L):
            cache.prefill(l, layers[l], xp[l], ids, out=yp)

    def decode_layers(xs, ys, ids):
        for l in range(L):
            cache.forward_one(l, layers[l], xs[l], ids, out=ys[l])

    def check_err(where):
        code = ctx.take_device_error()
        if code:
            names = {1: "tma timeout", 2: "mma timeout", 4: "softmax timeout", 8: "bounds", 16: "decode timeout"}
            raise RuntimeError(f"device error word 0x{code:x} ({[v for k, v in names.items() if code & k]}) "
                               f"after {where}")

    # eager reference step: allocates workspaces, counts launches, gives the
    # per-kernel breakdown (profiled, untimed)
    ctx.profile("")
    prefill(x_pre, y_pre, ids_dev)
    check_err("eager prefill")
    for s in range(S):
        decode_layers(x_dec[s], y_stage, ids_dev)
    breakdown = ctx.profile_report()
    ctx.profile(None)
    check_err("eager decode")
    launches_prefill = sum(n for k, (n, _) in breakdown.items() if not k.startswith("decode"))
    launches_decode_step = sum(n for k, (n, _) in breakdown.items() if k.startswith("decode")) // S

    # one decode step (24 layers) as a CUDA graph, replayed once per token
    graph = torch.cuda.CUDAGraph()
    prefill(x_pre, y_pre, ids_dev)
    x_stage.copy_(x_dec[0])
    cap_stream = torch.cuda.Stream(dev)
    cap_stream.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cap_stream):
        decode_layers(x_stage, y_stage, ids_dev)
    stream.wait_stream(cap_stream)
    ctx.set_stream(stream.cuda_stream)
    check_err("graph capture")

    def step(ev=None):
        prefill(x_pre, y_pre, ids_dev)
        if ev is not None:
            ev.record(stream)
        for s in range(S):
            x_stage.copy_(x_dec[s])
            graph.replay()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    for w in range(args.warmup):
        step()
        barrier()
        check_err(f"warm-up step {w}")

    if not args.no_prefill_profile:
        ctx.profile("attn_tc")
    if args.check_each_step:
        for k in range(args.steps):
            step()
            barrier()
            check_err(f"diagnostic step {k} (profiler {'off' if args.no_prefill_profile else 'on'})")
    clocks = Clocks(local)
    clocks.start()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e0.record(stream)
    for k in range(args.steps):
        starts[k].record(stream)
        step(ev=mids[k])
        ends[k].record(stream)
    e1.record(stream)
    barrier()
    clk = clocks.stop()
    prof = ctx.profile_report() if not args.no_prefill_profile else {}
    ctx.profile(None)
    ms_total = e0.elapsed_time(e1)
    pre_ms = sum(starts[k].elapsed_time(mids[k]) for k in range(args.steps)) / args.steps
    dec_ms = sum(mids[k].elapsed_time(ends[k]) for k in range(args.steps)) / args.steps
    ms_step = max_over_ranks(ms_total / args.steps, world, dev)
    pre_ms = max_over_ranks(pre_ms, world, dev)
    dec_ms = max_over_ranks(dec_ms, world, dev)
    tok_step = B * T + B * S
    value = world * tok_step / (ms_step / 1e3)
    check_err("the timed region")
    # every rank's output statistics of the last timed step, gathered to rank 0
    out_stats = gather_output_stats([y_pre, y_stage], world, dev)
    y_ref = y_stage.clone()  # the last decode step's outputs of the timed steps (for the end-to-end check)

    # rooflines: decode attention (HBM, the dominant kernel) and prefill
    # attention (tensor), each from CUDA events around its own launches
    hbm, bf16, peak_kind = peaks()
    bk = np.stack([np.stack([cache.read(l, b)[1] for b in range(B)]) for l in range(L)])
    byts, unmasked, keys = decode_bytes_exact(bk, T, S, H, hd)
    unm_pairs, dense_pairs = prefill_unmasked_pairs(bk, T)
    # decode_attn launch time: events around each launch, captured into a
    # copy of the decode graph and replayed once at the middle of the decode
    # phase (step S/2, after the timed region, which stays uninstrumented)
    s_mid = S // 2
    graph_p = torch.cuda.CUDAGraph()
    ctx.profile("decode_attn")
    cap2 = torch.cuda.Stream(dev)
    cap2.wait_stream(stream)
    with torch.cuda.graph(graph_p, stream=cap2):
        decode_layers(x_stage, y_stage, ids_dev)
    stream.wait_stream(cap2)
    ctx.set_stream(stream.cuda_stream)
    prefill(x_pre, y_pre, ids_dev)
    for s in range(s_mid):
        x_stage.copy_(x_dec[s])
        graph.replay()
    x_stage.copy_(x_dec[s_mid])
    graph_p.replay()
    barrier()
    prof_dec = ctx.profile_report()
    ctx.profile(None)
    del graph_p
    check_err("instrumented decode step")
    n_att, t_att = prof_dec.get("decode_attn", (0, 0.0))
    mid_bytes, _, _ = decode_bytes_exact(bk, T, s_mid + 1, H, hd, first=s_mid)
    per_launch_bytes = mid_bytes / L + B * E * 4  # + the x rows read and the o rows written once each
    per_launch_ms = t_att / max(1, n_att)
    if per_launch_ms <= 0:
        raise RuntimeError("the instrumented decode step recorded no decode_attn time")
    ach = per_launch_bytes / (per_launch_ms / 1e3) / 1e9
    traffic = int(round(per_launch_bytes * DECODE_ATTN_TRAFFIC_RATIO))
    roof = {"kernel": "decode_attn", "bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
            "frac": round(ach / hbm, 4), "traffic": traffic, "peak_kind": peak_kind,
            "algorithmic_bytes_per_launch": int(per_launch_bytes), "launch_ms": round(per_launch_ms, 5),
            "launches_timed": n_att,
            "timing": "CUDA events around each decode_attn launch of one decode step (24 layers, context "
                      f"{T + s_mid}), replayed from an instrumented copy of the decode graph",
            "traffic_note": "dram read+write bytes per launch = algorithmic bytes x the ratio measured by ncu "
                            "on the decode profile case (32 sequences, context ~1100)",
            "unmasked_key_fraction": round(unmasked / keys, 4),
            "decode_ms_per_layer_step": round(dec_ms / (S * L), 5)}
    roof_prefill = None
    if "attn_tc" in prof:
        n, tot = prof["attn_tc"]
        fl = attn_core_flops(B, T, H, hd, 0)  # serve prefill: no content bias
        fl_layer = prefill_flops_per_layer(B, T, E, H, hd, 0)
        a_ms = tot / n
        layer_ms = pre_ms / L
        roof_prefill = {"kernel": "attn_tc", "bound": "tensor", "achieved": round(fl / (a_ms / 1e3) / 1e12, 2),
                        "peak": bf16, "peak_kind": f"{peak_kind} bf16 dense, burst", "unit": "TFLOP/s",
                        "frac": round(fl / (a_ms / 1e3) / 1e12 / bf16, 4), "launch_ms": round(a_ms, 4),
                        "flops_per_launch": fl,
                        "note": "attn_tc's own algorithmic FLOPs 2*P*(2+C+hd) over the dense causal pairs "
                                "(C = 0 in the serve prefill) / its CUDA-event time",
                        "unmasked_pair_fraction": round(unm_pairs / dense_pairs, 4),
                        "unmasked_pairs_per_layer": unm_pairs // L,
                        "dense_pairs_per_layer": dense_pairs // L,
                        "layer": {"achieved": round(fl_layer / (layer_ms / 1e3) / 1e12, 2),
                                  "frac": round(fl_layer / (layer_ms / 1e3) / 1e12 / bf16, 4),
                                  "layer_ms": round(layer_ms, 4), "flops_per_layer": fl_layer,
                                  "note": "whole-layer algorithmic FLOPs (projections, attention, out_proj) / "
                                          "whole prefill layer time"}}

    # end to end through the public API: every step copies all of its inputs
    # from pinned host memory and all of its outputs back, inside the timed
    # region, the way a serving loop feeds the library: inputs go up on one
    # copy stream into one of two device buffer sets (the next step's inputs
    # travel while the current step computes), outputs come down on another
    # a layer (prefill) or a chunk of 16 steps (decode) behind the compute.
    # The compute is the same public calls (prefill per layer, the captured
    # forward_one graph per decode step).  The first timed step's inputs are
    # copied inside the timed region with nothing to hide behind.
    e2e = None
    e2e_sync = None
    if not args.no_e2e:
        xp_h = x_pre.cpu().pin_memory()
        xd_h = x_dec.cpu().pin_memory()
        yp_h = torch.empty((L, B, T, E)).pin_memory()
        yd_h = torch.empty((S, L, B, E)).pin_memory()
        xp_d = [torch.empty_like(x_pre) for _ in range(2)]
        xd_d = [torch.empty_like(x_dec) for _ in range(2)]
        yp_d = [torch.empty((L, B, T, E), device=dev) for _ in range(2)]
        yd_d = [torch.empty((S, L, B, E), device=dev) for _ in range(2)]
        c_in, c_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        DCH = 16                                   # decode steps per copy chunk
        chunks = [(c, min(S, c + DCH)) for c in range(0, S, DCH)]
        ev_in = [[torch.cuda.Event() for _ in range(L)] for _ in range(2)]
        ev_dec = [[torch.cuda.Event() for _ in chunks] for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(L)]
        ev_done = [torch.cuda.Event() for _ in chunks]
        ev_in_free = [torch.cuda.Event() for _ in range(2)]   # compute done with input set
        ev_out_free = [torch.cuda.Event() for _ in range(2)]  # copies done with output set
        n_e2e = max(1, args.e2e_steps)

        def inputs(k):
            j = k % 2
            if k >= 2:
                c_in.wait_event(ev_in_free[j])
            with torch.cuda.stream(c_in):
                for l in range(L):
                    xp_d[j][l].copy_(xp_h[l], non_blocking=True)
                    ev_in[j][l].record(c_in)
                for i, (a, b) in enumerate(chunks):
                    xd_d[j][a:b].copy_(xd_h[a:b], non_blocking=True)
                    ev_dec[j][i].record(c_in)

        def compute(k):
            j = k % 2
            if k >= 2:
                stream.wait_event(ev_out_free[j])
            cache.reset()
            for l in range(L):
                stream.wait_event(ev_in[j][l])
                cache.prefill(l, layers[l], xp_d[j][l], ids_dev, out=yp_d[j][l])
                ev_out[l].record(stream)
                c_out.wait_event(ev_out[l])
                with torch.cuda.stream(c_out):
                    yp_h[l].copy_(yp_d[j][l], non_blocking=True)
            for i, (a, b) in enumerate(chunks):
                stream.wait_event(ev_dec[j][i])
                for s in range(a, b):
                    x_stage.copy_(xd_d[j][s])
                    graph.replay()
                    yd_d[j][s].copy_(y_stage)
                ev_done[i].record(stream)
                c_out.wait_event(ev_done[i])
                with torch.cuda.stream(c_out):
                    yd_h[a:b].copy_(yd_d[j][a:b], non_blocking=True)
            ev_in_free[j].record(stream)
            ev_out_free[j].record(c_out)

        def run_e2e(n):
            c_in.wait_stream(stream)
            c_out.wait_stream(stream)
            inputs(0)
            if n > 1:
                inputs(1)
            for k in range(n):
                compute(k)
                if k + 2 < n:
                    inputs(k + 2)
            stream.wait_stream(c_in)
            stream.wait_stream(c_out)

        run_e2e(1)
        barrier()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        run_e2e(n_e2e)
        f1.record(stream)
        barrier()
        check_err("the end-to-end steps")
        e2e_ms = max_over_ranks(f0.elapsed_time(f1) / n_e2e, world, dev)
        e2e = {"value": round(world * tok_step / (e2e_ms / 1e3), 1), "unit": "tok/s",
               "outputs_equal_device_run": bool(torch.equal(yd_h[S - 1], y_ref.cpu())),
               "h2d_bytes_per_step": int((xp_h.numel() + xd_h.numel()) * 4),
               "d2h_bytes_per_step": int((yp_h.numel() + yd_h.numel()) * 4), "ms_per_step": round(e2e_ms, 3),
               "steps": n_e2e,
               "api": "KvCache.prefill per layer and the captured KvCache.forward_one graph per decode step, on "
                      "device tensors; every input copied up from pinned host memory (the next step's during the "
                      "current step, into a second buffer set) and every output copied back a layer / 16 decode "
                      "steps behind the compute, all inside the timed region; the first step's inputs are not "
                      "hidden"}

        # the same workload through the synchronous host-pointer calls (each
        # call copies its rows in and out and returns when y is on the host)
        yp_s = torch.empty((B, T, E)).pin_memory()
        yd_s = torch.empty((L, B, E)).pin_memory()

        def step_host():
            prefill(xp_h, yp_s, ids_host)
            for s in range(S):
                decode_layers(xd_h[s], yd_s, ids_host)

        step_host()
        barrier()
        f0.record(stream)
        step_host()
        f1.record(stream)
        barrier()
        check_err("the synchronous host-pointer step")
        sync_ms = max_over_ranks(f0.elapsed_time(f1), world, dev)
        e2e_sync = {"value": round(world * tok_step / (sync_ms / 1e3), 1), "unit": "tok/s",
                    "ms_per_step": round(sync_ms, 3),
                    "api": "KvCache.prefill / forward_one per layer with pinned host x and y (one synchronous "
                           "call per layer and decode step)"}

    out = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32 io; bf16 hi/lo features, fp16 P and values, tf32 projections, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) layer inputs)",
        "config": {"workload": WORKLOAD, "n_embd": E, "n_head": H, "head_dim": hd, "layers": L, "batch_per_gpu": B,
                   "seq_len": T, "decode_steps": S, "content_dim": C,
                   "l2": "inputs larger than L2 (100 MB per prefill layer input, 3 GB in all)",
                   "decode": "one CUDA graph per decode step (24 fused kernels + length updates)",
                   "kv_cache": args.kv,
                   "parallelism": f"dp{world} (sequences sharded, no collective)"},
        "prefill": {"tok_s": round(world * B * T / (pre_ms / 1e3), 1), "ms": round(pre_ms, 3)},
        "decode": {"tok_s": round(world * B * S / (dec_ms / 1e3), 1), "ms": round(dec_ms, 3)},
        "roofline": roof,
        "e2e_sync_host_calls": e2e_sync,
        "rank_output_stats": {"fields": ["sum", "sum_abs", "max_abs", "non_finite"],
                              "tensors": "last prefill layer output + last decode step outputs", "ranks": out_stats},
        "roofline_prefill": roof_prefill,
        "kernel_ms_eager_step": {k: round(v[1], 3) for k, v in sorted(breakdown.items())},
        "gpu_launches": (launches_prefill + launches_decode_step * S) * args.steps,
        "clocks": clk,
        "e2e": e2e,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args.cpu_seconds)
    del graph
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# CPU: the reference algorithm (oracle restatement) on the host cores
# ---------------------------------------------------------------------------
def cpu_sample(seconds_budget: float):
    """Bounded sample of the workload on all host threads: rounds of one-layer
    prefills of `nt` 1024-token sequences in parallel (one per thread) for
    about half the budget, then decode steps of those sequences for about a
    third of it.  Returns rates in token-layers/s."""
    import numpy as np
    from oracle import build as obuild
    from oracle import oracle
    import wave_engine_b200 as wb
    obuild.build()
    E, H, hd, C = CFG["n_embd"], CFG["n_head"], CFG["head_dim"], CFG["content_dim"]
    T, extra = CFG["seq_len"], 64
    nt = os.cpu_count() or 1
    w = wb.gaussian_block_attn(1000, H, E, C).packed()
    rng = np.random.default_rng(5)
    xs = [rng.standard_normal((T + extra, E)).astype(np.float32) for _ in range(nt)]
    states = [None] * nt

    def pre(i):
        _, states[i] = oracle.kv_prefill(w, xs[i][:T], cap=T + extra)

    rounds = 0
    t0 = time.perf_counter()
    while True:
        th = [threading.Thread(target=pre, args=(i,)) for i in range(nt)]
        [t.start() for t in th]
        [t.join() for t in th]
        rounds += 1
        if time.perf_counter() - t0 >= 0.5 * seconds_budget or rounds >= 16:
            break
    t_pre = time.perf_counter() - t0
    counts = [0] * nt
    t_end = time.perf_counter() + 0.3 * seconds_budget

    def dec(i):
        for s in range(extra):
            oracle.kv_decode(w, xs[i][T + s], states[i])
            counts[i] += 1
            if time.perf_counter() >= t_end:
                break

    t0 = time.perf_counter()
    th = [threading.Thread(target=dec, args=(i,)) for i in range(nt)]
    [t.start() for t in th]
    [t.join() for t in th]
    t_dec = time.perf_counter() - t0
    return {"nt": nt, "pre_rate": rounds * nt * T / t_pre, "dec_rate": sum(counts) / t_dec, "t_pre": t_pre,
            "t_dec": t_dec, "n_pre": rounds * nt, "n_dec": sum(counts)}


def cpu_value(r):
    L, B, T, S = CFG["n_layers"], CFG["batch"], CFG["seq_len"], CFG["decode_steps"]
    t = B * T * L / r["pre_rate"] + B * S * L / r["dec_rate"]
    return (B * T + B * S) / t


def cpu_desc(r):
    return (f"1 layer of the 768-dim workload on {r['nt']} threads (one sequence each): kv prefill of "
            f"{r['n_pre']} x 1024-token sequences ({r['t_pre']:.1f} s), then {r['n_dec']} single-position decode "
            f"calls at ctx 1024-1088 ({r['t_dec']:.1f} s); extrapolated linearly to batch 32 x 24 layers and "
            f"256 decode steps (decode at ctx ~1050 instead of 1024-1280)")


def cpu_baseline(seconds):
    r = cpu_sample(seconds)
    return {"value": round(cpu_value(r), 3), "unit": "tok/s", "cores": r["nt"], "kind": "port",
            "sample": cpu_desc(r)}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    vals = []
    for _ in range(args.warmup):
        cpu_sample(args.cpu_seconds / 4)
    last = None
    for _ in range(args.steps):
        last = cpu_sample(args.cpu_seconds / 4)
        vals.append(cpu_value(last))
    v = sorted(vals)[len(vals) // 2]
    out = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tok/s", "n_gpus": world,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": WORKLOAD, "host_cpu": True},
           "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": last["nt"], "kind": "port",
                            "sample": cpu_desc(last)},
           "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# prefill-only configurations: n_embd, heads, content dim, layers, batch, T
PREFILL_CFGS = {
    "prefill-168": dict(E=168, H=4, C=16, L=4, B=4, T=256,
                        desc="168-dim research model (4 heads x 42, 4 layers): batch 4, 256-token prefill"),
    "prefill-384": dict(E=384, H=8, C=16, L=6, B=16, T=512,
                        desc="384-dim grammar model (8 heads x 48, 6 layers): batch 16, 512-token prefill"),
    "prefill-4096": dict(E=4096, H=32, C=16, L=8, B=8, T=4096,
                         desc="4096-dim wide model (32 heads x 128, 8 layers): batch 8, 4096-token prefill"),
}


DOT_CFG = {"E": 768, "H": 12, "L": 4, "B": 32, "T": 1024,
           "desc": "legacy dot-product attention (ComputeBackend::attention, compute.rs:357-414) at the 768-dim "
                   "shape: batch 32 x 1024 tokens, 12 heads x 64, 4 layers; TF32 tensor-core projections, "
                   "tcgen05 bf16 attention core (fp32 fallback for tiles past the fixed-shift bound)"}


def run_dot_workload(args):
    """The legacy dot-product attention through wb_dot_attn_forward: seeded
    N(0, 0.02) weights, N(0, 1) per-layer inputs resident in HBM.  Prints its
    own JSON line: tok/s and the tcgen05 attention core's share of the
    measured bf16 peak (2 * 2 * head_dim FLOP per causal pair)."""
    import torch
    import wave_engine_b200 as wb
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    c = DOT_CFG
    E, H, L, B, T = c["E"], c["H"], c["L"], c["B"], c["T"]
    hd = E // H
    ctx = wb.Context(local)
    stream = torch.cuda.current_stream(dev)
    ctx.set_stream(stream.cuda_stream)
    layers = [wb.DotAttnLayer(ctx, wb.gaussian_attention_weights(5000 + l, H, E)) for l in range(L)]
    g = torch.Generator(device=dev).manual_seed(91 + rank)
    x = torch.randn((L, B, T, E), generator=g, device=dev)
    y = torch.empty((B, T, E), device=dev)

    def step():
        for l in range(L):
            y.copy_(wb.attention(layers[l], x[l], ctx=ctx))

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        step()
    barrier()
    ctx.profile("")
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    clk = clocks.stop()
    prof = ctx.profile_report()
    ctx.profile(None)
    err = ctx.take_device_error()
    if err:
        raise RuntimeError(f"device error word {err:#x} in the timed region")
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, dev)
    pairs = B * H * T * (T + 1) // 2
    core_fl = pairs * 2 * 2 * hd                                  # q.k and p.v per causal pair
    layer_fl = 2 * B * T * E * 3 * E + core_fl + 2 * B * T * E * E  # c_attn + core + c_proj
    n_att, t_att = prof.get("attn_tc", (0, 0.0))
    a_ms = t_att / max(1, n_att)
    _, bf16_peak, peak_src = peaks()
    out = {"metric": "dot-product attention tok/s (dot-768)", "value": round(world * B * T / (ms / 1e3), 1),
           "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
           "dtype": "fp32 io; TF32 tensor-core projections, bf16 tcgen05 attention core, fp32 accumulate",
           "data": "synthetic",
           "config": {"workload": c["desc"], "inputs": "per-layer inputs resident in HBM"},
           "roofline": {"kernel": "attn_tc (dot features)", "bound": "tensor", "peak": round(bf16_peak, 1),
                        "unit": "TFLOP/s", "peak_kind": f"{peak_src} dense bf16 (burst)",
                        "achieved": round(core_fl / (a_ms / 1e3) / 1e12, 2) if a_ms else None,
                        "frac": round(core_fl / (a_ms / 1e3) / 1e12 / bf16_peak, 4) if a_ms else None,
                        "launch_ms": round(a_ms, 4), "flops_per_launch": core_fl},
           "kernel_ms_per_layer": {k: round(v[1] / max(1, args.steps * L), 4) for k, v in sorted(prof.items())},
           "layer_ms": round(ms / L, 4), "layer_flops": layer_fl, "clocks": clk}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


SERVE_MODEL_CFG = {"E": 768, "H": 12, "L": 24, "B": 32, "T": 1024, "S": 32, "M": 16, "rk4": 16, "V": 50257,
                   "desc": "the whole 768-dim serve layer on the GPU (kv_cache.rs prefill / forward_one): embedding, "
                           "per layer LayerNorm -> wave attention (KV cache) and LayerNorm -> dual-maestro Kerr-ODE "
                           "FFN (maestro 16, RK4-16, AGC), residual; final LayerNorm and phase_native_decode over a "
                           "50257-token table; batch 32 x 1024-token prefill, then 32 decode steps"}


def run_serve_model_workload(args):
    """The serve loop of kv_cache.rs through ServeSession: seeded synthetic
    weights (N(0, 0.02) linear weights, the reference's ODE constants), a
    random token batch.  Prints its own JSON line: tok/s of prefill + decode,
    and the per-kernel time of one prefill and one decode step."""
    import numpy as np
    import torch
    import wave_engine_b200 as wb
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    c = SERVE_MODEL_CFG
    E, H, L, B, T, S, M, V = c["E"], c["H"], c["L"], c["B"], c["T"], c["S"], c["M"], c["V"]
    ctx = wb.Context(local)
    stream = torch.cuda.current_stream(dev)
    ctx.set_stream(stream.cuda_stream)
    g = np.random.default_rng(5 + rank)
    blocks = [wb.ServeBlock(np.ones(E, np.float32), np.zeros(E, np.float32), np.ones(E, np.float32),
                            np.zeros(E, np.float32), wb.gaussian_block_attn(1000 + l, H, E, 0),
                            wb.gaussian_ffn(2000 + l, E, M, rk4_steps=c["rk4"])) for l in range(L)]
    model = wb.ServeModel((g.standard_normal((V, E)) / np.sqrt(E)).astype(np.float32), None, blocks,
                          np.ones(E, np.float32), np.zeros(E, np.float32),
                          output_corrector=np.zeros(E // 2, np.float32))
    sess = wb.ServeSession(model, max_seqs=B, max_ctx=T + S * (args.warmup + args.steps + 2), ctx=ctx)
    tokens = g.integers(0, V, (B, T)).astype(np.int32)
    steps_tok = g.integers(0, V, (S, B)).astype(np.int32)
    ids = np.arange(B, dtype=np.int32)

    def run():
        sess.cache.reset()
        sess.prefill(tokens, ids)
        e_mid.record(stream)
        for s in range(S):
            sess.forward_one_graph(steps_tok[s], np.full(B, T + s, np.int32))

    # the decode step (24 layers: attention, FFN, residual, decoder) captured
    # once in a CUDA graph after a prefill has sized the workspaces
    sess.cache.reset()
    sess.prefill(tokens, ids)
    sess.capture_decode(ids)

    e_mid = torch.cuda.Event(enable_timing=True)
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pre_ms = 0.0
    e0.record(stream)
    for _ in range(args.steps):
        s0 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        run()
        torch.cuda.synchronize()
        pre_ms += s0.elapsed_time(e_mid)
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    pre_ms /= args.steps
    ctx.profile("")
    run()
    prof = ctx.profile_report()
    # one eager decode step, profiled (the graph replays record no per-kernel events)
    sess.forward_one(steps_tok[0], np.full(B, T + S, np.int32), ids)
    prof_dec = ctx.profile_report()
    ctx.profile(None)
    if ctx.take_device_error():
        raise RuntimeError("device error in the serve-model run")
    out = {"metric": "serve-model tok/s (prefill + decode, whole serve layer on the GPU)",
           "value": round(B * (T + S) / (ms / 1e3), 1), "unit": "tok/s", "n_gpus": 1, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "fp32 io; bf16/tf32 tensor-core attention and GEMMs, fp32 FFN",
           "data": "synthetic (seeded weights, random tokens)", "config": {"workload": c["desc"]},
           "prefill": {"tok_s": round(B * T / (pre_ms / 1e3), 1), "ms": round(pre_ms, 3)},
           "decode": {"tok_s": round(B * S / ((ms - pre_ms) / 1e3), 1), "ms": round(ms - pre_ms, 3)},
           "kernel_ms_prefill": {k: round(v[1], 3) for k, v in sorted(prof.items())},
           "kernel_us_eager_decode_step": {k: round(1e3 * v[1], 1) for k, v in sorted(prof_dec.items())},
           "agc": sess.agc.state(), "clocks": clk,
           "note": "prefill eager (host seq-id validation per layer call); each decode step one CUDA graph replay"}
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_prefill_workload(args):
    """Prefill through all attention layers of one of the prefill-only
    configurations (tensor path, content projection on): seeded N(0, 0.02)
    weights, seeded N(0, 1) per-layer inputs resident in HBM.  Prints its own
    JSON line: prefill tok/s, the attention kernel's share of the dense
    tensor peak (its own algorithmic FLOPs / its time) and the whole layer's
    (whole-layer algorithmic FLOPs / whole layer time)."""
    import torch
    import wave_engine_b200 as wb
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    c = PREFILL_CFGS[args.workload]
    E, H, C, L, B, T = c["E"], c["H"], c["C"], c["L"], c["B"], c["T"]
    hd = E // H
    by_heads = args.shard == "heads" and world > 1
    if by_heads and H % world:
        raise SystemExit(f"--shard heads needs the {H} heads to divide over {world} ranks")
    h0, h1 = (rank * H // world, (rank + 1) * H // world) if by_heads else (0, H)
    ctx = wb.Context(local)
    stream = torch.cuda.current_stream(dev)
    ctx.set_stream(stream.cuda_stream)
    layers = [wb.AttnLayer(ctx, wb.gaussian_block_attn(3000 + l, H, E, C)) for l in range(L)]
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    if by_heads:
        g = torch.Generator(device=dev).manual_seed(77)  # every rank holds the same inputs
    x = torch.randn((L, B, T, E), generator=g, device=dev)

    def step():
        for l in range(L):
            if by_heads:
                # this rank's heads and their share of out_proj, then one
                # all-reduce (sum) of the layer output over NCCL
                y = wb.wave_attention_forward_heads(layers[l], x[l], E // 2, h0, h1, add_bias=(rank == 0), ctx=ctx)
                torch.distributed.all_reduce(y)
            else:
                wb.wave_attention_forward(layers[l], x[l], E // 2, ctx=ctx)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        step()
    barrier()
    err = ctx.take_device_error()
    if err:
        raise RuntimeError(f"device error word {err:#x} during warm-up")
    ctx.profile("attn_tc")
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    clk = clocks.stop()
    prof = ctx.profile_report()
    ctx.profile(None)
    err = ctx.take_device_error()
    if err:
        raise RuntimeError(f"device error word {err:#x} in the timed region")
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world, dev)
    hbm, bf16, peak_kind = peaks()
    fl = prefill_flops_per_layer(B, T, E, H, hd, C)
    fl_attn = attn_core_flops(B, T, H, hd, C)
    if by_heads:
        fl //= world  # this rank's share of the layer
        fl_attn //= world
    n_att, t_att = prof.get("attn_tc", (0, 0.0))
    a_ms = t_att / max(1, n_att)
    layer_ms = ms / L
    tokens = B * T if by_heads else world * B * T
    out = {"metric": f"attn prefill tok/s ({args.workload})", "value": round(tokens / (ms / 1e3), 1),
           "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(ms, 3), "higher_is_better": True,
           "scaling": ("strong (heads split across ranks: each rank computes its heads and their share of "
                       "out_proj; one NCCL all-reduce of the layer output)") if by_heads else "weak",
           "vs_baseline": None,
           "dtype": "bf16 split (hi/lo) features, fp16 P and values, fp32 accumulation", "data": "synthetic",
           "config": {"workload": c["desc"], "inputs": "per-layer inputs resident in HBM"},
           "roofline": {"kernel": "attn_tc", "bound": "tensor", "peak": bf16, "unit": "TFLOP/s",
                        "peak_kind": f"{peak_kind} bf16 dense, burst",
                        "achieved": round(fl_attn / (a_ms / 1e3) / 1e12, 2) if a_ms else None,
                        "frac": round(fl_attn / (a_ms / 1e3) / 1e12 / bf16, 4) if a_ms else None,
                        "launch_ms": round(a_ms, 4), "flops_per_launch": fl_attn,
                        "note": "attn_tc's own algorithmic FLOPs 2*P*(2+C+hd) over the dense causal pairs / "
                                "its CUDA-event time"},
           "layer_roofline": {"achieved": round(fl / (layer_ms / 1e3) / 1e12, 2),
                              "frac": round(fl / (layer_ms / 1e3) / 1e12 / bf16, 4), "layer_ms": round(layer_ms, 4),
                              "note": "whole-layer algorithmic FLOPs / whole layer time"},
           "clocks": clk}
    if rank == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


def run_decode_stress(args):
    """Decode stress: 256 concurrent sequences, contexts uniform in
    [128, 4096], 12 heads x 64, fp32 KV cache of Gaussian values and uniform
    phases, one new token per sequence per step through 24 layers.  Under
    torchrun the sequences are split across ranks by cached keys.  One step
    (24 layers) is a CUDA graph; inputs are per-step N(0,1) rows.  Prints its
    own JSON line (metric: decode tok/s and HBM roofline)."""
    import numpy as np
    import torch
    import wave_engine_b200 as wb
    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    E, H, hd, L = CFG["n_embd"], CFG["n_head"], CFG["head_dim"], CFG["n_layers"]
    n_all, K, W = 256, args.steps, args.warmup
    rng = np.random.default_rng(4)
    lens_all = rng.integers(128, 4097, size=n_all).tolist()
    mine = shard_sequences(lens_all, world)[rank]
    lens = [lens_all[i] for i in mine]
    B = len(mine)
    cap = max(lens) + K + W + 1
    ctx = wb.Context(local)
    stream = torch.cuda.current_stream(dev)
    ctx.set_stream(stream.cuda_stream)
    layers = [wb.AttnLayer(ctx, wb.gaussian_block_attn(2000 + l, H, E, 0)) for l in range(L)]
    cache = wb.KvCache(L, H, hd, max_seqs=B, max_ctx=cap, ctx=ctx)
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    vpool = torch.randn((H, 4096, hd), generator=g, device=dev)
    for l in range(L):
        for b, n in enumerate(lens):
            ph = torch.atan2(torch.randn((H, n), generator=g, device=dev), torch.randn((H, n), generator=g, device=dev))
            cache.load(l, b, ph.contiguous(), vpool[:, :n].contiguous())
    x = torch.randn((K + W, L, B, E), generator=g, device=dev)
    ids = torch.arange(B, dtype=torch.int32, device=dev)
    stage = torch.empty((L, B, E), device=dev)
    y = torch.empty((L, B, E), device=dev)

    def step_layers():
        for l in range(L):
            cache.forward_one(l, layers[l], stage[l], ids, out=y[l])

    stage.copy_(x[0])
    step_layers()  # eager: allocates the decode scratch
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cs = torch.cuda.Stream(dev)
    cs.wait_stream(stream)
    with torch.cuda.graph(graph, stream=cs):
        step_layers()
    stream.wait_stream(cs)
    ctx.set_stream(stream.cuda_stream)
    for s in range(1, W):
        stage.copy_(x[s])
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    clocks = Clocks(local)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(W, W + K):
        stage.copy_(x[s])
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = max_over_ranks(e0.elapsed_time(e1) / K, world, dev)
    code = ctx.take_device_error()
    # exact algorithmic bytes of the timed steps from the cache's buckets
    bks = []
    for l in range(L):
        for b in range(B):
            bk = np.empty((H, cache.n_cached(l, b)), np.uint8)
            from wave_engine_b200 import _lib
            _lib.call("wb_kv_cache_read", ctx.handle, cache.handle, l, b, None, bk.ctypes.data, None)
            bks.append((bk, lens[b] + W))
    unm = 0
    keys = 0
    for bk, n0 in bks:
        b64 = bk.astype(np.int64)
        for p in range(n0, n0 + K):
            qb = b64[:, p]
            prev = b64[:, p - 1]
            kb = b64[:, :p]
            adj = (((kb - qb[:, None]) % 8)[:, :, None] == np.array([0, 1, 7])).any(-1)
            pm = ~np.isin((prev - qb) % 8, (0, 1, 7))
            unm += int(adj.sum() + pm.sum())
            keys += H * p
    byts = keys * 5 + unm * hd * 4 + K * L * B * E * 8
    hbm, _, peak_kind = peaks()
    ach = byts / K / (ms / 1e3) / 1e9
    out = {"metric": "decode tok/s (decode stress, 768-dim, 256 seqs, ctx U[128,4096], fp32 KV)",
           "value": round(n_all / (ms / 1e3), 1), "unit": "tok/s",
           "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": round(ms, 3), "higher_is_better": True,
           "scaling": "strong (256 sequences split by cached keys)", "seqs_this_rank": B,
           "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm, "unit": "GB/s",
                        "frac": round(ach / hbm, 4), "peak_kind": peak_kind,
                        "algorithmic_bytes_per_step": int(byts / K), "unmasked_key_fraction": round(unm / keys, 4),
                        "timing": "whole decode step (24 layers: attention + out_proj kernels) on this rank"},
           "clocks": clk, "device_error": code}
    del graph
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(out), flush=True)


def run_profile_case(args):
    """Small single-GPU cases for ncu captures (no timing, a few hundred MB
    on the device): 'decode' = 12 fused decode steps of one 768-dim layer,
    32 sequences at ctx ~1100; 'prefill' = 3 tensor-path prefills of one
    768-dim layer, 4 x 1024 tokens (content on); 'prefill-serve' = 3 serve
    prefills (KV cache, no content) of one 768-dim layer, 16 x 1024 tokens
    (about 10 work items per SM, as in the benchmark's 20); 'dot' = 3
    dot-product attention forwards of one 768-dim layer, 16 x 1024 tokens;
    'dot-4096' = the same for one 4096-dim layer (32 heads x 128), 2 x 4096
    tokens; 'serve-ffn' = 3 serve-layer FFN calls on 16 x 1024 rows."""
    import numpy as np
    import torch
    import wave_engine_b200 as wb
    ctx = wb.Context(0)
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    H, E, hd, C = CFG["n_head"], CFG["n_embd"], CFG["head_dim"], CFG["content_dim"]
    extra = {}
    w = wb.gaussian_block_attn(5, H, E, C)
    lay = wb.AttnLayer(ctx, w)
    g = torch.Generator(device="cuda").manual_seed(0)
    if args.profile_case == "decode-stress":
        # one layer of the decode-stress workload (~3.3 GB on the device)
        rng = np.random.default_rng(4)
        lens = rng.integers(128, 4097, size=256).tolist()
        B = 256
        cache = wb.KvCache(1, H, hd, max_seqs=B, max_ctx=max(lens) + 16, ctx=ctx)
        vpool = torch.randn((H, 4096, hd), generator=g, device="cuda")
        for b, n in enumerate(lens):
            ph = torch.atan2(torch.randn((H, n), generator=g, device="cuda"), torch.randn((H, n), generator=g, device="cuda"))
            cache.load(0, b, ph.contiguous(), vpool[:, :n].contiguous())
        lay0 = wb.AttnLayer(ctx, wb.gaussian_block_attn(5, H, E, 0))
        ids = torch.arange(B, dtype=torch.int32, device="cuda")
        x = torch.randn((6, B, E), generator=g, device="cuda")
        y = torch.empty((B, E), device="cuda")
        for s in range(6):
            cache.forward_one(0, lay0, x[s], ids, out=y)
        torch.cuda.synchronize()
        per_step = [B * E * 4] * 6
        for b, n in enumerate(lens):
            bk = cache.read(0, b)[1][None, None]  # [1][1][H][n + 6]
            for s in range(6):
                per_step[s] += int(decode_bytes_exact(bk, n, s + 1, H, hd, first=s)[0])
        extra["decode_attn_algorithmic_bytes"] = per_step
    elif args.profile_case == "decode":
        B, n = 32, 1100
        cache = wb.KvCache(1, H, hd, max_seqs=B, max_ctx=n + 16, ctx=ctx)
        rng = np.random.default_rng(0)
        for b in range(B):
            ph = np.arctan2(rng.standard_normal((H, n)), rng.standard_normal((H, n))).astype(np.float32)
            cache.load(0, b, ph, rng.standard_normal((H, n, hd)).astype(np.float32))
        ids = torch.arange(B, dtype=torch.int32, device="cuda")
        x = torch.randn((12, B, E), generator=g, device="cuda")
        y = torch.empty((B, E), device="cuda")
        for s in range(12):
            cache.forward_one(0, lay, x[s], ids, out=y)
        torch.cuda.synchronize()
        bk = np.stack([np.stack([cache.read(0, b)[1] for b in range(B)])])
        extra["decode_attn_algorithmic_bytes"] = [
            int(decode_bytes_exact(bk, n, s + 1, H, hd, first=s)[0] + B * E * 4) for s in range(12)]
    elif args.profile_case == "prefill-serve":
        B = 16
        cache = wb.KvCache(1, H, hd, max_seqs=B, max_ctx=CFG["seq_len"], ctx=ctx)
        ids = torch.arange(B, dtype=torch.int32, device="cuda")
        x = torch.randn((B, CFG["seq_len"], E), generator=g, device="cuda")
        y = torch.empty_like(x)
        for _ in range(3):
            cache.reset()
            cache.prefill(0, lay, x, ids, out=y)
    elif args.profile_case == "dot":
        # 3 dot-product attention forwards of one 768-dim layer, 16 x 1024 tokens
        dl = wb.DotAttnLayer(ctx, wb.gaussian_attention_weights(5000, H, E))
        x = torch.randn((16, CFG["seq_len"], E), generator=g, device="cuda")
        for _ in range(3):
            wb.attention(dl, x, ctx=ctx)
        extra["attn_core_flops_per_launch"] = 16 * H * CFG["seq_len"] * (CFG["seq_len"] + 1) // 2 * 4 * hd
    elif args.profile_case == "dot-4096":
        # 3 dot-product attention forwards of one 4096-dim layer (head_dim 128), 2 x 4096 tokens
        H4, E4, T4 = 32, 4096, 4096
        dl = wb.DotAttnLayer(ctx, wb.gaussian_attention_weights(5000, H4, E4))
        x = torch.randn((2, T4, E4), generator=g, device="cuda")
        for _ in range(3):
            wb.attention(dl, x, ctx=ctx)
        extra["attn_core_flops_per_launch"] = 2 * H4 * T4 * (T4 + 1) // 2 * 4 * (E4 // H4)
    elif args.profile_case == "serve-ffn":
        # 3 FFN calls (maestro 16, RK4-16) on 16 requests x 1024 rows of the 768-dim model
        ffn = wb.FfnLayer(ctx, wb.gaussian_ffn(2000, E, 16))
        agc = wb.Agc(ctx)
        x = torch.randn((16 * CFG["seq_len"], E), generator=g, device="cuda")
        for _ in range(3):
            wb.ffn_forward(ffn, agc, x, rows_per_call=CFG["seq_len"], ctx=ctx)
    else:
        x = torch.randn((4, CFG["seq_len"], E), generator=g, device="cuda")
        for _ in range(3):
            wb.wave_attention_forward(lay, x, E // 2, ctx=ctx)
    torch.cuda.synchronize()
    err = ctx.take_device_error()
    print(json.dumps({"profile_case": args.profile_case, "device_error": err, **extra}))
    if err:
        sys.exit(1)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--workload", choices=["serve-768", "decode-stress", "dot-768", "serve-model"] + sorted(PREFILL_CFGS),
                    default="serve-768",
                    help="serve-768: the headline configuration (default); decode-stress: 256 sequences of "
                         "context 128-4096; prefill-168/-384/-4096: prefill through all layers of the 168-, "
                         "384- and 4096-dim models; dot-768: the legacy dot-product attention at the 768-dim "
                         "shape; serve-model: the whole serve layer (attention + FFN + decoder) on the GPU")
    ap.add_argument("--profile-case", choices=["decode", "decode-stress", "prefill", "prefill-serve", "dot", "dot-4096", "serve-ffn"],
                    default=None,
                    help="run a small case for an ncu capture instead of the benchmark")
    ap.add_argument("--shard", choices=["batch", "heads"], default="batch",
                    help="prefill workloads under torchrun: every rank its own batch (weak scaling), or the heads "
                         "of one batch split across ranks with an all-reduce of each layer output")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--decode-steps", type=int, default=CFG["decode_steps"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-prefill-profile", action="store_true")
    ap.add_argument("--check-each-step", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=8,
                    help="consecutive steps of the pipelined end-to-end run (every step's copies are timed; only the "
                         "first step's uploads have no compute to hide behind)")
    ap.add_argument("--kv", choices=["contiguous", "paged"], default="contiguous",
                    help="serve-768's KV cache: fixed slots (default) or a pool of 128-position pages")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=20.0)
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.profile_case:
        run_profile_case(args)
    elif args.workload == "decode-stress" and args.impl == "ours":
        run_decode_stress(args)
    elif args.workload in PREFILL_CFGS and args.impl == "ours":
        run_prefill_workload(args)
    elif args.workload == "dot-768" and args.impl == "ours":
        run_dot_workload(args)
    elif args.workload == "serve-model" and args.impl == "ours":
        run_serve_model_workload(args)
    elif args.impl == "reference" and args.workload != "serve-768":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": f"the CPU reference arm times the serve-768 "
                                                                  f"workload only, not {args.workload}"}))
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
