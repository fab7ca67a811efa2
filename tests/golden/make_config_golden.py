"""Generate ``tests/golden/configs.npz``: the oracle's outputs for the
reduced benchmark configurations of ``config_cases.py`` (prefill outputs and
phases; decode outputs after a prefill), with the sha256 of every output
array.  Run from the repository root:
    python tests/golden/make_config_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import oracle  # noqa: E402
from tests.golden import config_cases as cc  # noqa: E402

OUT = Path(__file__).resolve().parent / "configs.npz"


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def build() -> dict:
    out = {}
    for name, E, H, C, B, T, init, seed in cc.PREFILL:
        w = cc.weights(init, seed, H, E, C)
        x = cc.inputs(seed, B, T, E)
        ys, phs = [], []
        for b in range(B):
            y, _, ph = oracle.attn_forward(w, x[b])
            ys.append(y)
            phs.append(ph)
        out[name + "/y"] = np.stack(ys)
        out[name + "/phases"] = np.stack(phs)
    for name, E, H, lens, steps, seed in cc.DECODE:
        w = dict(cc.weights("gauss", seed, H, E, 0))
        x = cc.inputs(seed, len(lens), max(lens) + steps, E)
        ys = np.zeros((steps, len(lens), E), np.float32)
        for b, n in enumerate(lens):
            _, st = oracle.kv_prefill(w, x[b, :n], cap=n + steps)
            for s in range(steps):
                ys[s, b] = oracle.kv_decode(w, x[b, n + s], st)
        out[name + "/y"] = ys
    for k in list(out):
        out[k + ".sha256"] = np.array(sha(out[k]))
    return out


if __name__ == "__main__":
    data = build()
    np.savez_compressed(OUT, **data)
    print(OUT, OUT.stat().st_size, "bytes;", ", ".join(k for k in data if not k.endswith(".sha256")))
