"""Parity helpers: the J10 tolerance model of the reference
(src/monitors/junctions/tier_parity.rs:23-35: an element passes when
|a - b| <= tol_abs + tol_rel * max(|a|, |b|)) and bucket-flip handling."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

TIGHT = (1e-5, 1e-5)    # tier_parity.rs:23
LINEAR = (1e-4, 1e-4)   # tier_parity.rs:24
EXACT_TOL = (1e-5, 0.0)  # fp32 SIMT path: max-abs 1e-5
TENSOR_TOL = (2e-3, 0.0)  # bf16 tensor-core path: max-abs 2e-3

TAU32 = np.float32(6.2831855)
BUCKET_W = TAU32 / np.float32(8)


@dataclass
class ParityDiff:
    section: str
    n_elements: int
    n_violations: int
    max_abs: float
    max_rel: float
    mean_abs: float
    worst: list

    @property
    def passed(self) -> bool:
        return self.n_violations == 0

    def __str__(self):
        return (f"{self.section}: n={self.n_elements} viol={self.n_violations} max_abs={self.max_abs:.3e} "
                f"max_rel={self.max_rel:.3e} mean_abs={self.mean_abs:.3e} worst={self.worst[:3]}")


def check(section, a, b, tol) -> ParityDiff:
    """tier_parity.rs:62-104 check_outputs_1d over flattened arrays."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if a.shape != b.shape:
        return ParityDiff(section, max(a.size, b.size), max(a.size, b.size), np.inf, np.inf, np.inf, [])
    tol_abs, tol_rel = tol
    with np.errstate(invalid="ignore"):
        d = np.abs(a - b)
    both_inf = np.isinf(a) & np.isinf(b) & (np.sign(a) == np.sign(b))
    d = np.where(both_inf, 0.0, d)
    scale = np.maximum(np.abs(np.where(both_inf, 0, a)), np.abs(np.where(both_inf, 0, b)))
    with np.errstate(invalid="ignore"):
        rel = np.where(scale < 1e-12, 0.0, d / np.where(scale < 1e-12, 1, scale))
    viol = ~(d <= tol_abs + tol_rel * scale)
    idx = np.argsort(-np.where(np.isnan(d), np.inf, d))[:10]
    worst = [(int(i), float(a[i]), float(b[i]), float(d[i])) for i in idx if viol[i]]
    return ParityDiff(section, a.size, int(viol.sum()), float(np.nanmax(d)) if d.size else 0.0,
                      float(np.nanmax(rel)) if d.size else 0.0, float(np.nanmean(d)) if d.size else 0.0, worst)


def phase_diff(a, b):
    """Angular difference folded into [-pi, pi] (atan2 may land on either side of +-pi)."""
    d = np.asarray(a, np.float64) - np.asarray(b, np.float64)
    return np.abs((d + np.pi) % (2 * np.pi) - np.pi)


def boundary_distance(theta):
    """Distance of each phase to the nearest bucket boundary (radians)."""
    t = np.mod(np.mod(np.asarray(theta, np.float64), 2 * np.pi) + 2 * np.pi, 2 * np.pi)
    w = 2 * np.pi / 8
    r = np.mod(t, w)
    return np.minimum(r, w - r)


def buckets_of(theta):
    """Bucket of each phase, float32 arithmetic as kv_cache.rs:66-70."""
    t = np.asarray(theta, np.float32)
    n = np.fmod(np.fmod(t, TAU32) + TAU32, TAU32).astype(np.float32)
    q = (n / BUCKET_W).astype(np.float32)
    return np.minimum(np.where(np.isnan(q) | (q <= 0), 0, q).astype(np.int64), 7)
