"""Seeded C-TARQ test cases shared by the CPU and GPU tests.

A case is a weight matrix W ~ N(0, 0.02) packed by the oracle (compress.rs:6-129 with
the threshold of compress.rs:137-176), activations X ~ N(0, 1) with a chosen set of
tokens scaled x8 (the router's "hard" tokens), and thresholds calibrated on the
f16-rounded activations like saccade-compile does (compile.rs:152-153).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import oracle as O

# Fast-path tolerance of the north-star contract: max |error| <= 1e-3 * RMS(reference)
# on the f32 accumulators; f16 outputs additionally allow one f16 ulp of the reference
# value, because two f32 sums that differ in their last bits can round to adjacent f16s.
TOL_REL_RMS = 1e-3


@dataclass
class Case:
    w: np.ndarray
    c: O.Compressed
    x_bits: np.ndarray      # f16 bits [m, k]
    t4: float
    t8: float
    n: int
    k: int
    m: int

    def oracle(self) -> O.OracleLinear:
        return O.OracleLinear(self.c, self.t4, self.t8)


def make_case(n: int, k: int, m: int, fill: float = 0.01, seed: int = 0, boost=None, pct=(0.75, 0.95),
              thresholds=None) -> Case:
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    thr = O.percentile_threshold(w, fill) if fill is not None else 1e30
    c = O.compress(w, thr)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if boost is None:
        boost = rng.choice(m, size=max(1, m // 4), replace=False) if m > 0 else []
    for t in boost:
        x[t] *= 8.0
    xb = x.astype(np.float16).view(np.uint16)
    if thresholds is not None:
        t4, t8 = thresholds
    elif m > 0:
        t4, t8 = O.calibrate(xb.view(np.float16).astype(np.float32), *pct)
    else:
        t4, t8 = 0.0, 0.0
    return Case(w, c, xb, float(t4), float(t8), n, k, m)


def f16_ulp(y_bits: np.ndarray) -> np.ndarray:
    y = np.abs(y_bits.view(np.float16).astype(np.float32)).astype(np.float16)
    return np.spacing(y).astype(np.float32)


def assert_fast_close(y_gpu_bits: np.ndarray, y_ref_bits: np.ndarray, what: str = "") -> None:
    """f16 outputs: |y - y_ref| <= 1e-3 * RMS(y_ref) + 1 ulp_f16(y_ref) elementwise."""
    yg = y_gpu_bits.view(np.float16).astype(np.float32)
    yr = y_ref_bits.view(np.float16).astype(np.float32)
    rms = float(np.sqrt(np.mean(yr.astype(np.float64) ** 2))) if yr.size else 0.0
    tol = TOL_REL_RMS * rms + f16_ulp(y_ref_bits)
    err = np.abs(yg - yr)
    bad = err > tol
    assert not bad.any(), f"{what}: {bad.sum()} of {bad.size} outside tolerance; max err {err.max():.3e}, rms {rms:.3e}"


def assert_acc_close(acc_gpu: np.ndarray, acc_ref: np.ndarray, what: str = "") -> None:
    """f32 accumulators: max |acc - acc_ref| <= 1e-3 * RMS(acc_ref)."""
    rms = float(np.sqrt(np.mean(acc_ref.astype(np.float64) ** 2))) if acc_ref.size else 0.0
    err = float(np.max(np.abs(acc_gpu - acc_ref))) if acc_ref.size else 0.0
    assert err <= TOL_REL_RMS * rms, f"{what}: max err {err:.3e} > {TOL_REL_RMS} * rms {rms:.3e}"


def sample_rows(c: O.Compressed, rows: np.ndarray) -> O.Compressed:
    """The layer restricted to output rows `rows` (ascending): its packed words, row scales and
    CSR rows.  The dW scale is the whole matrix's, so each sampled row computes exactly what it
    computes in the full layer (routing depends on the tokens only)."""
    rows = np.asarray(rows, dtype=np.int64)
    rp = c.delta_row_ptrs.astype(np.int64)
    cols, vals, ptrs = [], [], [0]
    for r in rows:
        lo, hi = rp[r], rp[r + 1]
        cols.append(c.delta_col_indices[lo:hi])
        vals.append(c.delta_values[lo:hi])
        ptrs.append(ptrs[-1] + int(hi - lo))
    ci = np.concatenate(cols).astype(np.uint32) if cols else np.zeros(0, np.uint32)
    cv = np.concatenate(vals).astype(np.uint8) if vals else np.zeros(0, np.uint8)
    return O.Compressed(np.ascontiguousarray(c.packed_base[rows]), np.ascontiguousarray(c.scale_base[rows]),
                        np.asarray(ptrs, dtype=np.uint32), ci, cv, c.delta_scale, int(rows.size), c.in_features)
