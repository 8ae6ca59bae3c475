"""Independent numpy restatement of saccade-core's CPU path, for cross-checking the C oracle.

Written separately from oracle/ctarq_oracle.c (different f16 conversion, rounding
and looping code) so that agreement between the two is evidence about both.
Vectorised across rows/tokens; every reduction keeps the reference's sequential
f32 order.  Small sizes only.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def round_half_away(x: np.ndarray) -> np.ndarray:
    """Rust f32::round on f32 values (exact in f64)."""
    x64 = np.asarray(x, dtype=np.float64)
    return np.trunc(x64 + np.copysign(0.5, x64))


def sat_i32(x: np.ndarray) -> np.ndarray:
    x64 = np.asarray(x, dtype=np.float64)
    out = np.where(np.isnan(x64), 0.0, np.clip(np.trunc(x64), -2147483648.0, 2147483647.0))
    return out.astype(np.int64)


def f16_bits(x32: np.ndarray) -> np.ndarray:
    return np.asarray(x32, dtype=np.float32).astype(np.float16).view(np.uint16)


def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def row_scales(w: np.ndarray) -> np.ndarray:
    """compress.rs:41-51: running strict max of |w| per row, then /7 (or 1.0 for all-zero rows)."""
    max_abs = np.zeros(w.shape[0], dtype=F32)
    for c in range(w.shape[1]):
        a = np.abs(w[:, c])
        max_abs = np.where(a > max_abs, a, max_abs)
    return np.where(max_abs > F32(0), (max_abs / F32(7)).astype(F32), F32(1)).astype(F32)


def quantize(w: np.ndarray):
    s = row_scales(w)
    q = sat_i32(round_half_away((w / s[:, None]).astype(F32)))
    q = np.clip(q, -8, 7)
    deq = (q.astype(F32) * s[:, None]).astype(F32)
    err = (w - deq).astype(F32)
    return s, q, err


def percentile_threshold(w: np.ndarray, fill: float) -> float:
    """compress.rs:137-176."""
    _, _, err = quantize(np.asarray(w, dtype=F32))
    e = np.abs(err).ravel()
    e = e[e > F32(1e-10)]
    if e.size == 0:
        return 0.001
    e = np.sort(e)
    prod = F32(F32(1.0) - F32(fill)) * F32(e.size)
    idx = int(np.trunc(np.float64(prod))) if prod > 0 else 0
    return float(e[min(idx, e.size - 1)])


def compress(w: np.ndarray, thr: float):
    """compress.rs:6-129 -> dict with the reference's key names."""
    w = np.asarray(w, dtype=F32)
    n, k = w.shape
    s, q, err = quantize(w)
    u = (q + 8).astype(np.uint32).reshape(n, k // 8, 8)
    packed = np.zeros((n, k // 8), dtype=np.uint32)
    for i in range(8):
        packed |= u[:, :, i] << np.uint32(4 * i)
    keep = np.abs(err) > F32(thr)
    kept = np.where(keep, err, F32(0))
    max_err = F32(np.max(np.abs(kept))) if kept.size else F32(0)
    ds = F32(max_err / F32(127)) if max_err > 0 else F32(1)
    nz = kept != 0
    rows, cols = np.nonzero(nz)
    qe = np.clip(sat_i32(round_half_away((kept[rows, cols] / ds).astype(F32))), -128, 127)
    row_ptrs = np.zeros(n + 1, dtype=np.uint32)
    row_ptrs[1:] = np.cumsum(np.bincount(rows, minlength=n)).astype(np.uint32)
    return {
        "packed_base": packed,
        "scale_base": f16_bits(s),
        "delta_row_ptrs": row_ptrs,
        "delta_col_indices": cols.astype(np.uint32),
        "delta_values": qe.astype(np.int8).view(np.uint8),
        "delta_scale": int(f16_bits(np.array([ds]))[0]),
    }


def variance_rows(x32: np.ndarray) -> np.ndarray:
    """heuristics.rs:3-14 / calibration.rs:36-45 vectorised over tokens (sequential over K)."""
    m, k = x32.shape
    s = np.zeros(m, dtype=F32)
    sq = np.zeros(m, dtype=F32)
    for i in range(k):
        v = x32[:, i]
        s = (s + v).astype(F32)
        sq = (sq + (v * v).astype(F32)).astype(F32)
    mean = (s / F32(k)).astype(F32)
    return ((sq / F32(k)).astype(F32) - (mean * mean).astype(F32)).astype(F32)


def calibrate(acts: np.ndarray, p4: float, p8: float):
    v = np.sort(variance_rows(np.asarray(acts, dtype=F32)), kind="stable")
    n = v.size

    def idx(p):
        r = round_half_away(F32(F32(n) * F32(p)))
        return min(int(max(r, 0)), n - 1)

    return float(v[idx(p4)]), float(v[idx(p8)])


def forward(c: dict, n: int, k: int, t4: float, t8: float, x_bits: np.ndarray, force_route=None):
    """op.rs:10-185 (non-bypass) -> (y f16 bits [m, n], routed [m], acc f32 [m, n])."""
    x32 = f16_to_f32(x_bits).reshape(-1, k)
    m = x32.shape[0]
    score = variance_rows(x32)
    routed = ((score >= F32(t4)) & (score < F32(t8))) | (score >= F32(t8))
    if force_route is not None:
        routed = np.asarray(force_route).astype(bool)
    packed = c["packed_base"]
    nib = np.stack([((packed >> np.uint32(4 * i)) & np.uint32(0xF)).astype(np.int64) - 8 for i in range(8)], -1)
    nib = nib.reshape(n, k).astype(F32)
    scale = f16_to_f32(c["scale_base"])
    ds = f16_to_f32(np.array([c["delta_scale"]], dtype=np.uint16))[0]
    rp, ci = c["delta_row_ptrs"], c["delta_col_indices"]
    dv = (c["delta_values"].view(np.int8).astype(F32) * ds).astype(F32)
    # CSC order = column-major over (col, row): stable sort of CSR entries by column
    rows_of = np.repeat(np.arange(n), np.diff(rp.astype(np.int64)))
    order = np.argsort(ci, kind="stable")
    acc_all = np.empty((m, n), dtype=F32)
    for t in range(m):
        x = x32[t]
        a = [np.zeros(n, dtype=F32) for _ in range(4)]
        for p in range(k // 8):
            for j in range(8):
                a[j % 4] = (a[j % 4] + (x[8 * p + j] * nib[:, 8 * p + j]).astype(F32)).astype(F32)
        acc = ((((a[0] + a[1]).astype(F32) + a[2]).astype(F32) + a[3]).astype(F32) * scale).astype(F32)
        if routed[t] and ci.size:
            for e in order:
                r = rows_of[e]
                acc[r] = F32(acc[r] + F32(x[ci[e]] * dv[e]))
        acc_all[t] = acc
    return f16_bits(acc_all), routed.astype(np.uint8), acc_all
