"""The exchange step of a row-sharded C-TARQ layer on the CPU (TEST INFRASTRUCTURE, parity unpinned).

A tensor-parallel rank that holds input columns [c0, c1) of a layer sees only that slice of every
token, while the router (heuristics.rs:3-14, op.rs:64-73) decides on the whole token.  The
exchange restated here -- the scheme the GPU library implements in sc_forward_split /
sc_finalize_split -- needs one all-reduce per layer:

    1. each rank: y_base  = (slice of x . (q - 8)) * s   for every token   (op.rs:80-150 on the slice)
                  y_delta = the slice's dW . x             for every token   (op.rs:152-170 on the slice)
                  stats   = sum x, sum x^2, sum |x| over the slice (f64, rounded to f32)
       laid out as one f32 vector [y_base m*n | y_delta m*n | stats m*3];
    2. one all-reduce (sum) of that vector over the ranks;
    3. per token: the routing decision on the summed sums -- f64 score, decided where both
       thresholds lie outside the error bound of the reference's sequential f32 variance (widened
       by the f32 rounding of the partial sums and of their sum) -- then
       y = f16(y_base + [routed] y_delta).

The base product comes from the C oracle (oracle.OracleLinear with no token routed); dW and the
sums are plain numpy.  Only tests/ may import this module.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

U = 2.0 ** -24


def slice_columns(c: O.Compressed, k0: int, k1: int) -> O.Compressed:
    """The reference-format layer restricted to input columns [k0, k1) (multiples of 8): what a
    ROWS shard keeps."""
    n = c.out_features
    packed = np.ascontiguousarray(c.packed_base[:, k0 // 8:k1 // 8])
    rp = c.delta_row_ptrs.astype(np.int64)
    cols = c.delta_col_indices.astype(np.int64)
    keep = (cols >= k0) & (cols < k1)
    counts = np.array([np.count_nonzero(keep[rp[r]:rp[r + 1]]) for r in range(n)], dtype=np.int64)
    new_rp = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint32)
    return O.Compressed(packed, c.scale_base, new_rp, (cols[keep] - k0).astype(np.uint32),
                        np.ascontiguousarray(c.delta_values[keep]), c.delta_scale, n, k1 - k0)


def _delta_scale(c: O.Compressed) -> float:
    return float(np.array([c.delta_scale], dtype=np.uint16).view(np.float16)[0])


def split_exchange(c_slice: O.Compressed, x_slice_bits: np.ndarray) -> np.ndarray:
    """Step 1 on one rank: the f32 exchange vector of the slice (x_slice_bits u16 f16 [m, K_slice])."""
    x = np.ascontiguousarray(x_slice_bits, dtype=np.uint16)
    m, k = x.shape
    n = c_slice.out_features
    no_route = np.zeros(m, dtype=np.uint8)
    _, _, base = O.OracleLinear(c_slice, 0.0, 0.0).forward(x, force_route=no_route)
    xf = x.view(np.float16).astype(np.float64)
    dw = np.zeros((n, k), dtype=np.float64)
    rp = c_slice.delta_row_ptrs.astype(np.int64)
    ds = np.float32(_delta_scale(c_slice))
    vals = c_slice.delta_values.view(np.int8).astype(np.float32) * ds  # f32 product, as the op forms it
    for r in range(n):
        e0, e1 = rp[r], rp[r + 1]
        dw[r, c_slice.delta_col_indices[e0:e1].astype(np.int64)] = vals[e0:e1]
    delta = (xf @ dw.T).astype(np.float32)
    stats = np.stack([xf.sum(axis=1), (xf * xf).sum(axis=1), np.abs(xf).sum(axis=1)], axis=1).astype(np.float32)
    return np.concatenate([base.reshape(-1).astype(np.float32), delta.reshape(-1), stats.reshape(-1)])


def route_band(S1: float, S2: float, SA: float, k: int, t4: float, t8: float, e1x: float, e2x: float):
    """(decision, score): decision 1 routed / 0 not routed when both thresholds lie outside the
    bound of the reference's sequential f32 variance around the f64 score, -1 otherwise.  The
    bound: |fl(sum) - sum| <= gamma_{k-1} sum|terms| (gamma_n = n u / (1 - n u)) carried through
    the mean, its square and the subtraction, doubled; e1x, e2x bound errors already in S1, S2."""
    nu = (k - 1) * U
    gam = nu / (1.0 - nu)
    inv = 1.0 / k
    e1 = gam * (SA + e1x) + e1x
    e2 = gam * (S2 + e2x) + e2x
    mean, a = S1 * inv, S2 * inv
    err_mean = (e1 + U * (abs(S1) + e1)) * inv
    err_a = (e2 + U * (S2 + e2)) * inv
    am = abs(mean) + err_mean
    err_sq = err_mean * (2.0 * abs(mean) + err_mean) + U * am * am
    var = a - mean * mean
    b = 2.0 * (err_a + err_sq + U * (abs(var) + err_a + err_sq)) + 1e-37
    if np.isfinite(var) and np.isfinite(b) and abs(var - t4) > b and abs(var - t8) > b:
        return (1 if ((t4 <= var < t8) or var >= t8) else 0), var
    return -1, var


def split_finalize(exchange: np.ndarray, m: int, n: int, k_full: int, ranks: int, t4: float, t8: float,
                   bypass: bool = False):
    """Step 3 on the summed vector: (y f16 bits [m, n], routed u8 [m], undecided count)."""
    base = exchange[:m * n].reshape(m, n).astype(np.float32)
    delta = exchange[m * n:2 * m * n].reshape(m, n).astype(np.float32)
    stats = exchange[2 * m * n:2 * m * n + 3 * m].reshape(m, 3).astype(np.float64)
    w = 2.0 * (ranks + 1) * U
    routed = np.zeros(m, dtype=np.uint8)
    undecided = 0
    for t in range(m):
        if bypass:
            routed[t] = 1
            continue
        S1, S2, SA = stats[t]
        d, var = route_band(S1, S2, SA, k_full, t4, t8, w * SA, w * S2)
        if d < 0:
            undecided += 1
            d = 1 if ((t4 <= var < t8) or var >= t8) else 0
        routed[t] = d
    acc = np.where(routed[:, None] == 1, (base + delta).astype(np.float32), base)
    return O.f32_to_f16_bits(acc.astype(np.float32)), routed, undecided
