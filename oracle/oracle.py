"""numpy front end to the C oracle (TEST INFRASTRUCTURE, parity unpinned).

The C library restates saccade-core's CPU path (compress.rs, config.rs,
heuristics.rs, calibration.rs, op.rs).  Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg may import this module; the shipped library
never does.

Parity status: UNPINNED -- the Rust reference cannot be built here and ships no
golden vectors.  tests/test_oracle.py checks this restatement against an
independent numpy restatement and hand-worked known answers.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_LIB_NATIVE = None

_u32p = ctypes.POINTER(ctypes.c_uint32)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)


def build(native: bool = False) -> str:
    """Compile the oracle with its Makefile (portable, or -march=native)."""
    target = "native" if native else "all"
    subprocess.run(["make", "-s", "-C", HERE, target], check=True)
    return os.path.join(HERE, "liboracle_ctarq_native.so" if native else "liboracle_ctarq.so")


def _declare(lib):
    lib.oracle_f32_to_f16.restype = ctypes.c_uint16
    lib.oracle_f32_to_f16.argtypes = [ctypes.c_float]
    lib.oracle_f16_to_f32.restype = ctypes.c_float
    lib.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
    lib.oracle_f32_to_f16_array.argtypes = [_f32p, _u16p, ctypes.c_int64]
    lib.oracle_bf16_to_f16_array.argtypes = [_u16p, _u16p, ctypes.c_int64]
    lib.oracle_variance_heuristic.restype = ctypes.c_float
    lib.oracle_variance_heuristic.argtypes = [_u16p, ctypes.c_int64]
    lib.oracle_percentile_threshold.restype = ctypes.c_float
    lib.oracle_percentile_threshold.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float]
    lib.oracle_compress.restype = ctypes.c_int
    lib.oracle_compress.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float,
                                    _u32p, _u16p, _u32p, _u32p, _u8p, _i64p, _u16p]
    lib.oracle_calibrate.restype = ctypes.c_int
    lib.oracle_calibrate.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_float,
                                     _f32p, _f32p]
    lib.oracle_build_csc.restype = ctypes.c_int
    lib.oracle_build_csc.argtypes = [_u32p, _u32p, _u8p, ctypes.c_int64, ctypes.c_uint16, ctypes.c_int64,
                                     ctypes.c_int64, _u32p, _u32p, _f32p]
    lib.oracle_dequant_dense.argtypes = [_u32p, _u16p, ctypes.c_int64, ctypes.c_int64, _u32p, _u32p, _f32p, _f32p]
    lib.oracle_route_bits.restype = ctypes.c_int
    lib.oracle_route_bits.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float]
    lib.oracle_forward.argtypes = [_u32p, _u16p, ctypes.c_int64, ctypes.c_int64, _u32p, _u32p, _f32p,
                                   ctypes.c_float, ctypes.c_float, _u16p, ctypes.c_int64,
                                   _u16p, _u8p, _f32p, _u8p, ctypes.c_int, _f32p, ctypes.c_int]
    return lib


def lib(native: bool = False):
    """Load (building if needed) the oracle shared library."""
    global _LIB, _LIB_NATIVE
    if native:
        if _LIB_NATIVE is None:
            _LIB_NATIVE = _declare(ctypes.CDLL(build(native=True)))
        return _LIB_NATIVE
    if _LIB is None:
        path = os.path.join(HERE, "liboracle_ctarq.so")
        if not os.path.exists(path):
            build()
        _LIB = _declare(ctypes.CDLL(path))
    return _LIB


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t) if a is not None else None


# ---------------------------------------------------------------- f16 helpers

def f32_to_f16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16_array(_p(a, _f32p), _p(out, _u16p), a.size)
    return out


def bf16_bits_to_f16_bits(a: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().oracle_bf16_to_f16_array(_p(a, _u16p), _p(out, _u16p), a.size)
    return out


# ---------------------------------------------------------------- format producer

@dataclass
class Compressed:
    """compress.rs:113-127 key set: packed_base, scale_base and the optional delta_* CSR."""
    packed_base: np.ndarray        # u32 [N, K/8]
    scale_base: np.ndarray         # u16 (f16 bits) [N]
    delta_row_ptrs: np.ndarray     # u32 [N+1]
    delta_col_indices: np.ndarray  # u32 [nnz]
    delta_values: np.ndarray       # u8 (i8 bits) [nnz]
    delta_scale: int               # f16 bits
    out_features: int
    in_features: int

    @property
    def nnz(self) -> int:
        return int(self.delta_values.size)


def percentile_threshold(w: np.ndarray, target_fill_pct: float) -> float:
    """compress.rs:137-176 compute_percentile_threshold."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    return float(lib().oracle_percentile_threshold(_p(w, _f32p), n, k, target_fill_pct))


def compress(w: np.ndarray, delta_threshold: float) -> Compressed:
    """compress.rs:6-129 compress_tensor_to_saccade."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    if k % 8:
        raise ValueError("in_features must be a multiple of 8")
    packed = np.empty((n, k // 8), dtype=np.uint32)
    scale = np.empty(n, dtype=np.uint16)
    row_ptrs = np.empty(n + 1, dtype=np.uint32)
    cols = np.empty(max(n * k, 1), dtype=np.uint32)
    vals = np.empty(max(n * k, 1), dtype=np.uint8)
    nnz = ctypes.c_int64(0)
    ds = ctypes.c_uint16(0)
    rc = lib().oracle_compress(_p(w, _f32p), n, k, delta_threshold, _p(packed, _u32p), _p(scale, _u16p),
                               _p(row_ptrs, _u32p), _p(cols, _u32p), _p(vals, _u8p), ctypes.byref(nnz),
                               ctypes.byref(ds))
    if rc != 0:
        raise ValueError("oracle_compress failed")
    z = nnz.value
    return Compressed(packed, scale, row_ptrs, cols[:z].copy(), vals[:z].copy(), int(ds.value), n, k)


def calibrate(acts: np.ndarray, pct_t4: float, pct_t8: float) -> tuple[float, float]:
    """calibration.rs:10-47 ProfileRunner::calibrate (acts already f32)."""
    acts = np.ascontiguousarray(acts, dtype=np.float32)
    n, k = acts.shape
    t4 = ctypes.c_float()
    t8 = ctypes.c_float()
    if lib().oracle_calibrate(_p(acts, _f32p), n, k, pct_t4, pct_t8, ctypes.byref(t4), ctypes.byref(t8)) != 0:
        raise ValueError("calibrate needs at least one token")
    return float(t4.value), float(t8.value)


def variance(x_f16_bits: np.ndarray) -> float:
    """heuristics.rs:3-14 variance_heuristic of one f16 token."""
    x = np.ascontiguousarray(x_f16_bits, dtype=np.uint16)
    return float(lib().oracle_variance_heuristic(_p(x, _u16p), x.size))


def route_bits(score: float, t4: float, t8: float) -> int:
    return int(lib().oracle_route_bits(score, t4, t8))


# ---------------------------------------------------------------- the op

class OracleLinear:
    """SaccadeLinearOp::new (config.rs:76-150) + cpu_fwd (op.rs:10-185)."""

    def __init__(self, c: Compressed, t4: float, t8: float):
        self.c = c
        self.t4 = float(t4)
        self.t8 = float(t8)
        n, k = c.out_features, c.in_features
        self.out_features, self.in_features = n, k
        if c.nnz > 0:
            self.col_ptrs = np.empty(k + 1, dtype=np.uint32)
            self.csc_rows = np.empty(c.nnz, dtype=np.uint32)
            self.csc_vals = np.empty(c.nnz, dtype=np.float32)
            rc = lib().oracle_build_csc(_p(c.delta_row_ptrs, _u32p), _p(c.delta_col_indices, _u32p),
                                        _p(c.delta_values, _u8p), c.nnz, c.delta_scale, n, k,
                                        _p(self.col_ptrs, _u32p), _p(self.csc_rows, _u32p),
                                        _p(self.csc_vals, _f32p))
            if rc != 0:
                raise ValueError("column index out of range")
        else:
            self.col_ptrs = self.csc_rows = self.csc_vals = None
        self._dense = None

    def dense_weight(self) -> np.ndarray:
        """config.rs:112-142 dense base + dW weight used by the bypass path."""
        if self._dense is None:
            n, k = self.out_features, self.in_features
            w = np.empty((n, k), dtype=np.float32)
            lib().oracle_dequant_dense(_p(self.c.packed_base, _u32p), _p(self.c.scale_base, _u16p), n, k,
                                       _p(self.col_ptrs, _u32p), _p(self.csc_rows, _u32p),
                                       _p(self.csc_vals, _f32p), _p(w, _f32p))
            self._dense = w
        return self._dense

    def forward(self, x_f16_bits: np.ndarray, *, bypass: bool = False, force_route=None,
                n_threads: int = 0, native: bool = False, t4=None, t8=None):
        """op.rs:10-185.  x: u16 f16 bits [..., K].  Returns (y f16 bits [..., N], routed u8 [M], acc f32)."""
        x = np.ascontiguousarray(x_f16_bits, dtype=np.uint16)
        k, n = self.in_features, self.out_features
        lead = x.shape[:-1]
        if x.shape[-1] != k:
            raise ValueError("last dimension must equal in_features")
        m = int(np.prod(lead)) if lead else 1
        y = np.empty(lead + (n,), dtype=np.uint16)
        routed = np.zeros(m, dtype=np.uint8)
        acc = np.empty(lead + (n,), dtype=np.float32)
        fr = None
        if force_route is not None:
            fr = np.ascontiguousarray(force_route, dtype=np.uint8)
        dense = self.dense_weight() if bypass else None
        L = lib(native)
        L.oracle_forward(_p(self.c.packed_base, _u32p), _p(self.c.scale_base, _u16p), n, k,
                         _p(self.col_ptrs, _u32p), _p(self.csc_rows, _u32p), _p(self.csc_vals, _f32p),
                         self.t4 if t4 is None else t4, self.t8 if t8 is None else t8,
                         _p(x, _u16p), m, _p(y, _u16p), _p(routed, _u8p), _p(acc, _f32p), _p(fr, _u8p),
                         1 if bypass else 0, _p(dense, _f32p), n_threads)
        return y, routed, acc
