"""The C-TARQ format producer on the GPU, with the reference's names.

    compress_tensor_to_saccade     compress.rs:6-129
    compute_percentile_threshold   compress.rs:137-176
    ProfileRunner.calibrate        calibration.rs:10-47

The outputs are bit-identical to the reference's (same IEEE f32 steps on the device);
keys follow compress.rs:113-127, delta_* absent when no coordinate is kept.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import LIB, check


def _stream(dev):
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _as_f32_cuda(t: torch.Tensor, device=None) -> torch.Tensor:
    if t.dim() != 2:
        raise ValueError("Only 2D tensors are supported")
    if device is None:
        device = t.device if t.is_cuda else torch.device("cuda", torch.cuda.current_device())
    return t.to(device=device, dtype=torch.float32).contiguous()


def compute_percentile_threshold(base_tensor: torch.Tensor, target_fill_pct: float) -> float:
    """Error magnitude at the (1 - fill) quantile of the nonzero 4-bit reconstruction errors."""
    w = _as_f32_cuda(base_tensor)
    n, k = w.shape
    out = ctypes.c_float()
    check(LIB.sc_percentile_threshold(w.data_ptr(), n, k, float(target_fill_pct), ctypes.byref(out),
                                      _stream(w.device)))
    return float(out.value)


def compress_tensor_to_saccade(base_tensor: torch.Tensor, delta_threshold: float) -> dict:
    """4-bit row-scaled pack plus the i8 CSR of errors above the threshold."""
    w = _as_f32_cuda(base_tensor)
    n, k = w.shape
    if k % 8:
        raise ValueError("in_features must be a multiple of 8")
    dev = w.device
    packed = torch.empty((n, k // 8), dtype=torch.int32, device=dev)
    scale = torch.empty(n, dtype=torch.float16, device=dev)
    row_ptrs = torch.empty(n + 1, dtype=torch.int32, device=dev)
    nnz = ctypes.c_int64()
    ds = ctypes.c_uint16()
    s = _stream(dev)
    check(LIB.sc_compress(w.data_ptr(), n, k, float(delta_threshold), packed.data_ptr(), scale.data_ptr(),
                          row_ptrs.data_ptr(), None, None, 0, ctypes.byref(nnz), ctypes.byref(ds), s))
    out = {"packed_base": packed.view(torch.uint32), "scale_base": scale}
    z = int(nnz.value)
    if z > 0:
        cols = torch.empty(z, dtype=torch.int32, device=dev)
        vals = torch.empty(z, dtype=torch.uint8, device=dev)
        check(LIB.sc_compress(w.data_ptr(), n, k, float(delta_threshold), packed.data_ptr(), scale.data_ptr(),
                              row_ptrs.data_ptr(), cols.data_ptr(), vals.data_ptr(), z, ctypes.byref(nnz),
                              ctypes.byref(ds), s))
        out["delta_row_ptrs"] = row_ptrs.view(torch.uint32)
        out["delta_col_indices"] = cols.view(torch.uint32)
        out["delta_values"] = vals
        out["delta_scale"] = torch.tensor([ds.value], dtype=torch.int16).view(torch.float16).to(dev)
    return out


class ProfileRunner:
    """calibration.rs:6-47."""

    @staticmethod
    def calibrate(activations: torch.Tensor, pct_t4: float, pct_t8: float) -> tuple:
        """Per-token variance of a 2-D activation tensor, then the order statistics at
        round(n * pct) (clamped to n - 1) as (t4, t8)."""
        if activations.dim() != 2:
            raise ValueError("Calibration expects 2D activation tensors (batch, hidden_dim)")
        a = activations
        if not a.is_cuda:
            a = a.to(torch.device("cuda", torch.cuda.current_device()))
        if a.dtype not in (torch.float32, torch.float16):
            a = a.to(torch.float32)
        a = a.contiguous()
        n, k = a.shape
        t4, t8 = ctypes.c_float(), ctypes.c_float()
        check(LIB.sc_calibrate(a.data_ptr(), _lib.SC_F32 if a.dtype == torch.float32 else _lib.SC_F16, n, k,
                               float(pct_t4), float(pct_t8), ctypes.byref(t4), ctypes.byref(t8), _stream(a.device)))
        return float(t4.value), float(t8.value)


def saccade_op_from_compressed(blocks: dict, config, out_features: int, in_features: int, **kw):
    """SaccadeLinearOp::new from a compress_tensor_to_saccade() result (keys of compress.rs:113-127)."""
    from .op import SaccadeLinearOp, SparseDeltaMatrix

    sp = None
    if "delta_row_ptrs" in blocks:
        sp = SparseDeltaMatrix(blocks["delta_row_ptrs"], blocks["delta_col_indices"], blocks["delta_values"],
                               blocks["delta_scale"])
    return SaccadeLinearOp(blocks["packed_base"], blocks["scale_base"], sp, config, out_features, in_features, **kw)
