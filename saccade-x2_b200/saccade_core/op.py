"""SaccadeLinearOp: the C-TARQ linear on a B200, mirroring saccade-core's operator.

    SaccadeConfig        config.rs:19-24
    SparseDeltaMatrix    config.rs:28-33
    SaccadeLinearOp      config.rs:60-150 (construction), op.rs:5-185 (name, forward)
    set_bypass_c_tarq / is_c_tarq_bypassed   config.rs:4-12

Construction copies the reference-format buffers to the device layout through
sc_layer_create; forward() runs sc_forward_ws on the current CUDA stream with a
per-(device, stream) workspace that is zero-filled once and reused.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional

import torch

from . import _lib
from ._lib import LIB, check

_DT = {torch.float16: _lib.SC_F16, torch.bfloat16: _lib.SC_BF16, torch.float32: _lib.SC_F32}


def set_bypass_c_tarq(val: bool) -> None:
    """config.rs:6-8: global switch to the dense base+dW product for every token."""
    LIB.sc_set_bypass_c_tarq(1 if val else 0)


def is_c_tarq_bypassed() -> bool:
    """config.rs:10-12."""
    return bool(LIB.sc_is_c_tarq_bypassed())


@dataclass
class SaccadeConfig:
    """config.rs:19-24.  `block_size` is carried for surface compatibility (unused by the
    reference too); the heuristic is the variance heuristic (heuristics.rs:3-14)."""
    t4: float
    t8: float
    block_size: int = 16
    heuristic: str = "variance"


@dataclass
class SparseDeltaMatrix:
    """config.rs:28-33: CSR dW (u32 row_ptrs [N+1], u32 col_indices [nnz], u8 values
    holding i8 bits [nnz], f16 scale [1])."""
    row_ptrs: torch.Tensor
    col_indices: torch.Tensor
    values: torch.Tensor
    scale: torch.Tensor


_MODES = {"fast": _lib.SC_MODE_FAST, "exact": _lib.SC_MODE_EXACT, "fast_tc": _lib.SC_MODE_FAST_TC,
          "fast_tc8": _lib.SC_MODE_FAST_TC8}


def _mode_code(mode: str) -> int:
    if mode not in _MODES:
        raise ValueError(f"mode must be one of {sorted(_MODES)}, got {mode!r}")
    return _MODES[mode]


def _f16_bits(t: torch.Tensor) -> int:
    return int(t.reshape(-1)[:1].to(torch.float16).view(torch.int16).item()) & 0xFFFF


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


class _Workspaces:
    """Zero-filled workspaces keyed by (device, stream); grown on demand.  A replaced workspace is
    kept alive: a CUDA graph captured with it still writes there when replayed."""

    def __init__(self):
        self._ws = {}
        self._retired = []

    def get(self, device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> torch.Tensor:
        key = (device.index, stream.cuda_stream)
        ws = self._ws.get(key)
        if ws is None or ws.numel() < nbytes:
            if ws is not None:
                self._retired.append(ws)
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws


WORKSPACES = _Workspaces()

# Handles whose release (cudaFree inside the library) would fall into a CUDA graph capture: freeing
# device memory while a stream captures invalidates the capture, and the garbage collector may run
# a destructor at any point of the captured Python code.  They are released after the capture.
_DEFERRED = []


def release_handle(destroy, h) -> None:
    try:
        capturing = torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()
    except Exception:  # noqa: BLE001 - interpreter shutdown
        capturing = False
    if capturing:
        _DEFERRED.append((destroy, h))
    else:
        destroy(h)
        flush_deferred()


def flush_deferred() -> None:
    """Releases the handles deferred during a capture (call outside of any capture)."""
    while _DEFERRED:
        destroy, h = _DEFERRED.pop()
        destroy(h)


def _u32(t: torch.Tensor) -> torch.Tensor:
    """Reinterpret a u32/i32/i64 index tensor as contiguous 32-bit words."""
    if t.dtype in (torch.int64, torch.long):
        t = t.to(torch.int32)
    if t.dtype == torch.uint32:
        t = t.view(torch.int32)
    return t.contiguous()


class SaccadeLinearOp:
    """One C-TARQ linear layer resident on a B200.

    packed_base u32 [N, K/8] (8 nibbles of q+8 per word along K, compress.rs:54-83),
    scale_base f16 [N], optional SparseDeltaMatrix, SaccadeConfig thresholds.
    mode "fast" (tensor cores, default), "fast_tc" (the same contract; decode dequantises the
    weights into tensor memory for tcgen05 MMAs), "fast_tc8" (as fast_tc, one-token decode on fp8
    tcgen05 MMAs with an exact e4m3 split of x) or "exact" (op.rs's f32 order, bit-identical).
    shard=("columns"|"rows", index, count) keeps a tensor-parallel slice; ("columns_range"|"rows_range",
    begin, end) keeps exactly output rows / input columns [begin, end).
    """

    NAME = "fused_c_tarq_saccade_linear"

    def __init__(self, packed_base: torch.Tensor, scale_base: torch.Tensor,
                 sparse_delta_q8: Optional[SparseDeltaMatrix], config: SaccadeConfig,
                 out_features: int, in_features: int, *, device=None, mode: str = "fast",
                 shard: Optional[tuple] = None):
        if device is None:
            device = packed_base.device if packed_base.is_cuda else torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("SaccadeLinearOp runs on a CUDA device only")
        dev_index = device.index if device.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", dev_index)
        self.config = config
        self.full_out_features = int(out_features)
        self.full_in_features = int(in_features)
        on_dev = packed_base.is_cuda
        keep = []  # keep temporaries alive across the create call

        def prep(t, dtype=None):
            if t is None:
                return None
            t = t.contiguous()
            if on_dev and t.device != self.device:  # host tensors, or another GPU's: the layer's device
                t = t.to(self.device)
            if not on_dev and t.is_cuda:
                t = t.cpu()
            keep.append(t)
            return t

        pb = prep(_u32(packed_base))
        sb = prep(scale_base.to(torch.float16) if scale_base.dtype != torch.float16 else scale_base)
        d = _lib.ScLayerDesc()
        d.out_features = int(out_features)
        d.in_features = int(in_features)
        if pb.numel() != out_features * (in_features // 8) or in_features % 8:
            raise ValueError("packed_base must be [out_features, in_features/8] with in_features % 8 == 0")
        d.packed_base = pb.data_ptr()
        d.scale_base = sb.data_ptr()
        if sparse_delta_q8 is not None and sparse_delta_q8.values.numel() > 0:
            rp = prep(_u32(sparse_delta_q8.row_ptrs))
            ci = prep(_u32(sparse_delta_q8.col_indices))
            vals = sparse_delta_q8.values
            if vals.dtype == torch.int8:
                vals = vals.view(torch.uint8)
            cv = prep(vals.to(torch.uint8) if vals.dtype != torch.uint8 else vals)
            d.delta_row_ptrs = rp.data_ptr()
            d.delta_col_indices = ci.data_ptr()
            d.delta_values = cv.data_ptr()
            d.delta_nnz = cv.numel()
            d.delta_scale = _f16_bits(sparse_delta_q8.scale)
        d.t4 = float(config.t4)
        d.t8 = float(config.t8)
        d.device = dev_index
        d.buffers_on_device = 1 if on_dev else 0
        d.mode = _mode_code(mode)
        if shard is not None:
            kind, a, b = shard
            base_kind = kind[:-6] if kind.endswith("_range") else kind
            d.shard_kind = {"columns": _lib.SC_SHARD_COLUMNS, "rows": _lib.SC_SHARD_ROWS}[base_kind]
            if kind.endswith("_range"):
                d.shard_begin, d.shard_end = int(a), int(b)
            else:
                d.shard_index, d.shard_count = int(a), int(b)
        if on_dev:
            torch.cuda.synchronize(self.device)
        h = ctypes.c_void_p()
        check(LIB.sc_layer_create(ctypes.byref(d), ctypes.byref(h)))
        self._h = h
        info = _lib.ScLayerInfo()
        check(LIB.sc_layer_get_info(self._h, ctypes.byref(info)))
        self.info = info
        self.out_features = int(info.out_features)
        self.in_features = int(info.in_features)
        self.shard_kind = (shard[0][:-6] if shard[0].endswith("_range") else shard[0]) if shard else None
        self.col_begin = int(info.col_begin)
        self.row_begin = int(info.row_begin)
        self.undecided = torch.zeros(1, dtype=torch.int32, device=self.device)  # split routing, see finalize_split
        self.mode = mode

    # ------------------------------------------------------------------ surface of op.rs
    def name(self) -> str:
        return LIB.sc_op_name().decode()

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            release_handle(LIB.sc_layer_destroy, h)
            self._h = None

    @property
    def delta_nnz(self) -> int:
        return int(self.info.delta_nnz)

    def set_thresholds(self, t4: float, t8: float) -> None:
        check(LIB.sc_layer_set_thresholds(self._h, float(t4), float(t8)))
        self.config.t4, self.config.t8 = float(t4), float(t8)
        LIB.sc_layer_get_info(self._h, ctypes.byref(self.info))

    def set_mode(self, mode: str) -> None:
        check(LIB.sc_layer_set_mode(self._h, _mode_code(mode)))
        self.mode = mode

    def check_device(self) -> None:
        """Raise if a kernel recorded a device-side error (bounded wait ran out, bad index)."""
        check(LIB.sc_layer_check(self._h, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))

    def workspace_size(self, m: int) -> int:
        return int(LIB.sc_workspace_size(self._h, int(m)))

    def _prep_x(self, x: torch.Tensor, k: int):
        if not x.is_cuda or x.device != self.device:
            raise ValueError(f"input must be on {self.device}")
        if x.dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("input dtype must be float16 or bfloat16 (op.rs:19 reads f16)")
        if x.shape[-1] != k:
            raise ValueError(f"last dimension {x.shape[-1]} != in_features {k}")
        if not x.is_contiguous():
            raise ValueError("input must be contiguous (op.rs:19-24 ignores strides)")
        m = x.numel() // k if k else 0
        return m

    def forward(self, x: torch.Tensor, *, out_dtype: torch.dtype = torch.float16,
                bias: Optional[torch.Tensor] = None, return_routing: bool = False,
                out: Optional[torch.Tensor] = None):
        """op.rs:10-185.  x [..., K] f16/bf16 on this device -> y [..., N] (f16 by default).
        bias (f32 [N]) is added after the f16 rounding; out_dtype f32/bf16 widens/rounds after.
        out: optional contiguous tensor of y's shape and out_dtype to write into (it is returned)."""
        if self.shard_kind == "rows":
            raise ValueError("a rows shard yields partial sums: use forward_partial + all-reduce + finalize")
        m = self._prep_x(x, self.in_features)
        shape = x.shape[:-1] + (self.out_features,)
        if out is None:
            y = torch.empty(shape, dtype=out_dtype, device=self.device)
        else:
            if out.shape != shape or out.dtype != out_dtype or out.device != self.device or not out.is_contiguous():
                raise ValueError(f"out must be a contiguous {out_dtype} tensor of shape {tuple(shape)} on {self.device}")
            y = out
        mask = torch.empty(m, dtype=torch.uint8, device=self.device) if return_routing else None
        ridx = torch.empty(max(m, 1), dtype=torch.int32, device=self.device) if return_routing else None
        nr = torch.zeros(1, dtype=torch.int32, device=self.device) if return_routing else None
        if bias is not None:
            bias = bias.to(device=self.device, dtype=torch.float32).contiguous()
        if m > 0:
            stream = torch.cuda.current_stream(self.device)
            need = self.workspace_size(m)
            ws = WORKSPACES.get(self.device, stream, need)
            check(LIB.sc_forward_ws(self._h, x.data_ptr(), _DT[x.dtype], m, y.data_ptr(), _DT[out_dtype],
                                    _ptr(bias), _ptr(mask), _ptr(ridx), _ptr(nr), ws.data_ptr(), ws.numel(),
                                    ctypes.c_void_p(stream.cuda_stream)))
        if return_routing:
            return y, mask, ridx, nr
        return y

    __call__ = forward

    def forward_partial(self, x_full: torch.Tensor, *, return_routing: bool = False):
        """For tensor parallelism: f32 contribution [..., N] of this shard (rows shard: the input
        is the whole [..., full_K] token), before the cross-shard sum and the f16 rounding."""
        m = self._prep_x(x_full, self.full_in_features if self.shard_kind == "rows" else self.in_features)
        y = torch.empty(x_full.shape[:-1] + (self.out_features,), dtype=torch.float32, device=self.device)
        mask = torch.empty(m, dtype=torch.uint8, device=self.device) if return_routing else None
        if m > 0:
            stream = torch.cuda.current_stream(self.device)
            need = self.workspace_size(m)
            ws = WORKSPACES.get(self.device, stream, need)
            check(LIB.sc_forward_partial(self._h, x_full.data_ptr(), _DT[x_full.dtype], m, y.data_ptr(),
                                         _ptr(mask), None, None, ws.data_ptr(), ws.numel(),
                                         ctypes.c_void_p(stream.cuda_stream)))
        return (y, mask) if return_routing else y


    def exchange_size(self, m: int) -> int:
        """f32 elements of the split exchange buffer for m tokens: [y_base m*N | y_delta m*N | stats m*3]."""
        return int(LIB.sc_split_exchange_floats(self._h, int(m)))

    def forward_split(self, x_slice: torch.Tensor, exchange: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Rows shard, tensor parallelism without the whole token: x_slice [..., K_slice] (this shard's
        input columns only) -> the f32 exchange buffer to be summed over the ranks (all-reduce), then
        passed to finalize_split."""
        if self.shard_kind != "rows":
            raise ValueError("forward_split needs a rows shard")
        m = self._prep_x(x_slice, self.in_features)
        size = self.exchange_size(m)
        if exchange is None:
            exchange = torch.empty(size, dtype=torch.float32, device=self.device)
        elif exchange.numel() < size or exchange.dtype != torch.float32 or not exchange.is_contiguous():
            raise ValueError(f"exchange must be a contiguous f32 tensor of >= {size} elements")
        if m > 0:
            stream = torch.cuda.current_stream(self.device)
            need = self.workspace_size(m)
            ws = WORKSPACES.get(self.device, stream, need)
            check(LIB.sc_forward_split(self._h, x_slice.data_ptr(), _DT[x_slice.dtype], m, exchange.data_ptr(),
                                       ws.data_ptr(), ws.numel(), ctypes.c_void_p(stream.cuda_stream)))
        return exchange

    def finalize_split(self, exchange: torch.Tensor, m: int, ranks: int, *, out_dtype=torch.float16,
                       bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                       return_routing: bool = False):
        """The summed exchange buffer -> y [m, N]: routed on the summed router sums, f16-rounded, bias
        after.  Tokens whose decision the f32 error bound leaves open add to self.undecided."""
        y = out if out is not None else torch.empty((m, self.out_features), dtype=out_dtype, device=self.device)
        mask = torch.empty(max(m, 1), dtype=torch.uint8, device=self.device) if return_routing else None
        if bias is not None:
            bias = bias.to(device=self.device, dtype=torch.float32).contiguous()
        if m > 0:
            check(LIB.sc_finalize_split(self._h, exchange.data_ptr(), int(m), int(ranks), y.data_ptr(),
                                        _DT[y.dtype], _ptr(bias), _ptr(mask), self.undecided.data_ptr(),
                                        ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))
        return (y, mask[:m]) if return_routing else y


def finalize(acc: torch.Tensor, *, out_dtype=torch.float16, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """f32 accumulators [..., N] -> f16 rounding (op.rs:172-178), then bias/out dtype."""
    acc = acc.contiguous()
    n = acc.shape[-1]
    m = acc.numel() // n
    y = torch.empty(acc.shape, dtype=out_dtype, device=acc.device)
    if bias is not None:
        bias = bias.to(device=acc.device, dtype=torch.float32).contiguous()
    check(LIB.sc_finalize(acc.data_ptr(), m, n, y.data_ptr(), _DT[out_dtype], _ptr(bias),
                          ctypes.c_void_p(torch.cuda.current_stream(acc.device).cuda_stream)))
    return y


def variance_heuristic(x: torch.Tensor) -> torch.Tensor:
    """heuristics.rs:3-14 per token of x [..., K] (f16/bf16/f32 on CUDA), in the reference's
    exact sequential f32 order.  Returns f32 [...]."""
    k = x.shape[-1]
    x = x.contiguous()
    m = x.numel() // k
    out = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    check(LIB.sc_variance_heuristic(x.data_ptr(), _DT[x.dtype], m, k, out.data_ptr(),
                                    ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)))
    return out


class SaccadeLinearGroup:
    """Layers that read the same input -- q, k and v, or gate and up -- computed by one launch
    (sc_group_create / sc_forward_group).  No reference counterpart (the reference applies each
    projection separately, saccade-runner/src/model.rs:217-219, 296-297); forward(x) returns one
    output per layer: the layer's own masks and routed lists, its outputs bit for bit in exact mode
    and within the fast-mode tolerance otherwise (the group may split the columns differently)."""

    def __init__(self, ops):
        ops = list(ops)
        if not 1 <= len(ops) <= 4:
            raise ValueError("a group holds 1..4 layers")
        self.ops = ops
        self.device = ops[0].device
        arr = (ctypes.c_void_p * len(ops))(*[op._h for op in ops])
        h = ctypes.c_void_p()
        check(LIB.sc_group_create(arr, len(ops), ctypes.byref(h)))
        self._h = h

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and LIB is not None:
            release_handle(LIB.sc_group_destroy, h)
            self._h = None

    def _outputs(self, x, out_dtype, outs):
        shapes = [x.shape[:-1] + (op.out_features,) for op in self.ops]
        if outs is None:
            return [torch.empty(sh, dtype=out_dtype, device=self.device) for sh in shapes]
        ys = list(outs)
        for y, sh in zip(ys, shapes):
            if y.shape != sh or y.dtype != out_dtype or not y.is_contiguous() or y.device != self.device:
                raise ValueError(f"outs must be contiguous {out_dtype} tensors of shapes {shapes}")
        return ys

    def _bias_ptrs(self, biases):
        if biases is None:
            return None
        bl = [None if b is None else b.to(device=self.device, dtype=torch.float32).contiguous() for b in biases]
        self._keep_bias = bl
        return (ctypes.c_void_p * len(bl))(*[None if b is None else b.data_ptr() for b in bl])

    def takes_routing(self, m: int) -> bool:
        """True when forward_routed serves m tokens: the group runs the 9..64-token launch."""
        return bool(LIB.sc_group_takes_routing(self._h, m, int(LIB.sc_group_workspace_size(self._h, m))))

    def forward_routed(self, x: torch.Tensor, routing: "GroupRouting", *, out_dtype: torch.dtype = torch.float16,
                       outs=None, biases=None):
        """forward(x) with the routing a fused router already wrote for x (sc_forward_group_routed):
        x is the f16 output of sc_qwen2_add_rmsnorm_route / sc_qwen2_silu_mul_route for this group."""
        if x.dtype != torch.float16:
            raise ValueError("forward_routed takes the f16 rows the fused router wrote")
        m = self.ops[0]._prep_x(x, self.ops[0].in_features)
        ys = self._outputs(x, out_dtype, outs)
        if m > 0:
            stream = torch.cuda.current_stream(self.device)
            need = int(LIB.sc_group_workspace_size(self._h, m))
            ws = WORKSPACES.get(self.device, stream, need)
            yp = (ctypes.c_void_p * len(ys))(*[y.data_ptr() for y in ys])
            check(LIB.sc_forward_group_routed(self._h, x.data_ptr(), m, yp, _DT[out_dtype], self._bias_ptrs(biases),
                                              routing.mask_p, routing.ridx_p, routing.count_p, ws.data_ptr(),
                                              ws.numel(), ctypes.c_void_p(stream.cuda_stream)))
        return ys

    def forward(self, x: torch.Tensor, *, out_dtype: torch.dtype = torch.float16, outs=None,
                return_routing: bool = False, biases=None):
        """biases: optional per-layer f32 [N] tensors (or None entries), added after the f16 rounding."""
        n = len(self.ops)
        m = self.ops[0]._prep_x(x, self.ops[0].in_features)
        ys = self._outputs(x, out_dtype, outs)
        routing = None
        if return_routing:
            routing = [(torch.empty(m, dtype=torch.uint8, device=self.device),
                        torch.empty(max(m, 1), dtype=torch.int32, device=self.device),
                        torch.zeros(1, dtype=torch.int32, device=self.device)) for _ in range(n)]
        if m > 0:
            stream = torch.cuda.current_stream(self.device)
            need = int(LIB.sc_group_workspace_size(self._h, m))
            ws = WORKSPACES.get(self.device, stream, need)
            yp = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
            mp = rp = np_ = None
            if routing is not None:
                mp = (ctypes.c_void_p * n)(*[r[0].data_ptr() for r in routing])
                rp = (ctypes.c_void_p * n)(*[r[1].data_ptr() for r in routing])
                np_ = (ctypes.c_void_p * n)(*[r[2].data_ptr() for r in routing])
            bp = self._bias_ptrs(biases)
            check(LIB.sc_forward_group(self._h, x.data_ptr(), _DT[x.dtype], m, yp, _DT[out_dtype], bp, mp, rp, np_,
                                       ws.data_ptr(), ws.numel(), ctypes.c_void_p(stream.cuda_stream)))
        if return_routing:
            return ys, routing
        return ys

    __call__ = forward


class GroupRouting:
    """The routing of a group's layers for m tokens as a fused router writes it and forward_routed
    reads it: per layer a mask [m] (u8), the ascending routed list [m] (int32) and its count (int32),
    plus the router's completion counter (zero between calls; the router leaves it zero)."""

    def __init__(self, n_layers: int, m: int, device):
        self.n, self.m = n_layers, m
        self.masks = torch.zeros((n_layers, (m + 15) // 16 * 16), dtype=torch.uint8, device=device)
        self.ridx = torch.zeros((n_layers, max(m, 1)), dtype=torch.int32, device=device)
        self.counts = torch.zeros((n_layers, 4), dtype=torch.int32, device=device)
        self.counter = torch.zeros(4, dtype=torch.int32, device=device)
        arr = ctypes.c_void_p * n_layers
        self.mask_p = arr(*[self.masks[i].data_ptr() for i in range(n_layers)])
        self.ridx_p = arr(*[self.ridx[i].data_ptr() for i in range(n_layers)])
        self.count_p = arr(*[self.counts[i].data_ptr() for i in range(n_layers)])

    def layer(self, i: int):
        """(mask [m], routed list, count) of layer i, read back to the host."""
        c = int(self.counts[i, 0].item())
        return self.masks[i, :self.m], self.ridx[i, :c], c
