"""ctypes binding of libsaccade_ctarq.so (declarations in include/saccade_ctarq.h).

The CUDA library is the only compute path: if it is missing this module raises at
import time instead of falling back to anything else.
"""
from __future__ import annotations

import ctypes
import os

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("SACCADE_CTARQ_LIB", os.path.join(PKG_ROOT, "libsaccade_ctarq.so"))

SC_OK, SC_EINVAL, SC_ENONCONTIG, SC_ECUDA, SC_ETIMEOUT, SC_EDEVICE, SC_ENOMEM, SC_EUNSUPPORTED = range(8)
SC_F16, SC_BF16, SC_F32 = 0, 1, 2
SC_MODE_FAST, SC_MODE_EXACT, SC_MODE_FAST_TC, SC_MODE_FAST_TC8 = 0, 1, 2, 3
SC_SHARD_NONE, SC_SHARD_COLUMNS, SC_SHARD_ROWS = 0, 1, 2

STATUS_NAMES = {
    SC_OK: "SC_OK", SC_EINVAL: "SC_EINVAL", SC_ENONCONTIG: "SC_ENONCONTIG", SC_ECUDA: "SC_ECUDA",
    SC_ETIMEOUT: "SC_ETIMEOUT", SC_EDEVICE: "SC_EDEVICE", SC_ENOMEM: "SC_ENOMEM", SC_EUNSUPPORTED: "SC_EUNSUPPORTED",
}


class ScLayerDesc(ctypes.Structure):
    _fields_ = [
        ("out_features", ctypes.c_int64),
        ("in_features", ctypes.c_int64),
        ("packed_base", ctypes.c_void_p),
        ("scale_base", ctypes.c_void_p),
        ("delta_row_ptrs", ctypes.c_void_p),
        ("delta_col_indices", ctypes.c_void_p),
        ("delta_values", ctypes.c_void_p),
        ("delta_nnz", ctypes.c_int64),
        ("delta_scale", ctypes.c_uint16),
        ("t4", ctypes.c_float),
        ("t8", ctypes.c_float),
        ("device", ctypes.c_int),
        ("buffers_on_device", ctypes.c_int),
        ("mode", ctypes.c_int),
        ("shard_kind", ctypes.c_int),
        ("shard_index", ctypes.c_int),
        ("shard_count", ctypes.c_int),
        ("shard_begin", ctypes.c_int64),
        ("shard_end", ctypes.c_int64),
    ]


class ScLayerInfo(ctypes.Structure):
    _fields_ = [
        ("out_features", ctypes.c_int64),
        ("in_features", ctypes.c_int64),
        ("row_begin", ctypes.c_int64),
        ("col_begin", ctypes.c_int64),
        ("full_out_features", ctypes.c_int64),
        ("full_in_features", ctypes.c_int64),
        ("delta_nnz", ctypes.c_int64),
        ("device_bytes", ctypes.c_int64),
        ("t4", ctypes.c_float),
        ("t8", ctypes.c_float),
        ("mode", ctypes.c_int),
        ("device", ctypes.c_int),
    ]


class CTarqError(RuntimeError):
    """A C-ABI call returned a status other than SC_OK."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float

# name -> (restype, argtypes); the authoritative list of exported entry points
SIGNATURES = {
    "sc_abi_version": (_int, []),
    "sc_op_name": (ctypes.c_char_p, []),
    "sc_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
    "sc_layer_create": (_int, [ctypes.POINTER(ScLayerDesc), ctypes.POINTER(_vp)]),
    "sc_layer_destroy": (None, [_vp]),
    "sc_layer_get_info": (_int, [_vp, ctypes.POINTER(ScLayerInfo)]),
    "sc_layer_set_thresholds": (_int, [_vp, _f32, _f32]),
    "sc_layer_set_mode": (_int, [_vp, _int]),
    "sc_layer_check": (_int, [_vp, _vp]),
    "sc_set_bypass_c_tarq": (None, [_int]),
    "sc_is_c_tarq_bypassed": (_int, []),
    "sc_test_drop_weight_copy": (None, [_int]),
    "sc_workspace_size": (ctypes.c_size_t, [_vp, _i64]),
    "sc_forward": (_int, [_vp, _vp, _int, _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp]),
    "sc_forward_ws": (_int, [_vp, _vp, _int, _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "sc_forward_static": (_int, [_vp, _vp, _int, _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp]),
    "sc_group_create": (_int, [_vp, _int, _vp]),
    "sc_group_destroy": (None, [_vp]),
    "sc_group_workspace_size": (ctypes.c_size_t, [_vp, _i64]),
    "sc_forward_group": (_int, [_vp, _vp, _int, _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "sc_group_takes_routing": (_int, [_vp, _i64, ctypes.c_size_t]),
    "sc_forward_group_routed": (_int, [_vp, _vp, _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "sc_forward_partial": (_int, [_vp, _vp, _int, _i64, _vp, _vp, _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "sc_finalize": (_int, [_vp, _i64, _i64, _vp, _int, _vp, _vp]),
    "sc_split_exchange_floats": (ctypes.c_size_t, [_vp, _i64]),
    "sc_forward_split": (_int, [_vp, _vp, _int, _i64, _vp, _vp, ctypes.c_size_t, _vp]),
    "sc_finalize_split": (_int, [_vp, _vp, _i64, _int, _vp, _int, _vp, _vp, _vp, _vp]),
    "sc_launch_count": (ctypes.c_uint64, []),
    "sc_variance_heuristic": (_int, [_vp, _int, _i64, _i64, _vp, _vp]),
    "sc_percentile_threshold": (_int, [_vp, _i64, _i64, _f32, ctypes.POINTER(_f32), _vp]),
    "sc_compress": (_int, [_vp, _i64, _i64, _f32, _vp, _vp, _vp, _vp, _vp, _i64, ctypes.POINTER(_i64),
                           ctypes.POINTER(ctypes.c_uint16), _vp]),
    "sc_calibrate": (_int, [_vp, _int, _i64, _i64, _f32, _f32, ctypes.POINTER(_f32), ctypes.POINTER(_f32), _vp]),
}

# the Qwen2 decoder glue (include/saccade_qwen2.h)
SIGNATURES_QWEN2 = {
    "sc_qwen2_embed": (_int, [_vp, _i64, _vp, _i64, _i64, _vp, _vp, _vp]),
    "sc_qwen2_add_rmsnorm": (_int, [_vp, _vp, _vp, _i64, _i64, _f32, _vp, _int, _vp]),
    "sc_qwen2_rope_append": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _int, _vp, _vp, _vp]),
    "sc_qwen2_attention_scratch": (ctypes.c_size_t, [_i64, _int, _int, _int, _int]),
    "sc_qwen2_attention": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _int, _int, _vp, ctypes.c_size_t,
                                  _vp, _vp]),
    "sc_qwen2_silu_mul": (_int, [_vp, _vp, _i64, _vp, _vp]),
    "sc_qwen2_add_rmsnorm_route": (_int, [_vp, _vp, _vp, _i64, _i64, _f32, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sc_qwen2_silu_mul_route": (_int, [_vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "sc_qwen2_f16_to_f32": (_int, [_vp, _i64, _vp, _vp]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libsaccade_ctarq.so not found at {LIB_PATH}; build it with "
            "`make -C saccade-x2_b200/csrc` (or __graft_entry__.build()). There is no fallback path.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in list(SIGNATURES.items()) + list(SIGNATURES_QWEN2.items()):
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    LIB.sc_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> None:
    if status != SC_OK:
        raise CTarqError(status, last_error())
