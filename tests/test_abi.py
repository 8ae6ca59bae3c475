"""CPU checks of the C-ABI library: it loads without a GPU, exports exactly the entry
points include/saccade_ctarq.h declares, and its host-only calls behave."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "saccade_ctarq.h")
HEADER_QWEN2 = os.path.join(ROOT, "include", "saccade_qwen2.h")


def declared_symbols(path=HEADER):
    text = open(path).read()
    return sorted(set(re.findall(r"^SC_API\s+[\w\s\*]+?\b(sc_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for must in ("sc_layer_create", "sc_forward", "sc_forward_ws", "sc_op_name", "sc_compress", "sc_calibrate"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from saccade_core import _lib
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(declared_symbols()) == set(_lib.SIGNATURES), "ctypes signatures must cover the header exactly"
    for name in declared_symbols(HEADER_QWEN2):
        assert hasattr(lib, name), f"{name} declared in saccade_qwen2.h but not exported"
    assert set(declared_symbols(HEADER_QWEN2)) == set(_lib.SIGNATURES_QWEN2)


def test_only_c_abi_is_exported():
    from saccade_core import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True, check=True)
    funcs = [ln.split()[-1] for ln in out.stdout.splitlines() if " T " in ln]
    assert funcs and all(f.startswith("sc_") for f in funcs), [f for f in funcs if not f.startswith("sc_")][:10]


def test_host_only_calls():
    from saccade_core import _lib
    L = _lib.LIB
    assert L.sc_op_name() == b"fused_c_tarq_saccade_linear"
    assert L.sc_abi_version() == 2  # 2: explicit shard ranges in sc_layer_desc
    assert ctypes.sizeof(_lib.ScLayerDesc) == 120  # the C struct's size on x86-64
    assert isinstance(L.sc_launch_count(), int)
    L.sc_set_bypass_c_tarq(1)
    assert L.sc_is_c_tarq_bypassed() == 1
    L.sc_set_bypass_c_tarq(0)
    assert L.sc_is_c_tarq_bypassed() == 0


def test_invalid_arguments_fail_before_touching_a_device():
    from saccade_core import _lib
    L = _lib.LIB
    d = _lib.ScLayerDesc()
    d.out_features, d.in_features = 4, 12  # K % 8 != 0
    h = ctypes.c_void_p()
    assert L.sc_layer_create(ctypes.byref(d), ctypes.byref(h)) == _lib.SC_EINVAL
    assert "multiple of 8" in _lib.last_error()
    assert L.sc_layer_create(None, ctypes.byref(h)) == _lib.SC_EINVAL
    assert L.sc_forward(None, None, 0, 1, None, 0, None, None, None, None, None) == _lib.SC_EINVAL
    assert L.sc_finalize(None, 1, 1, None, 0, None, None) == _lib.SC_EINVAL
    assert L.sc_workspace_size(None, 4) == 0


def test_error_type_is_raised():
    from saccade_core import _lib
    with pytest.raises(_lib.CTarqError):
        _lib.check(_lib.SC_EINVAL)


def test_routed_group_entry_points_validate_on_the_host():
    """The fused-router entry points reject missing groups, routing arrays or counters, and the
    routed GEMM rejects missing routing, before any device call."""
    from saccade_core import _lib
    L = _lib.LIB
    arr = (ctypes.c_void_p * 1)(None)
    buf = ctypes.create_string_buffer(64)
    assert L.sc_group_takes_routing(None, 16, 1 << 20) == 0
    assert L.sc_forward_group_routed(None, buf, 16, arr, _lib.SC_F16, None, arr, arr, arr, None, 0, None) == _lib.SC_EINVAL
    assert L.sc_qwen2_add_rmsnorm_route(buf, None, buf, 16, 896, ctypes.c_float(1e-6), buf, None, arr, arr, arr, buf,
                                        None) == _lib.SC_EINVAL
    assert "null group" in _lib.last_error()
    assert L.sc_qwen2_add_rmsnorm_route(buf, None, buf, 16, 900, ctypes.c_float(1e-6), buf, None, arr, arr, arr, buf,
                                        None) == _lib.SC_EINVAL  # hidden not a multiple of 8
    assert L.sc_qwen2_silu_mul_route(buf, buf, 16, 1020, buf, None, arr, arr, arr, buf, None) == _lib.SC_EINVAL
    assert L.sc_qwen2_add_rmsnorm_route(buf, None, buf, 0, 896, ctypes.c_float(1e-6), buf, None, arr, arr, arr, buf,
                                        None) == _lib.SC_OK  # no tokens: nothing to do


def test_group_routing_buffers_layout():
    """GroupRouting: per layer a 16-byte-padded mask row, a routed list and a 16-byte count slot,
    and pointer arrays that address exactly those rows."""
    torch = pytest.importorskip("torch")
    from saccade_core import GroupRouting
    r = GroupRouting(3, 21, "cpu")
    assert r.masks.shape == (3, 32) and r.masks.dtype == torch.uint8
    assert r.ridx.shape == (3, 21) and r.counts.shape == (3, 4)
    assert int(r.counter.sum()) == 0
    for i in range(3):
        assert r.mask_p[i] == r.masks[i].data_ptr()
        assert r.ridx_p[i] == r.ridx[i].data_ptr()
        assert r.count_p[i] == r.counts[i].data_ptr()
    r.counts[1, 0] = 2
    r.ridx[1, :2] = torch.tensor([4, 9], dtype=torch.int32)
    mask, ridx, c = r.layer(1)
    assert c == 2 and ridx.tolist() == [4, 9] and mask.shape == (21,)
