"""sc_forward_static: the forward with a static, library-owned scratch array.

Collected last on purpose (file name), so it runs both on its own and after every other
test has left its workspaces, layers and bypass setting behind.  Each case runs the existing
entry point (sc_forward_ws with a caller workspace) and then sc_forward_static twice in a row
on the same inputs; the static calls must reproduce it bit for bit, router outputs included,
and must not change the device's free memory.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from ctarq_cases import make_case

pytestmark = pytest.mark.gpu

STATIC_BYTES = 8 * 1024 * 1024  # SC_STATIC_SCRATCH_BYTES


@pytest.fixture(scope="module")
def sc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import saccade_core
    saccade_core.set_bypass_c_tarq(False)
    return saccade_core


def make_op(sc, case, mode):
    dev = torch.device("cuda", 0)
    c = case.c

    def t(a, dt):
        return torch.from_numpy(np.ascontiguousarray(a).view(dt)).to(dev)

    sp = None
    if c.nnz:
        sp = sc.SparseDeltaMatrix(t(c.delta_row_ptrs, np.int32), t(c.delta_col_indices, np.int32),
                                  t(c.delta_values, np.uint8),
                                  torch.tensor([c.delta_scale], dtype=torch.int16).view(torch.float16))
    return sc.SaccadeLinearOp(t(c.packed_base, np.int32), t(c.scale_base, np.float16), sp,
                              sc.SaccadeConfig(case.t4, case.t8), case.n, case.k, device=dev, mode=mode)


def outputs(m, n):
    dev = torch.device("cuda", 0)
    return (torch.empty(m, n, dtype=torch.float16, device=dev), torch.empty(m, dtype=torch.uint8, device=dev),
            torch.empty(m, dtype=torch.int32, device=dev), torch.empty(1, dtype=torch.int32, device=dev))


def call_static(sc, op, x, y, mask, ridx, nr):
    from saccade_core._lib import LIB, SC_F16, check
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(LIB.sc_forward_static(op._h, x.data_ptr(), SC_F16, x.shape[0], y.data_ptr(), SC_F16, None,
                                mask.data_ptr(), ridx.data_ptr(), nr.data_ptr(), stream))


def call_ws(sc, op, x, y, mask, ridx, nr):
    from saccade_core._lib import LIB, SC_F16, check
    m = x.shape[0]
    ws = torch.zeros(LIB.sc_workspace_size(op._h, m), dtype=torch.uint8, device=x.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(LIB.sc_forward_ws(op._h, x.data_ptr(), SC_F16, m, y.data_ptr(), SC_F16, None, mask.data_ptr(),
                            ridx.data_ptr(), nr.data_ptr(), ws.data_ptr(), ws.numel(), stream))


def host(y, mask, ridx, nr):
    k = int(nr.item())
    return (y.cpu().numpy().view(np.uint16), mask.cpu().numpy(), ridx.cpu().numpy()[:k])


@pytest.mark.parametrize("n,k,m,mode", [
    (4864, 896, 8, "fast"),      # router folded into the decode kernel, split-K partials
    (512, 3584, 1, "fast"),      # one token, many column splits
    (1000, 512, 40, "fast"),     # router kernel, then two token chunks of the tensor-core kernel
    (300, 1024, 5, "exact"),     # router kernel, then the exact CUDA-core kernel
])
def test_static_matches_workspace_entry(sc, n, k, m, mode):
    case = make_case(n, k, m, 0.02, seed=7 * n + m)
    op = make_op(sc, case, mode)
    x = torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")
    ref = outputs(m, n)
    call_ws(sc, op, x, *ref)
    torch.cuda.synchronize()
    want = host(*ref)
    assert want[2].size > 0, "the case should route at least one token"

    got = [outputs(m, n) for _ in range(2)]
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info(0)[0]      # sc_layer_create has already looked the array up
    call_static(sc, op, x, *got[0])
    call_static(sc, op, x, *got[1])
    call_static(sc, op, x, *got[0])
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info(0)[0] == free0, "sc_forward_static must not allocate device memory"
    op.check_device()
    for g in got:
        h = host(*g)
        assert np.array_equal(h[0], want[0]), "y differs from sc_forward_ws"
        assert np.array_equal(h[1], want[1])
        assert np.array_equal(h[2], want[2])


def test_static_rejects_oversize_and_bad_input(sc):
    from saccade_core._lib import LIB, SC_EINVAL, SC_F16, last_error
    case = make_case(256, 896, 4, 0.02, seed=3)
    op = make_op(sc, case, "fast")
    m = 5000
    assert LIB.sc_workspace_size(op._h, m) > STATIC_BYTES
    x = torch.zeros(m, 896, dtype=torch.float16, device="cuda:0")
    y = torch.empty(m, 256, dtype=torch.float16, device="cuda:0")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    st = LIB.sc_forward_static(op._h, x.data_ptr(), SC_F16, m, y.data_ptr(), SC_F16, None, None, None, None, stream)
    assert st == SC_EINVAL
    assert "use sc_forward_ws" in last_error()
    st = LIB.sc_forward_static(op._h, x.data_ptr(), SC_F16, -1, y.data_ptr(), SC_F16, None, None, None, None, stream)
    assert st == SC_EINVAL
    st = LIB.sc_forward_static(None, x.data_ptr(), SC_F16, 4, y.data_ptr(), SC_F16, None, None, None, None, stream)
    assert st == SC_EINVAL
    # a rejected call leaves the entry point usable
    xs = torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")
    a, b = outputs(4, 256), outputs(4, 256)
    call_ws(sc, op, xs, *a)
    call_static(sc, op, xs, *b)
    torch.cuda.synchronize()
    assert np.array_equal(host(*a)[0], host(*b)[0])
