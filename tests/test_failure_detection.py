"""Failure detection without a GPU fault: a bounded device wait that runs out.

sc_test_drop_weight_copy makes the one-token decode kernel's producer skip its first weight
copy, so the base-product warps wait on a ring stage that nothing ever completes.  The wait is
bounded (2 s of %globaltimer): the kernel records SC_ETIMEOUT in the layer's device status word
and returns.  The test checks that status through sc_layer_check, then turns the hook off and
shows that the same layer, in the same context, computes the oracle's result again.
"""
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from ctarq_cases import assert_fast_close, make_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import saccade_core
    return saccade_core


def test_bounded_wait_runs_out_and_context_stays_usable(sc):
    from saccade_core._lib import LIB, SC_ETIMEOUT
    # 128 x 128: one 128-row tile of two 64-column blocks, so the decode has one CTA (no cluster)
    # and a single weight stage; one token takes the integer engine of SC_MODE_FAST
    case = make_case(128, 128, 1, 0.05, seed=91, boost=[0], thresholds=(8.0, 3e38))
    dev = torch.device("cuda", 0)
    c = case.c

    def t(a, dt):
        return torch.from_numpy(np.ascontiguousarray(a).view(dt)).to(dev)

    sp = sc.SparseDeltaMatrix(t(c.delta_row_ptrs, np.int32), t(c.delta_col_indices, np.int32),
                              t(c.delta_values, np.uint8),
                              torch.tensor([c.delta_scale], dtype=torch.int16).view(torch.float16))
    op = sc.SaccadeLinearOp(t(c.packed_base, np.int32), t(c.scale_base, np.float16), sp,
                            sc.SaccadeConfig(case.t4, case.t8), case.n, case.k, device=dev, mode="fast")
    x = torch.from_numpy(case.x_bits.view(np.float16)).to(dev)
    yr, rr, _ = case.oracle().forward(case.x_bits)
    assert rr[0] == 1, "the token is routed, so the dW path runs beside the stalled weights"

    y = op.forward(x)  # healthy call first
    torch.cuda.synchronize()
    op.check_device()
    assert_fast_close(y.cpu().numpy().view(np.uint16), yr, "before the injected stall")

    LIB.sc_test_drop_weight_copy(1)
    try:
        t0 = time.time()
        op.forward(x)
        torch.cuda.synchronize()
        waited = time.time() - t0
    finally:
        LIB.sc_test_drop_weight_copy(0)
    with pytest.raises(sc.CTarqError) as err:
        op.check_device()
    assert err.value.status == SC_ETIMEOUT
    assert 1.0 < waited < 30.0, f"the wait is bounded near 2 s, took {waited:.2f} s"

    # the status word was cleared by the check; the same layer works again
    y2 = op.forward(x)
    torch.cuda.synchronize()
    op.check_device()
    assert_fast_close(y2.cpu().numpy().view(np.uint16), yr, "after the injected stall")
