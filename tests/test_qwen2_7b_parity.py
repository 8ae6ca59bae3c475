"""GPU parity on the Qwen2-7B projection shapes at the token counts, routed fractions and dW
densities of the single-call sweep (gate/up 18944 x 3584, down 3584 x 18944; M up to 1024;
0 / 25 / 100 % routed; 0.5 % and 4 % dW).

The layer runs whole on the GPU; the oracle checks a seeded sample of 256 output rows (the
packed rows, scales and CSR rows of those rows, with the matrix's own dW scale), which keeps
its time bounded without shrinking K.  Routed tokens are the boosted ones (x8, variance ~64)
under t4 = 8, so the routed fraction is exact.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from ctarq_cases import Case, assert_acc_close, assert_fast_close, sample_rows

pytestmark = pytest.mark.gpu

SAMPLE = 256
_CACHE = {}


@pytest.fixture(scope="module")
def sc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import saccade_core
    saccade_core.set_bypass_c_tarq(False)
    return saccade_core


def packed_layer(sc, n, k, fill):
    """W ~ N(0, 0.02) packed on the GPU (bit-identical to the oracle's packer, tested elsewhere)."""
    key = (n, k, fill)
    if key not in _CACHE:
        g = torch.Generator(device="cuda").manual_seed(n * 7 + k + int(fill * 1000))
        w = torch.randn(n, k, device="cuda", generator=g) * 0.02
        thr = sc.compute_percentile_threshold(w, fill)
        blocks = sc.compress_tensor_to_saccade(w, thr)
        del w
        host = {kk: v.cpu() for kk, v in blocks.items()}
        u32 = lambda t: t.view(torch.int32).numpy().view(np.uint32)
        c = O.Compressed(u32(host["packed_base"]), host["scale_base"].numpy().view(np.uint16),
                         u32(host["delta_row_ptrs"]), u32(host["delta_col_indices"]),
                         host["delta_values"].numpy().view(np.uint8),
                         int(host["delta_scale"].view(torch.int16).item()) & 0xFFFF, n, k)
        op = sc.saccade_op_from_compressed(blocks, sc.SaccadeConfig(8.0, 3e38), n, k, mode="fast")
        rows = np.sort(np.random.default_rng(n + k).choice(n, size=SAMPLE, replace=False))
        _CACHE[key] = (op, c, rows, O.OracleLinear(sample_rows(c, rows), 8.0, 3e38))
    return _CACHE[key]


def tokens(k, m, routed_frac, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    nr = int(round(routed_frac * m))
    boost = rng.choice(m, size=nr, replace=False) if nr else []
    x[boost] *= 8.0
    return x.astype(np.float16).view(np.uint16), nr


CASES = [
    # n, k, fill, m, routed fraction
    *[(18944, 3584, 0.04, m, f) for m in (64, 256, 1024) for f in (0.0, 0.25, 1.0)],
    *[(3584, 18944, 0.005, m, f) for m in (64, 256, 1024) for f in (0.0, 0.25, 1.0)],
    (18944, 3584, 0.005, 64, 0.25),
    (3584, 18944, 0.04, 64, 0.25),
    (3584, 18944, 0.04, 16, 0.25),
    (3584, 18944, 0.04, 1, 1.0),     # one routed token, dense dW: the in-place dW block walk
    (18944, 3584, 0.04, 1, 1.0),
    (3584, 18944, 0.005, 4, 0.5),
]


@pytest.mark.parametrize("n,k,fill,m,frac", CASES)
def test_qwen2_7b_shape_sampled_rows(sc, n, k, fill, m, frac):
    op, c, rows, orc = packed_layer(sc, n, k, fill)
    xb, nr = tokens(k, m, frac, seed=n + 3 * m + int(frac * 100))
    x = torch.from_numpy(xb.view(np.float16)).to("cuda:0")
    y, mask, ridx, nrt = op.forward(x, return_routing=True)
    acc = op.forward_partial(x)
    torch.cuda.synchronize()
    op.check_device()
    yr, rr, acc_ref = orc.forward(xb)
    assert int(rr.sum()) == nr
    assert np.array_equal(mask.cpu().numpy(), rr), "router mask must equal the reference's"
    assert np.array_equal(ridx.cpu().numpy()[: int(nrt.item())], np.nonzero(rr)[0])
    yg = y.cpu().numpy().view(np.uint16)[:, rows]
    assert_fast_close(yg, yr, f"{n}x{k} dW {fill} m={m} routed {nr}")
    assert_acc_close(acc.cpu().numpy()[:, rows], acc_ref, f"{n}x{k} dW {fill} m={m} routed {nr} acc")
