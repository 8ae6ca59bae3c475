"""Row shards that see only their slice of each token (sc_forward_split / sc_finalize_split), on one
GPU: R shards of the same layer (explicit column ranges, as a tensor-parallel o or down keeps),
each fed only its input columns, their exchange buffers summed in rank order (the all-reduce), then
the routing decision on the summed router sums.  The result must equal the unsharded oracle on a
seeded sample of output rows (fast tolerance), with the oracle's routing mask and no undecided
token; each buffer's router sums must equal f64 sums of the slice.

Shapes: Qwen2-7B down (3584 x 18944, intermediate split over 2 or 8 ranks) and o (3584 x 3584,
28 heads of 128 split unevenly over 8 ranks, 4,4,4,4,3,3,3,3), M from 1 (router-fused decode) over 4, 16
(the 9..16-token GEMM) to 64 and 200 (the prefill GEMM), f16 and bf16 inputs, bypass.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from ctarq_cases import assert_fast_close, sample_rows

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


def packed(sc, n, k, fill):
    key = (n, k, fill)
    if key not in _CACHE:
        g = torch.Generator(device="cuda").manual_seed(n * 5 + k + int(fill * 1000))
        w = torch.randn(n, k, device="cuda", generator=g) * 0.02
        blocks = sc.compress_tensor_to_saccade(w, sc.compute_percentile_threshold(w, fill))
        del w
        host = {kk: v.cpu() for kk, v in blocks.items()}
        u32 = lambda t: t.view(torch.int32).numpy().view(np.uint32)  # noqa: E731
        c = O.Compressed(u32(host["packed_base"]), host["scale_base"].numpy().view(np.uint16),
                         u32(host["delta_row_ptrs"]), u32(host["delta_col_indices"]),
                         host["delta_values"].numpy().view(np.uint8),
                         int(host["delta_scale"].view(torch.int16).item()) & 0xFFFF, n, k)
        rows = np.sort(np.random.default_rng(n + k).choice(n, size=SAMPLE, replace=False))
        _CACHE[key] = (blocks, c, rows, O.OracleLinear(sample_rows(c, rows), 8.0, 3e38))
    return _CACHE[key]


def shards(sc, blocks, n, k, ranges):
    return [sc.saccade_op_from_compressed(blocks, sc.SaccadeConfig(8.0, 3e38), n, k, mode="fast",
                                          shard=("rows_range", c0, c1)) for c0, c1 in ranges]


def even_ranges(k, r):
    kb = k // 64
    return [((kb * i // r) * 64, (kb * (i + 1) // r) * 64 if i + 1 < r else k) for i in range(r)]


HEADS_8 = [(0, 512), (512, 1024), (1024, 1536), (1536, 2048), (2048, 2432), (2432, 2816), (2816, 3200),
           (3200, 3584)]

CASES = [
    # n, k, ranges, m, routed fraction, x dtype
    (3584, 18944, even_ranges(18944, 2), 1, 1.0, torch.float16),
    (3584, 18944, even_ranges(18944, 2), 4, 0.5, torch.float16),
    (3584, 18944, even_ranges(18944, 2), 16, 0.25, torch.float16),
    (3584, 18944, even_ranges(18944, 8), 64, 0.25, torch.float16),
    (3584, 18944, even_ranges(18944, 8), 200, 0.1, torch.bfloat16),
    (3584, 3584, HEADS_8, 64, 0.25, torch.float16),
    (3584, 3584, HEADS_8, 13, 0.3, torch.bfloat16),
    (3584, 3584, HEADS_8, 1, 0.0, torch.float16),
]


def run_split(ops, x, ranks):
    """forward_split per shard on its columns, the exchange buffers summed in rank order, finalize."""
    m = x.shape[0]
    total = None
    bufs = []
    for op in ops:
        ex = op.forward_split(x[:, op.col_begin:op.col_begin + op.in_features].contiguous())
        bufs.append(ex.clone())
        total = ex.clone() if total is None else total + ex
    y, mask = ops[0].finalize_split(total, m, ranks, return_routing=True)
    return y, mask, bufs


@pytest.mark.parametrize("n,k,ranges,m,frac,dtype", CASES)
def test_split_shards_match_unsharded_oracle(sc, n, k, ranges, m, frac, dtype):
    blocks, c, rows, orc = packed(sc, n, k, 0.01)
    ops = shards(sc, blocks, n, k, ranges)
    assert [(op.col_begin, op.col_begin + op.in_features) for op in ops] == ranges
    rng = np.random.default_rng(n + m)
    x = rng.standard_normal((m, k)).astype(np.float32)
    nr = int(round(frac * m))
    if nr:
        x[rng.choice(m, size=nr, replace=False)] *= 8.0
    xt = torch.from_numpy(x).to("cuda:0").to(dtype)
    y, mask, bufs = run_split(ops, xt, len(ops))
    torch.cuda.synchronize()
    for op in ops:
        op.check_device()
    assert int(ops[0].undecided.item()) == 0
    xb = xt.to(torch.float16).cpu().numpy().view(np.uint16)  # what the op reads (bf16 -> f16 first)
    y_ref, r_ref, _ = orc.forward(xb)
    assert int(r_ref.sum()) == nr
    assert np.array_equal(mask.cpu().numpy(), r_ref)
    assert_fast_close(y.cpu().numpy().view(np.uint16)[:, rows], y_ref, f"split {len(ops)} ranks m={m}")
    # the router sums of each slice equal f64 sums of its columns (rounded to f32)
    xf = xb.view(np.float16).astype(np.float64)
    for op, ex in zip(ops, bufs):
        st = ex[2 * m * n:].cpu().numpy().reshape(m, 3).astype(np.float64)
        sl = xf[:, op.col_begin:op.col_begin + op.in_features]
        ref = np.stack([sl.sum(1), (sl * sl).sum(1), np.abs(sl).sum(1)], 1)
        assert np.all(np.abs(st - ref) <= 2 ** -23 * np.abs(ref)[:, [2, 1, 2]] + 1e-30)


def test_split_bypass_routes_every_token(sc):
    blocks, c, rows, orc = packed(sc, 3584, 3584, 0.01)
    ops = shards(sc, blocks, 3584, 3584, HEADS_8)
    x = torch.randn(9, 3584, device="cuda:0").to(torch.float16)
    sc.set_bypass_c_tarq(True)
    try:
        y, mask, _ = run_split(ops, x, len(ops))
        torch.cuda.synchronize()
    finally:
        sc.set_bypass_c_tarq(False)
    y_ref, _, _ = orc.forward(x.cpu().numpy().view(np.uint16), bypass=True)
    assert mask.cpu().numpy().tolist() == [1] * 9
    assert_fast_close(y.cpu().numpy().view(np.uint16)[:, rows], y_ref, "split bypass")


def test_split_rejects_other_shards(sc):
    blocks, c, rows, orc = packed(sc, 3584, 3584, 0.01)
    col = sc.saccade_op_from_compressed(blocks, sc.SaccadeConfig(8.0, 3e38), 3584, 3584,
                                        shard=("columns_range", 0, 512))
    assert (col.out_features, col.in_features, col.row_begin) == (512, 3584, 0)
    with pytest.raises(ValueError):
        col.forward_split(torch.zeros(1, 3584, dtype=torch.float16, device="cuda:0"))
    with pytest.raises(sc.CTarqError):
        sc.saccade_op_from_compressed(blocks, sc.SaccadeConfig(8.0, 3e38), 3584, 3584,
                                      shard=("rows_range", 32, 512))  # not on a 64-column boundary
