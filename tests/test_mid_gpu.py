"""The 9..64-token path (batched decode): the router kernel, then the tcgen05 f16 GEMM with the
tokens as the MMA's N side; dW of the routed tokens from the staged token tiles (9..16 tokens), or
from 17 tokens folded into a second tensor-memory A, (q - 8) + dW/s, whose products the routed
tokens take (layers whose fold lists exceed 8 KB, e.g. 30 % dW, keep the staged-tile path).

The products are exact (f16 tokens times integers q - 8, f32 accumulation); these cases cover wide
dynamic ranges, tiny and huge values, a single outlier, subnormals, non-finite inputs, groups with
per-layer thresholds, column splits with f32 partials, rows shards, bf16 and unaligned input, all
against the oracle under the fast-mode tolerance, with masks and routed lists identical.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from ctarq_cases import assert_acc_close, assert_fast_close, make_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import saccade_core
    saccade_core.set_bypass_c_tarq(False)
    return saccade_core


def to_op(sc, case, mode="fast", shard=None):
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
                              sc.SaccadeConfig(case.t4, case.t8), case.n, case.k, device=dev, mode=mode, shard=shard)


def run(op, x_bits):
    x = torch.from_numpy(x_bits.view(np.float16)).to("cuda:0")
    y, mask, ridx, nr = op.forward(x, return_routing=True)
    torch.cuda.synchronize()
    op.check_device()
    return y.cpu().numpy().view(np.uint16), mask.cpu().numpy(), ridx.cpu().numpy()[: int(nr.item())]


@pytest.mark.parametrize("n,k,m,fill", [
    (4864, 896, 16, 0.01),    # the single-layer configuration
    (3584, 3584, 64, 0.01),   # q/o at batch 64: column splits, f32 partials
    (512, 3584, 33, 0.02),    # k/v
    (1000, 520, 9, 0.04),     # the smallest token count; K not a multiple of 64
    (130, 200, 64, 0.3),      # ragged rows, dense dW
    (18944, 3584, 24, 0.01),  # gate/up: one CTA per row tile
])
@pytest.mark.parametrize("mode", ["fast", "fast_tc"])
def test_mid_matches_oracle(sc, n, k, m, fill, mode):
    case = make_case(n, k, m, fill, seed=n + 5 * m)
    op = to_op(sc, case, mode)
    y, mask, ridx = run(op, case.x_bits)
    yr, rr, acc_ref = case.oracle().forward(case.x_bits)
    assert rr.any() and not rr.all()
    assert np.array_equal(mask, rr)
    assert np.array_equal(ridx, np.nonzero(rr)[0])
    assert_fast_close(y, yr, f"mid {n}x{k} m={m}")
    acc = op.forward_partial(torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")).cpu().numpy()
    assert_acc_close(acc, acc_ref, f"mid acc {n}x{k} m={m}")


@pytest.mark.parametrize("kind", ["wide", "tiny", "outlier", "huge", "zero_token", "subnormal"])
@pytest.mark.parametrize("m", [12, 64])
def test_mid_extreme_inputs(sc, kind, m):
    n, k = 768, 2048
    case = make_case(n, k, m, 0.02, seed=66, boost=[0])
    rng = np.random.default_rng(m)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if kind == "wide":
        x *= 10.0 ** rng.uniform(-7, 4, (m, k))
    elif kind == "tiny":
        x *= 1e-6
    elif kind == "outlier":
        x[:, 7] = 3.0e4      # one huge channel per token: every other element sits far below the max
    elif kind == "huge":
        x *= 8000.0
    elif kind == "zero_token":
        x[1] = 0.0
    else:
        x *= 3e-7            # f16 subnormals
    case.x_bits = x.astype(np.float16).view(np.uint16)
    yr, rr, acc_ref = case.oracle().forward(case.x_bits)
    op = to_op(sc, case)
    y, mask, _ = run(op, case.x_bits)
    assert np.array_equal(mask, rr)
    assert_fast_close(y, yr, f"{kind} m={m}")
    acc = op.forward_partial(torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")).cpu().numpy()
    assert_acc_close(acc, acc_ref, f"{kind} m={m} acc")


@pytest.mark.parametrize("what", ["inf", "neg_inf", "nan"])
def test_mid_non_finite_token(sc, what):
    n, k, m = 384, 1024, 12
    case = make_case(n, k, m, 0.02, seed=13, boost=[2])
    x = np.random.default_rng(3).standard_normal((m, k)).astype(np.float32)
    x[5, 300] = {"inf": np.inf, "neg_inf": -np.inf, "nan": np.nan}[what]
    case.x_bits = x.astype(np.float16).view(np.uint16)
    yr, rr, _ = case.oracle().forward(case.x_bits)
    op = to_op(sc, case)
    y, mask, _ = run(op, case.x_bits)
    assert np.array_equal(mask, rr)
    got = y.view(np.float16).astype(np.float32)
    ref = yr.view(np.float16).astype(np.float32)
    assert np.array_equal(np.isnan(got[5]), np.isnan(ref[5]))
    assert np.array_equal(np.isposinf(got[5]), np.isposinf(ref[5]))
    assert np.array_equal(np.isneginf(got[5]), np.isneginf(ref[5]))
    keep = np.ones(m, bool)
    keep[5] = False
    assert_fast_close(np.ascontiguousarray(y[keep]), np.ascontiguousarray(yr[keep]), "finite tokens")


def test_mid_bf16_and_bypass(sc):
    case = make_case(900, 1536, 20, 0.03, seed=17)
    xf = case.x_bits.view(np.float16).astype(np.float32)
    xbf = torch.from_numpy(xf).to(torch.bfloat16)
    from oracle import oracle as O
    x16 = O.bf16_bits_to_f16_bits(xbf.view(torch.int16).numpy().view(np.uint16))
    op = to_op(sc, case)
    y, mask, _, _ = op.forward(xbf.to("cuda:0"), return_routing=True)
    torch.cuda.synchronize()
    yr, rr, _ = case.oracle().forward(x16)
    assert np.array_equal(mask.cpu().numpy(), rr)
    assert_fast_close(y.cpu().numpy().view(np.uint16), yr, "bf16")
    try:
        sc.set_bypass_c_tarq(True)
        y, mask, _ = run(op, case.x_bits)
        yr, _, _ = case.oracle().forward(case.x_bits, bypass=True)
        assert mask.all()
        assert_fast_close(y, yr, "bypass")
    finally:
        sc.set_bypass_c_tarq(False)


@pytest.mark.parametrize("shapes,m", [
    ([(3584, 3584), (512, 3584), (512, 3584)], 64),   # q, k, v at batch 64
    ([(2048, 1024), (2048, 1024)], 16),               # gate/up-like pair
    ([(256, 512), (128, 512), (384, 512), (130, 512)], 40),
])
def test_mid_group_one_launch(sc, shapes, m):
    k = shapes[0][1]
    cases = [make_case(n, k, m, 0.02, seed=2000 + i, boost=[0, 3, m - 1]) for i, (n, _) in enumerate(shapes)]
    for i, c in enumerate(cases):
        c.t4 = c.t4 * (1.0 + 0.1 * i)   # per-layer thresholds differ
    x_bits = cases[0].x_bits
    for c in cases:
        c.x_bits = x_bits
    ops = [to_op(sc, c) for c in cases]
    grp = sc.SaccadeLinearGroup(ops)
    x = torch.from_numpy(x_bits.view(np.float16)).to("cuda:0")
    ys, routing = grp.forward(x, return_routing=True)
    torch.cuda.synchronize()
    for op, c, y, (mask, ridx, nr) in zip(ops, cases, ys, routing):
        op.check_device()
        yr, rr, _ = c.oracle().forward(x_bits)
        assert np.array_equal(mask.cpu().numpy(), rr)
        assert np.array_equal(ridx.cpu().numpy()[: int(nr.item())], np.nonzero(rr)[0])
        assert_fast_close(y.cpu().numpy().view(np.uint16), yr, f"group {c.n}x{c.k} m={m}")


@pytest.mark.parametrize("count", [2, 3])
def test_mid_rows_shards(sc, count):
    case = make_case(640, 2048, 24, 0.03, seed=51)
    _, rr, acc_ref = case.oracle().forward(case.x_bits)
    x = torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")
    total = None
    for i in range(count):
        op = to_op(sc, case, shard=("rows", i, count))
        part, mask = op.forward_partial(x, return_routing=True)
        torch.cuda.synchronize()
        op.check_device()
        assert np.array_equal(mask.cpu().numpy(), rr), "every shard routes on the whole token"
        total = part if total is None else total + part
    assert_acc_close(total.cpu().numpy(), acc_ref, "rows shards, 24 tokens")


def test_mid_unaligned_input(sc):
    # a token matrix starting 2 bytes past an aligned address: staged through an aligned copy
    case = make_case(640, 1024, 20, 0.02, seed=23)
    flat = torch.empty(20 * 1024 + 1, dtype=torch.float16, device="cuda:0")
    x = flat[1:].view(20, 1024)
    x.copy_(torch.from_numpy(case.x_bits.view(np.float16)))
    assert x.data_ptr() % 16 != 0
    op = to_op(sc, case)
    y, mask, _, _ = op.forward(x, return_routing=True)
    torch.cuda.synchronize()
    op.check_device()
    yr, rr, _ = case.oracle().forward(case.x_bits)
    assert np.array_equal(mask.cpu().numpy(), rr)
    assert_fast_close(y.cpu().numpy().view(np.uint16), yr, "unaligned x")


def test_mid_deterministic(sc):
    case = make_case(3584, 3584, 48, 0.01, seed=5)
    op = to_op(sc, case)
    first = run(op, case.x_bits)[0]
    for _ in range(3):
        assert np.array_equal(run(op, case.x_bits)[0], first)
