"""GPU parity of the CUDA library against the oracle, through the C ABI (ctypes).

Exact mode must be bit-identical to the oracle; the fast (tensor-core) mode must keep
router masks identical and outputs within the tolerance of ctarq_cases.TOL_REL_RMS.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O
from ctarq_cases import assert_acc_close, assert_fast_close, make_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import saccade_core
    return saccade_core


def to_op(sc, case, mode="fast", on_device=True, shard=None):
    c = case.c
    dev = torch.device("cuda", 0)

    def t(a, dt):
        x = torch.from_numpy(np.ascontiguousarray(a).view(dt))
        return x.to(dev) if on_device else x

    sp = None
    if c.nnz:
        sp = sc.SparseDeltaMatrix(t(c.delta_row_ptrs, np.int32), t(c.delta_col_indices, np.int32),
                                  t(c.delta_values, np.uint8),
                                  torch.tensor([c.delta_scale], dtype=torch.int16).view(torch.float16))
    return sc.SaccadeLinearOp(t(c.packed_base, np.int32), t(c.scale_base, np.float16), sp,
                              sc.SaccadeConfig(case.t4, case.t8), case.n, case.k, device=dev, mode=mode,
                              shard=shard)


def run_gpu(op, x_bits, dtype=torch.float16, **kw):
    x = torch.from_numpy(x_bits.view(np.float16)).to("cuda:0")
    if dtype == torch.bfloat16:
        x = x.to(torch.bfloat16)
    y, mask, ridx, nr = op.forward(x, return_routing=True, **kw)
    torch.cuda.synchronize()
    op.check_device()
    return y, mask.cpu().numpy(), ridx.cpu().numpy()[: int(nr.item())]


def y_bits(y):
    return y.cpu().numpy().view(np.uint16)


SHAPES = [
    # n, k, m, fill
    (4864, 896, 16, 0.01),     # the single-layer configuration (4864x896, 16 tokens, 1 % dW)
    (40, 64, 5, 0.05),
    (33, 136, 9, 0.1),          # ragged rows and a K that is not a multiple of 64
    (130, 200, 1, 0.02),
    (256, 8, 3, 0.3),           # K = 8: one packed word per row
    (512, 3584, 2, 0.01),       # k/v projection shape
    (1000, 512, 17, 0.04),
    (96, 256, 33, 0.01),
    (300, 1024, 64, 0.01),
    (64, 384, 100, 0.02),
]


@pytest.mark.parametrize("n,k,m,fill", SHAPES)
def test_exact_mode_bit_identical(sc, n, k, m, fill):
    case = make_case(n, k, m, fill, seed=n + k + m)
    op = to_op(sc, case, mode="exact")
    y, mask, ridx = run_gpu(op, case.x_bits)
    yr, rr, _ = case.oracle().forward(case.x_bits)
    assert np.array_equal(mask, rr)
    assert np.array_equal(ridx, np.nonzero(rr)[0])
    assert np.array_equal(y_bits(y), yr), "exact mode must reproduce op.rs bit for bit"


FAST_MODES = ["fast", "fast_tc", "fast_tc8"]  # mma.sync, tcgen05 f16 and fp8 decode engines, one tolerance


@pytest.mark.parametrize("mode", FAST_MODES)
@pytest.mark.parametrize("n,k,m,fill", SHAPES)
def test_fast_mode_within_tolerance(sc, n, k, m, fill, mode):
    case = make_case(n, k, m, fill, seed=n * 3 + k + m)
    op = to_op(sc, case, mode=mode)
    y, mask, ridx = run_gpu(op, case.x_bits)
    yr, rr, acc_ref = case.oracle().forward(case.x_bits)
    assert np.array_equal(mask, rr), "router mask must equal the reference's"
    assert np.array_equal(ridx, np.nonzero(rr)[0])
    assert_fast_close(y_bits(y), yr, f"fast {n}x{k} m={m}")
    acc = op.forward_partial(torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")).cpu().numpy()
    assert_acc_close(acc, acc_ref, f"fast acc {n}x{k} m={m}")


@pytest.mark.parametrize("mode", FAST_MODES)
@pytest.mark.parametrize("n,k,m", [(256, 3584, 1), (256, 3584, 4), (384, 3584, 8)])
def test_fused_decode_dw_blocks_in_global_memory(sc, n, k, m, mode):
    # 25 % dW: with at most 16 column splits a CTA covers >= 224 columns, so its dW block
    # (~3 B per entry, 128 rows) is > 16 KB and is read in place instead of being copied.
    assert 128 * (k // 16) * 0.25 * 3 > 16 * 1024
    case = make_case(n, k, m, 0.25, seed=n + k + 7 * m)
    op = to_op(sc, case, mode=mode)
    y, mask, ridx = run_gpu(op, case.x_bits)
    yr, rr, acc_ref = case.oracle().forward(case.x_bits)
    assert rr.any(), "the case routes at least one token"
    assert np.array_equal(mask, rr)
    assert np.array_equal(ridx, np.nonzero(rr)[0])
    assert_fast_close(y_bits(y), yr, f"fast {n}x{k} m={m} 25% dW")
    grp = sc.SaccadeLinearGroup([op, to_op(sc, make_case(128, k, m, 0.25, seed=5), mode=mode)])
    ys = grp.forward(torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0"))
    torch.cuda.synchronize()
    op.check_device()
    assert_fast_close(y_bits(ys[0]), yr, f"group {n}x{k} m={m} 25% dW")


def test_threshold_token_exactly_on_t4(sc):
    # calibrate() puts t4 exactly on one token's score; the router must reproduce the
    # reference's f32 decision for it (score >= t4 -> routed).
    case = make_case(4864, 896, 16, 0.01, seed=42, boost=[1, 6, 9, 14])
    scores = [O.variance(case.x_bits[t]) for t in range(16)]
    assert case.t4 in scores
    for mode in ("fast", "fast_tc", "exact"):
        op = to_op(sc, case, mode=mode)
        _, mask, _ = run_gpu(op, case.x_bits)
        _, rr, _ = case.oracle().forward(case.x_bits)
        assert np.array_equal(mask, rr)
        assert mask[scores.index(case.t4)] == 1


def test_bf16_input(sc):
    case = make_case(700, 448, 6, 0.02, seed=9)
    xf = case.x_bits.view(np.float16).astype(np.float32)
    xbf = torch.from_numpy(xf).to(torch.bfloat16)
    bf_bits = xbf.view(torch.int16).numpy().view(np.uint16)
    x16 = O.bf16_bits_to_f16_bits(bf_bits)
    for mode in ("exact", "fast", "fast_tc"):
        op = to_op(sc, case, mode=mode)
        y, mask, _ = op.forward(xbf.to("cuda:0"), return_routing=True)[:3]
        yr, rr, _ = case.oracle().forward(x16)
        assert np.array_equal(mask.cpu().numpy(), rr)
        if mode == "exact":
            assert np.array_equal(y_bits(y), yr)
        else:
            assert_fast_close(y_bits(y), yr, "bf16 fast")


@pytest.mark.parametrize("out_dtype", ["f16", "f32", "bf16"])
def test_bias_and_output_dtype(sc, out_dtype):
    case = make_case(200, 320, 4, 0.02, seed=5)
    rng = np.random.default_rng(1)
    b = (rng.standard_normal(200) * 0.01).astype(np.float32)
    op = to_op(sc, case, mode="exact")
    dt = {"f16": torch.float16, "f32": torch.float32, "bf16": torch.bfloat16}[out_dtype]
    x = torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")
    y = op.forward(x, out_dtype=dt, bias=torch.from_numpy(b)).float().cpu().numpy()
    yr, _, _ = case.oracle().forward(case.x_bits)
    ref = torch.from_numpy((yr.view(np.float16).astype(np.float32) + b).astype(np.float32)).to(dt).float().numpy()
    assert np.array_equal(y, ref)


def test_no_delta_and_dense_delta(sc):
    for fill, thr_case in ((None, "none"), (1.0, "dense")):
        case = make_case(96, 128, 5, fill, seed=11)
        if thr_case == "none":
            assert case.c.nnz == 0
        for mode in ("exact", "fast", "fast_tc"):
            op = to_op(sc, case, mode=mode)
            y, mask, _ = run_gpu(op, case.x_bits)
            yr, rr, _ = case.oracle().forward(case.x_bits)
            assert np.array_equal(mask, rr)
            if mode == "exact":
                assert np.array_equal(y_bits(y), yr)
            else:
                assert_fast_close(y_bits(y), yr, f"{thr_case} fast")


def test_forced_routes_and_t8_below_t4(sc):
    base = make_case(160, 192, 8, 0.05, seed=21)
    for t4, t8 in ((3.0e38, 3.0e38), (-1e30, -1e30), (2.0, 0.5), (0.5, 2.0)):
        base.t4, base.t8 = t4, t8
        op = to_op(sc, base, mode="exact")
        y, mask, _ = run_gpu(op, base.x_bits)
        yr, rr, _ = base.oracle().forward(base.x_bits)
        assert np.array_equal(mask, rr), (t4, t8)
        assert np.array_equal(y_bits(y), yr), (t4, t8)


def test_bypass(sc):
    case = make_case(128, 256, 4, 0.05, seed=3)
    try:
        sc.set_bypass_c_tarq(True)
        for mode in ("exact", "fast", "fast_tc"):
            op = to_op(sc, case, mode=mode)
            y, mask, _ = run_gpu(op, case.x_bits)
            yr, _, _ = case.oracle().forward(case.x_bits, bypass=True)
            assert mask.all()
            if mode == "exact":
                assert np.array_equal(y_bits(y), yr), "exact bypass must match op.rs:30-58"
            else:
                assert_fast_close(y_bits(y), yr, "bypass fast")
    finally:
        sc.set_bypass_c_tarq(False)


def test_host_buffers_and_empty_batch(sc):
    case = make_case(64, 64, 3, 0.05, seed=4)
    op = to_op(sc, case, mode="exact", on_device=False)
    y, mask, _ = run_gpu(op, case.x_bits)
    yr, rr, _ = case.oracle().forward(case.x_bits)
    assert np.array_equal(y_bits(y), yr) and np.array_equal(mask, rr)
    y0 = op.forward(torch.empty((0, 64), dtype=torch.float16, device="cuda:0"))
    assert y0.shape == (0, 64)


def test_rejects_bad_inputs(sc):
    case = make_case(32, 64, 2, 0.05, seed=6)
    op = to_op(sc, case)
    with pytest.raises(ValueError):
        op.forward(torch.zeros((2, 63), dtype=torch.float16, device="cuda:0"))
    with pytest.raises(ValueError):
        op.forward(torch.zeros((2, 64), dtype=torch.float32, device="cuda:0"))
    with pytest.raises(ValueError):
        op.forward(torch.zeros((64, 2), dtype=torch.float16, device="cuda:0").t())
    bad = case.c.delta_col_indices.copy()
    if bad.size:
        bad[0] = 64
        with pytest.raises(sc.CTarqError):
            sc.SaccadeLinearOp(torch.from_numpy(case.c.packed_base.view(np.int32)),
                               torch.from_numpy(case.c.scale_base.view(np.float16)),
                               sc.SparseDeltaMatrix(torch.from_numpy(case.c.delta_row_ptrs.view(np.int32)),
                                                    torch.from_numpy(bad.view(np.int32)),
                                                    torch.from_numpy(case.c.delta_values),
                                                    torch.tensor([case.c.delta_scale], dtype=torch.int16).view(
                                                        torch.float16)),
                               sc.SaccadeConfig(0.0, 1.0), 32, 64, device="cuda:0")


@pytest.mark.parametrize("mode", FAST_MODES)
@pytest.mark.parametrize("m", [3, 12])  # router-fused decode (cluster split-K) and router + decode
def test_repeated_calls_reuse_workspace(sc, m, mode):
    case = make_case(3840, 2560, m, 0.02, seed=8)
    op = to_op(sc, case, mode=mode)
    yr, rr, _ = case.oracle().forward(case.x_bits)
    first = None
    for _ in range(3):
        y, mask, _ = run_gpu(op, case.x_bits)
        assert np.array_equal(mask, rr)
        if first is None:
            first = y_bits(y)
        assert np.array_equal(y_bits(y), first), "the fast path is deterministic run to run"


@pytest.mark.parametrize("mode", FAST_MODES)
@pytest.mark.parametrize("n,k,m", [(3584, 3584, 1), (18944, 3584, 4), (3584, 18944, 16), (512, 3584, 1)])
def test_qwen2_7b_shapes(sc, n, k, m, mode):
    case = make_case(n, k, m, 0.01, seed=n + m, boost=[0])
    op = to_op(sc, case, mode=mode)
    y, mask, _ = run_gpu(op, case.x_bits)
    yr, rr, acc_ref = case.oracle().forward(case.x_bits)
    assert np.array_equal(mask, rr)
    assert_fast_close(y_bits(y), yr, f"7B {n}x{k}")
    acc = op.forward_partial(torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")).cpu().numpy()
    assert_acc_close(acc, acc_ref, f"7B acc {n}x{k}")


# ------------------------------------------------------------------ tensor-parallel slices

# ------------------------------------------------------------------ prefill GEMM (9+ tokens)

@pytest.mark.parametrize("n,k,m,nroute,fill", [
    (300, 3584, 300, 300, 0.02),   # every tile routed (dW folded into the weights), column splits
    (300, 3584, 300, 200, 0.02),   # a folded tile, a mixed tile (dW in the epilogue), an unrouted tile
    (4864, 896, 257, 100, 0.01),   # many row tiles, no column split, ragged last tile
    (1000, 520, 40, 40, 0.04),     # one tile, all routed, K not a multiple of 64
    (130, 200, 9, 0, 0.02),        # the smallest GEMM call, nothing routed
    (96, 128, 20, 20, 1.0),        # dense dW: lists too long to fold, dW in the epilogue
    (4864, 896, 1100, 300, 0.01),  # enough tiles for two row tiles per CTA
    (4736, 512, 1100, 400, 0.02),  # two row tiles per CTA, the last CTA holding one
    (300, 3584, 300, 300, 0.15),   # 15 % dW (the compile default): ~5.4 KB lists, the 8 KB-slot variant
    (300, 3584, 300, 200, 0.15),   # the same with a mixed and an unrouted tile
])
def test_prefill_gemm_routing(sc, n, k, m, nroute, fill):
    rng = np.random.default_rng(n + m + nroute)
    boost = sorted(rng.choice(m, size=nroute, replace=False).tolist()) if nroute else []
    case = make_case(n, k, m, fill, seed=n + k + m, boost=boost, thresholds=(8.0, 3e38))
    yr, rr, acc_ref = case.oracle().forward(case.x_bits)
    assert int(rr.sum()) == nroute
    for mode in FAST_MODES:
        op = to_op(sc, case, mode=mode)
        y, mask, ridx = run_gpu(op, case.x_bits)
        assert np.array_equal(mask, rr)
        assert np.array_equal(ridx, np.nonzero(rr)[0])
        assert_fast_close(y_bits(y), yr, f"gemm {n}x{k} m={m} routed={nroute} {mode}")
        acc = op.forward_partial(torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")).cpu().numpy()
        assert_acc_close(acc, acc_ref, f"gemm {n}x{k} m={m} routed={nroute} {mode} acc")


@pytest.mark.parametrize("count", [2, 3])
def test_column_shards_concatenate(sc, count):
    case = make_case(520, 256, 6, 0.02, seed=31)
    yr, rr, _ = case.oracle().forward(case.x_bits)
    x = torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")
    parts = []
    for i in range(count):
        op = to_op(sc, case, mode="exact", shard=("columns", i, count))
        parts.append(y_bits(op.forward(x)))
    assert np.array_equal(np.concatenate(parts, axis=1), yr)


@pytest.mark.parametrize("mode", FAST_MODES)
@pytest.mark.parametrize("count", [2, 4])
def test_row_shards_sum_to_full(sc, count, mode):
    case = make_case(300, 1024, 5, 0.02, seed=41)
    _, rr, acc_ref = case.oracle().forward(case.x_bits)
    x = torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")
    total = None
    for i in range(count):
        op = to_op(sc, case, mode=mode, shard=("rows", i, count))
        part, mask = op.forward_partial(x, return_routing=True)
        assert np.array_equal(mask.cpu().numpy(), rr), "every shard routes on the whole token"
        total = part if total is None else total + part
    assert_acc_close(total.cpu().numpy(), acc_ref, "rows shards")
    y = sc.finalize(total)
    yr, _, _ = case.oracle().forward(case.x_bits)
    assert_fast_close(y_bits(y), yr, "rows shards f16")


@pytest.mark.parametrize("t4", [0.5, 2.0])   # the N(0, 1) token (variance ~1) routed / not routed
@pytest.mark.parametrize("count", [1, 3])
def test_row_shards_one_token(sc, count, t4):
    # one token: the integer engine stages the whole token with one bulk copy and routes on its
    # own sums; a rows shard's slice starts inside the token and the last one ends in a padded
    # block (K = 1000 is not a multiple of 64)
    case = make_case(300, 1000, 1, 0.05, seed=43, boost=[], thresholds=(t4, 3e38))
    yr, rr, acc_ref = case.oracle().forward(case.x_bits)
    assert rr[0] == (t4 < 1.0)
    x = torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")
    total = None
    for i in range(count):
        op = to_op(sc, case, mode="fast", shard=("rows", i, count) if count > 1 else None)
        part, mask = op.forward_partial(x, return_routing=True)
        op.check_device()
        assert np.array_equal(mask.cpu().numpy(), rr)
        total = part if total is None else total + part
    assert_acc_close(total.cpu().numpy(), acc_ref, "rows shards, one token")
    assert_fast_close(y_bits(sc.finalize(total)), yr, "rows shards, one token, f16")


# ------------------------------------------------------------------ format producer on the GPU

@pytest.mark.parametrize("n,k,fill", [(4864, 896, 0.01), (77, 200, 0.15), (256, 64, 1.0), (33, 8, 0.5)])
def test_gpu_packer_bit_identical(sc, n, k, fill):
    rng = np.random.default_rng(n + k)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[min(2, n - 1)] = 0.0
    wt = torch.from_numpy(w).to("cuda:0")
    thr = sc.compute_percentile_threshold(wt, fill)
    assert np.float32(thr) == np.float32(O.percentile_threshold(w, fill))
    blocks = sc.compress_tensor_to_saccade(wt, thr)
    ref = O.compress(w, thr)
    assert np.array_equal(blocks["packed_base"].view(torch.int32).cpu().numpy().view(np.uint32), ref.packed_base)
    assert np.array_equal(blocks["scale_base"].cpu().numpy().view(np.uint16), ref.scale_base)
    if ref.nnz:
        assert np.array_equal(blocks["delta_row_ptrs"].view(torch.int32).cpu().numpy().view(np.uint32),
                              ref.delta_row_ptrs)
        assert np.array_equal(blocks["delta_col_indices"].view(torch.int32).cpu().numpy().view(np.uint32),
                              ref.delta_col_indices)
        assert np.array_equal(blocks["delta_values"].cpu().numpy(), ref.delta_values)
        assert int(blocks["delta_scale"].view(torch.int16).item()) & 0xFFFF == ref.delta_scale
    else:
        assert "delta_row_ptrs" not in blocks


def test_gpu_calibrate_and_variance(sc):
    rng = np.random.default_rng(12)
    acts = rng.standard_normal((300, 512)).astype(np.float32)
    acts[::7] *= 8
    a16 = acts.astype(np.float16)
    for p4, p8 in ((0.75, 0.95), (0.0, 1.0), (0.5, 0.333)):
        assert sc.ProfileRunner.calibrate(torch.from_numpy(acts), p4, p8) == O.calibrate(acts, p4, p8)
        assert sc.ProfileRunner.calibrate(torch.from_numpy(a16), p4, p8) == O.calibrate(
            a16.astype(np.float32), p4, p8)
    v = sc.variance_heuristic(torch.from_numpy(a16).to("cuda:0")).cpu().numpy()
    ref = np.array([O.variance(a16[t].view(np.uint16)) for t in range(300)], dtype=np.float32)
    assert np.array_equal(v.view(np.uint32), ref.view(np.uint32))


def test_end_to_end_from_dense_weights(sc):
    # W on the GPU -> GPU packer -> layer -> forward, against the oracle run on the same W
    case = make_case(1024, 896, 16, 0.01, seed=77)
    wt = torch.from_numpy(case.w).to("cuda:0")
    thr = sc.compute_percentile_threshold(wt, 0.01)
    blocks = sc.compress_tensor_to_saccade(wt, thr)
    op = sc.saccade_op_from_compressed(blocks, sc.SaccadeConfig(case.t4, case.t8), 1024, 896, mode="exact")
    y, mask, _ = run_gpu(op, case.x_bits)
    yr, rr, _ = case.oracle().forward(case.x_bits)
    assert np.array_equal(mask, rr) and np.array_equal(y_bits(y), yr)


# ------------------------------------------------------------------ groups (one launch, shared x)

@pytest.mark.parametrize("mode", FAST_MODES + ["exact"])
@pytest.mark.parametrize("shapes,m", [
    ([(3584, 3584), (512, 3584), (512, 3584)], 1),   # q, k, v
    ([(1024, 1024), (1024, 1024)], 4),               # gate/up-like pair
    ([(256, 512), (128, 512), (384, 512), (130, 512)], 3),
    ([(640, 768), (256, 768)], 20),                  # more than 8 tokens: one launch per layer
])
def test_group_matches_individual_calls(sc, shapes, m, mode):
    k = shapes[0][1]
    cases = [make_case(n, k, m, 0.02, seed=1000 + i, boost=[0]) for i, (n, _) in enumerate(shapes)]
    x_bits = cases[0].x_bits
    ops = [to_op(sc, c, mode=mode) for c in cases]
    grp = sc.SaccadeLinearGroup(ops)
    x = torch.from_numpy(x_bits.view(np.float16)).to("cuda:0")
    ys, routing = grp.forward(x, return_routing=True)
    torch.cuda.synchronize()
    for op, c, y, (mask, ridx, nr) in zip(ops, cases, ys, routing):
        yi, mi, ri, ni = op.forward(x, return_routing=True)
        torch.cuda.synchronize()
        op.check_device()
        if mode == "exact":
            assert np.array_equal(y_bits(y), y_bits(yi)), "exact mode: a group reproduces the layer's own call"
        else:  # the group may split the columns differently: f32 split-K sums in another order
            assert_fast_close(y_bits(y), y_bits(yi), f"group vs single {c.n}x{c.k} {mode}")
        assert np.array_equal(mask.cpu().numpy(), mi.cpu().numpy())
        assert int(nr.item()) == int(ni.item())
        assert np.array_equal(ridx.cpu().numpy()[: int(nr.item())], ri.cpu().numpy()[: int(ni.item())])
        yr, rr, _ = c.oracle().forward(x_bits)
        assert np.array_equal(mask.cpu().numpy(), rr)
        if mode == "exact":
            assert np.array_equal(y_bits(y), yr)
        else:
            assert_fast_close(y_bits(y), yr, f"group {c.n}x{c.k} {mode}")


@pytest.mark.parametrize("kind", ["wide", "zeros", "tiny", "one_hot"])
def test_one_token_extreme_inputs(sc, kind):
    # one-token decode: fast_tc runs the fp8 engine (x split into e4m3 columns); every engine
    # must stay within the tolerance on inputs spanning the f16 range
    n, k = 1024, 2048
    case = make_case(n, k, 1, 0.02, seed=55, boost=[0])
    rng = np.random.default_rng(5)
    if kind == "wide":
        x = (rng.standard_normal(k) * 10.0 ** rng.uniform(-7, 4, k)).astype(np.float32)
    elif kind == "zeros":
        x = np.zeros(k, dtype=np.float32)
    elif kind == "tiny":
        x = (rng.standard_normal(k) * 1e-6).astype(np.float32)
    else:
        x = np.zeros(k, dtype=np.float32)
        x[777] = 3.0e4
        x[5] = 1e-3
    case.x_bits = x.astype(np.float16).view(np.uint16).reshape(1, k)
    yr, rr, acc_ref = case.oracle().forward(case.x_bits)
    for mode in FAST_MODES:
        op = to_op(sc, case, mode=mode)
        y, mask, _ = run_gpu(op, case.x_bits)
        assert np.array_equal(mask, rr)
        assert_fast_close(y_bits(y), yr, f"{kind} {mode}")
        acc = op.forward_partial(torch.from_numpy(case.x_bits.view(np.float16)).to("cuda:0")).cpu().numpy()
        assert_acc_close(acc, acc_ref, f"{kind} {mode} acc")


@pytest.mark.parametrize("kind", ["inf", "neg_inf", "nan"])
def test_one_token_non_finite_inputs(sc, kind):
    # one-token decode: the integer engine of "fast" cannot represent inf/nan and runs the f16 loop
    # for the column split holding one, so every row keeps the reference's nan / +inf / -inf
    # (inf times a zero weight is nan, otherwise the weight's sign); the fp8 engine of "fast_tc8"
    # documents nan rows instead
    n, k = 512, 3584
    case = make_case(n, k, 1, 0.01, seed=77, boost=[0])
    x = np.random.default_rng(9).standard_normal(k).astype(np.float32)
    x[1234] = {"inf": np.inf, "neg_inf": -np.inf, "nan": np.nan}[kind]
    case.x_bits = x.astype(np.float16).view(np.uint16).reshape(1, k)
    yr, rr, _ = case.oracle().forward(case.x_bits)
    r = yr.view(np.float16).astype(np.float32)
    assert not np.isfinite(r).any()
    for mode in FAST_MODES:
        op = to_op(sc, case, mode=mode)
        y, mask, _ = run_gpu(op, case.x_bits)
        assert np.array_equal(mask, rr)
        got = y_bits(y).view(np.float16).astype(np.float32)
        if mode == "fast_tc8":
            assert not np.isfinite(got).any(), mode
            continue
        assert np.array_equal(np.isnan(got), np.isnan(r)), mode
        assert np.array_equal(np.isposinf(got), np.isposinf(r)), mode
        assert np.array_equal(np.isneginf(got), np.isneginf(r)), mode
