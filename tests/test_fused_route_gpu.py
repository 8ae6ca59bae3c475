"""The routers fused into the kernels that write the linears' inputs: sc_qwen2_add_rmsnorm_route
(the input of q,k,v and of gate,up) and sc_qwen2_silu_mul_route (the input of down), consumed by
sc_forward_group_routed.  Against the unfused path on the same inputs (sc_qwen2_add_rmsnorm or
sc_qwen2_silu_mul, then sc_forward_group routing on its own): the same residual, f16 rows, masks,
routed lists, counts and outputs, bit for bit; and the masks equal the oracle's sequential f32
scores (heuristics.rs:3-14) against the thresholds (op.rs:69-72), with thresholds set on tokens'
exact scores and one f32 ulp beside them (decisions only the exact replay can take).

Token counts 9, 16 (the 9..16-token launch), 33 and 64 (17..64, dW folded); rows of 896 and 3584
(norm) and 4864 and 18944 (silu); the first layer's norm without a residual delta; bypass; the
argument checks; and a small Qwen2 model decoding 16 and 40 sequences with no fused router, with
the RMSNorm ones and with all of them: the same greedy tokens and logits bits.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O

pytestmark = pytest.mark.gpu

EPS = 1e-6


@pytest.fixture(scope="module")
def sc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import saccade_core
    saccade_core.set_bypass_c_tarq(False)
    return saccade_core


_GROUPS = {}


def group(sc, k, ns, fill=0.01):
    """A group of layers [n, k] for n in ns (seeded weights, the GPU packer)."""
    key = (k, tuple(ns), fill)
    if key not in _GROUPS:
        ops = []
        for i, n in enumerate(ns):
            g = torch.Generator(device="cuda").manual_seed(k * 7 + n + i)
            w = torch.randn(n, k, device="cuda", generator=g) * 0.02
            blocks = sc.compress_tensor_to_saccade(w, sc.compute_percentile_threshold(w, fill))
            ops.append(sc.saccade_op_from_compressed(blocks, sc.SaccadeConfig(1.0, 3e38), n, k, mode="fast"))
        _GROUPS[key] = (ops, sc.SaccadeLinearGroup(ops))
    return _GROUPS[key]


def oracle_scores(x16):
    xb = x16.cpu().numpy().view(np.uint16)
    return np.array([O.variance(r) for r in xb], dtype=np.float32)


def rule(s, t4, t8):
    """op.rs:69-72: routed when t4 <= s < t8 or s >= t8."""
    return (((s >= t4) & (s < t8)) | (s >= t8)).astype(np.uint8)


def set_thresholds(ops, s):
    """Thresholds on the tokens' exact scores and one f32 ulp beside them (t8 above every score for
    the first two layers, inside the scores for the third)."""
    m = len(s)
    picks = [(s[m // 2], np.float32(3e38)),
             (np.nextafter(s[m // 3], np.float32(np.inf)), np.float32(3e38)),
             (np.nextafter(s[m // 4], np.float32(0)), s[(3 * m) // 4])]
    out = []
    for op, (t4, t8) in zip(ops, picks):
        op.set_thresholds(float(t4), float(t8))
        out.append((np.float32(t4), np.float32(t8)))
    return out


def f16_rows(k, m, seed):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()


def check_same(sc, grp, ops, x_a, ys_a, rout_a, x_b, ys_b, R, thr, s):
    assert torch.equal(x_a.view(torch.int16), x_b.view(torch.int16)), "fused kernel writes the same f16 rows"
    for i, op in enumerate(ops):
        mask_a, ridx_a, nr_a = rout_a[i]
        mask_b, ridx_b, nr_b = R.layer(i)
        assert torch.equal(mask_a, mask_b), f"layer {i} mask"
        assert int(nr_a.item()) == nr_b, f"layer {i} count"
        assert torch.equal(ridx_a[:nr_b], ridx_b), f"layer {i} routed list"
        want = rule(s, *thr[i])
        assert np.array_equal(mask_b.cpu().numpy(), want), (i, np.nonzero(mask_b.cpu().numpy() != want)[0][:8])
        assert torch.equal(ys_a[i].view(torch.int16) if ys_a[i].dtype == torch.float16 else ys_a[i],
                           ys_b[i].view(torch.int16) if ys_b[i].dtype == torch.float16 else ys_b[i]), f"layer {i} y"
    assert int(R.counter[0].item()) == 0, "the router leaves its counter at zero"
    for op in ops:
        op.check_device()


@pytest.mark.parametrize("k", [896, 3584])
@pytest.mark.parametrize("m", [9, 16, 33, 64])
@pytest.mark.parametrize("with_delta", [True, False])
def test_norm_route_matches_unfused(sc, k, m, with_delta):
    from saccade_core._lib import LIB, SC_F16, check
    ops, grp = group(sc, k, (256, 128, 128))
    assert grp.takes_routing(m)
    resid0 = f16_rows(k, m, seed=k + m) * 3.0
    delta = f16_rows(k, m, seed=k + m + 1) if with_delta else None
    w = (1.0 + 0.1 * f16_rows(k, 1, seed=k)).reshape(-1).contiguous()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    dptr = delta.data_ptr() if delta is not None else None
    # the plain kernel first: the thresholds go on the rows it writes
    resid_a = resid0.clone()
    x_a = torch.empty(m, k, dtype=torch.float16, device="cuda")
    check(LIB.sc_qwen2_add_rmsnorm(resid_a.data_ptr(), dptr, w.data_ptr(), m, k, ctypes.c_float(EPS), x_a.data_ptr(),
                                   SC_F16, st))
    s = oracle_scores(x_a)
    thr = set_thresholds(ops, s)
    ys_a, rout_a = grp.forward(x_a, out_dtype=torch.float32, return_routing=True)
    # fused
    resid_b = resid0.clone()
    x_b = torch.empty(m, k, dtype=torch.float16, device="cuda")
    R = sc.GroupRouting(3, m, "cuda")
    check(LIB.sc_qwen2_add_rmsnorm_route(resid_b.data_ptr(), dptr, w.data_ptr(), m, k, ctypes.c_float(EPS),
                                         x_b.data_ptr(), grp._h, R.mask_p, R.ridx_p, R.count_p,
                                         R.counter.data_ptr(), st))
    ys_b = grp.forward_routed(x_b, R, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(resid_a, resid_b), "same residual"
    check_same(sc, grp, ops, x_a, ys_a, rout_a, x_b, ys_b, R, thr, s)


@pytest.mark.parametrize("width", [4864, 18944])
@pytest.mark.parametrize("m", [9, 16, 64])
def test_silu_route_matches_unfused(sc, width, m):
    from saccade_core._lib import LIB, check
    ops, grp = group(sc, width, (256,))
    assert grp.takes_routing(m)
    g = (f16_rows(width, m, seed=width + m) * 2.0).to(torch.float16)
    u = f16_rows(width, m, seed=width + m + 1).to(torch.float16)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    h_a = torch.empty(m, width, dtype=torch.float16, device="cuda")
    check(LIB.sc_qwen2_silu_mul(g.data_ptr(), u.data_ptr(), m * width, h_a.data_ptr(), st))
    s = oracle_scores(h_a)
    thr = set_thresholds(ops, s)
    ys_a, rout_a = grp.forward(h_a, return_routing=True)
    h_b = torch.empty_like(h_a)
    R = sc.GroupRouting(1, m, "cuda")
    check(LIB.sc_qwen2_silu_mul_route(g.data_ptr(), u.data_ptr(), m, width, h_b.data_ptr(), grp._h, R.mask_p,
                                      R.ridx_p, R.count_p, R.counter.data_ptr(), st))
    ys_b = grp.forward_routed(h_b, R)
    torch.cuda.synchronize()
    check_same(sc, grp, ops, h_a, ys_a, rout_a, h_b, ys_b, R, thr, s)
    # the element-wise kernel against the oracle's silu (model.rs:295-299)
    from oracle import qwen2_oracle as QO
    gf = g.float().cpu().numpy()
    ref = (QO.silu(gf) * u.float().cpu().numpy()).astype(np.float16)
    assert np.array_equal(h_b.cpu().numpy().view(np.uint16), ref.view(np.uint16))


def test_bypass_routes_every_token(sc):
    from saccade_core._lib import LIB, SC_F16, check
    k, m = 896, 24
    ops, grp = group(sc, k, (256, 128, 128))
    resid = f16_rows(k, m, seed=5)
    w = torch.ones(k, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    x_a = torch.empty(m, k, dtype=torch.float16, device="cuda")
    check(LIB.sc_qwen2_add_rmsnorm(resid.clone().data_ptr(), None, w.data_ptr(), m, k, ctypes.c_float(EPS),
                                   x_a.data_ptr(), SC_F16, st))
    for op in ops:
        op.set_thresholds(3e38, 3e38)  # nothing routes unless bypassed
    sc.set_bypass_c_tarq(True)
    try:
        ys_a, rout_a = grp.forward(x_a, return_routing=True)
        R = sc.GroupRouting(3, m, "cuda")
        x_b = torch.empty_like(x_a)
        check(LIB.sc_qwen2_add_rmsnorm_route(resid.clone().data_ptr(), None, w.data_ptr(), m, k, ctypes.c_float(EPS),
                                             x_b.data_ptr(), grp._h, R.mask_p, R.ridx_p, R.count_p,
                                             R.counter.data_ptr(), st))
        ys_b = grp.forward_routed(x_b, R)
        torch.cuda.synchronize()
    finally:
        sc.set_bypass_c_tarq(False)
    for i in range(3):
        mask, ridx, c = R.layer(i)
        assert c == m and mask.cpu().numpy().tolist() == [1] * m
        assert ridx.cpu().numpy().tolist() == list(range(m))
        assert torch.equal(ys_a[i].view(torch.int16), ys_b[i].view(torch.int16))


def test_argument_checks(sc):
    from saccade_core._lib import LIB, SC_OK
    k, m = 896, 16
    ops, grp = group(sc, k, (256, 128, 128))
    R = sc.GroupRouting(3, m, "cuda")
    resid = torch.zeros(m, 1024, device="cuda")
    w = torch.ones(1024, device="cuda")
    x = torch.empty(m, 1024, dtype=torch.float16, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # rows of another length than the group's layers read
    assert LIB.sc_qwen2_add_rmsnorm_route(resid.data_ptr(), None, w.data_ptr(), m, 1024, ctypes.c_float(EPS),
                                          x.data_ptr(), grp._h, R.mask_p, R.ridx_p, R.count_p, R.counter.data_ptr(),
                                          st) != SC_OK
    # no counter
    assert LIB.sc_qwen2_add_rmsnorm_route(resid.data_ptr(), None, w.data_ptr(), m, k, ctypes.c_float(EPS),
                                          x.data_ptr(), grp._h, R.mask_p, R.ridx_p, R.count_p, None, st) != SC_OK
    # silu rows not a multiple of 8
    assert LIB.sc_qwen2_silu_mul_route(x.data_ptr(), x.data_ptr(), m, 1020, x.data_ptr(), grp._h, R.mask_p,
                                       R.ridx_p, R.count_p, R.counter.data_ptr(), st) != SC_OK
    # outside the 9..64-token launch the group takes no routing
    assert not grp.takes_routing(4) and not grp.takes_routing(65)
    with pytest.raises(sc.CTarqError):
        grp.forward_routed(torch.zeros(4, k, dtype=torch.float16, device="cuda"), sc.GroupRouting(3, 4, "cuda"))
    torch.cuda.synchronize()


@pytest.mark.parametrize("batch", [16, 40])
def test_model_decode_same_with_fused_routers(sc, batch):
    from saccade_core import qwen2 as q2
    cfg = q2.Qwen2Config(hidden=256, intermediate=704, layers=3, heads=4, kv_heads=2, head_dim=64, vocab=4096)
    ck = q2.random_checkpoint(cfg, seed=3, fill=0.01)
    rng = np.random.default_rng(3)
    S, steps = 12, 6
    q2.calibrate(ck, torch.from_numpy(rng.integers(0, cfg.vocab, (batch, S))).cuda(), max_pos=S + steps + 2)
    prompt = torch.from_numpy(rng.integers(0, cfg.vocab, (batch, S))).cuda()
    runs = []
    for fused in ("none", "norm", "all"):
        model = q2.Qwen2Model(ck, max_batch=batch, max_pos=S + steps + 2, fused_route=fused)
        dec = q2.GreedyDecoder(model, batch)
        toks, gaps = dec.generate(prompt, steps, record_logits=True)
        torch.cuda.synchronize()
        model.check_device()
        used = sorted(k[1] for k, v in model._bufs.items() if k[0] == "route" and v is not None)
        assert used == {"none": [], "norm": ["gateup", "qkv"], "all": ["down", "gateup", "qkv"]}[fused]
        runs.append((toks.cpu().numpy(), dec.logits.cpu().numpy(), dec.launches_per_step))
        del dec, model
    (t0, l0, n0) = runs[0]
    for t1, l1, n1 in runs[1:]:
        assert np.array_equal(t0, t1)
        assert np.array_equal(l0.view(np.uint32), l1.view(np.uint32)), "same logits bits"
        assert n1 < n0, "fewer launches per decode step with the routers fused"
    assert runs[2][2] < runs[1][2]
