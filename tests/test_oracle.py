"""CPU tests of the C oracle: hand-worked known answers and agreement with the
independent numpy restatement (tests/np_restatement.py).  The Rust reference
ships no golden vectors and cannot be built here, so these cases are what the
oracle is checked against (parity unpinned)."""
import numpy as np
import pytest

from oracle import oracle as O
import np_restatement as R


# ------------------------------------------------------------------ f16

def test_f16_roundtrip_all_patterns():
    lib = O.lib()
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    f = bits.view(np.float16).astype(np.float32)
    ok = ~np.isnan(f)
    back = O.f32_to_f16_bits(f)
    assert np.array_equal(back[ok], bits[ok])
    for b in (0x0001, 0x03FF, 0x0400, 0x3C00, 0x7BFF, 0x8001, 0xFBFF):
        assert lib.oracle_f16_to_f32(b) == np.uint16(b).view(np.float16).astype(np.float32)


def test_f32_to_f16_rne_matches_numpy():
    rng = np.random.default_rng(1)
    vals = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 200000),
        np.array([65504.0, 65519.99, 65520.0, 1e9, -1e9, 2.0 ** -25, 2.0 ** -25 * 1.0000001,
                  2.0 ** -24 * 1.5, 2.0 ** -24 * 2.5, 0.0, -0.0, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11],
                 dtype=np.float32),
    ]).astype(np.float32)
    assert np.array_equal(O.f32_to_f16_bits(vals), vals.astype(np.float16).view(np.uint16))


def test_bf16_to_f16():
    rng = np.random.default_rng(2)
    f = rng.standard_normal(10000).astype(np.float32)
    bf = (f.view(np.uint32) >> 16).astype(np.uint16)
    f_bf = (bf.astype(np.uint32) << 16).view(np.float32)
    assert np.array_equal(O.bf16_bits_to_f16_bits(bf), f_bf.astype(np.float16).view(np.uint16))


# ------------------------------------------------------------------ hand-worked known answers

def test_kat_pack_one_word():
    # Row of 8 exactly-representable weights; scale = (7/16)/7 = 1/16 exactly.
    w = (np.array([[7, -7, 3.5, -3.5, 0, 1, 0.5, -0.5]], dtype=np.float32) / 16).astype(np.float32)
    c = O.compress(w, 0.01)
    # q = round-half-away(w*16) = [7,-7,4,-4,0,1,1,-1]; nibble = q+8 = [15,1,12,4,8,9,9,7]
    assert c.packed_base[0, 0] == 0x79984C1F
    assert c.scale_base[0] == 0x2C00  # f16(1/16)
    # errors: cols 2,6 -> -1/32; cols 3,7 -> +1/32
    assert list(c.delta_row_ptrs) == [0, 4]
    assert list(c.delta_col_indices) == [2, 3, 6, 7]
    ds = np.float32(np.float32(1 / 32) / np.float32(127))
    q = [int(R.round_half_away(np.float32(np.float32(e) / ds))) for e in (-1 / 32, 1 / 32, -1 / 32, 1 / 32)]
    assert list(c.delta_values.view(np.int8)) == q
    assert c.delta_scale == int(np.float32(ds).astype(np.float16).view(np.uint16))
    assert abs(q[0]) == 127
    assert O.percentile_threshold(w, 0.5) == np.float32(1 / 32)


def test_kat_forward_one_word():
    w = (np.array([[7, -7, 3.5, -3.5, 0, 1, 0.5, -0.5]], dtype=np.float32) / 16).astype(np.float32)
    c = O.compress(w, 0.01)
    op = O.OracleLinear(c, t4=-1e30, t8=-1e30)
    x = np.ones((1, 8), dtype=np.float16).view(np.uint16)
    y, routed, acc = op.forward(x)
    # Phase 1: a0=7+0, a1=-7+1, a2=4+1, a3=-4-1 -> 1 * 1/16
    base = np.float32(1.0 / 16)
    dval = np.float32(np.float32(127) * np.float32(np.uint16(c.delta_scale).view(np.float16)))
    expect = base
    for sgn in (-1, 1, -1, 1):  # CSC column order 2,3,6,7
        expect = np.float32(expect + np.float32(np.float32(1.0) * np.float32(sgn * dval)))
    assert routed[0] == 1
    assert acc[0, 0] == expect
    assert y[0, 0] == np.float32(expect).astype(np.float16).view(np.uint16)
    # route OFF: base only
    y0, r0, acc0 = O.OracleLinear(c, t4=3.0e38, t8=3.0e38).forward(x)
    assert r0[0] == 0 and acc0[0, 0] == base


def test_kat_variance_and_calibrate():
    x = np.array([1, -1, 1, -1, 3, -3, 0, 0], dtype=np.float16).view(np.uint16)
    # sum = 0, sum_sq = 1+1+1+1+9+9 = 22 -> 22/8 - 0 = 2.75
    assert O.variance(x) == np.float32(2.75)
    acts = np.array([[0, 0], [1, -1], [2, -2], [3, -3]], dtype=np.float32)  # variances 0,1,4,9
    # idx = min(round(4*0.75)=3, 3) -> 9 ; round(4*0.3)=1 -> 1
    assert O.calibrate(acts, 0.75, 0.3) == (9.0, 1.0)
    assert O.calibrate(acts, 0.5, 2.0) == (4.0, 9.0)  # round(2.0)=2 ; 8 clamps to 3


def test_route_bits_truth_table():
    # routed = (s >= t4 && s < t8) || s >= t8, including t8 < t4 and NaN
    assert O.route_bits(1.0, 0.5, 2.0) == 1
    assert O.route_bits(3.0, 0.5, 2.0) == 2
    assert O.route_bits(0.1, 0.5, 2.0) == 0
    assert O.route_bits(1.0, 2.0, 0.5) == 2   # t8 < t4: s >= t8 still routes
    assert O.route_bits(float("nan"), 0.5, 2.0) == 0
    assert O.route_bits(1.0, 0.5, float("nan")) == 0


# ------------------------------------------------------------------ C oracle == numpy restatement

def _weights(rng, n, k, zero_row=True):
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if zero_row and n > 2:
        w[1] = 0.0
    return w


@pytest.mark.parametrize("n,k,fill", [(7, 8, 0.3), (33, 64, 0.01), (64, 136, 0.15), (20, 96, 1.0), (5, 16, 0.0)])
def test_compress_matches_numpy(n, k, fill):
    rng = np.random.default_rng(n * 1000 + k)
    w = _weights(rng, n, k)
    thr_c = O.percentile_threshold(w, fill)
    thr_n = R.percentile_threshold(w, fill)
    assert np.float32(thr_c) == np.float32(thr_n)
    c = O.compress(w, thr_c)
    d = R.compress(w, thr_c)
    assert np.array_equal(c.packed_base, d["packed_base"])
    assert np.array_equal(c.scale_base, d["scale_base"])
    assert np.array_equal(c.delta_row_ptrs, d["delta_row_ptrs"])
    assert np.array_equal(c.delta_col_indices, d["delta_col_indices"])
    assert np.array_equal(c.delta_values, d["delta_values"])
    if c.nnz:
        assert c.delta_scale == d["delta_scale"]


def test_compress_threshold_extremes():
    rng = np.random.default_rng(5)
    w = _weights(rng, 9, 32)
    c = O.compress(w, 1e9)      # nothing kept
    assert c.nnz == 0 and c.delta_row_ptrs[-1] == 0
    c = O.compress(w, -1.0)     # every nonzero error kept
    d = R.compress(w, -1.0)
    assert np.array_equal(c.delta_col_indices, d["delta_col_indices"])
    assert np.array_equal(c.delta_values, d["delta_values"])
    with pytest.raises(ValueError):
        O.compress(np.zeros((2, 12), np.float32), 0.1)


def test_calibrate_matches_numpy():
    rng = np.random.default_rng(7)
    acts = rng.standard_normal((37, 64)).astype(np.float32)
    acts[5] *= 8
    for p4, p8 in ((0.75, 0.95), (0.0, 1.0), (0.5, 0.2)):
        assert O.calibrate(acts, p4, p8) == R.calibrate(acts, p4, p8)


@pytest.mark.parametrize("n,k,m,fill", [(16, 64, 5, 0.05), (40, 128, 16, 0.01), (24, 8, 3, 0.5), (48, 200, 4, 0.1)])
def test_forward_matches_numpy(n, k, m, fill):
    rng = np.random.default_rng(n + k + m)
    w = _weights(rng, n, k)
    thr = O.percentile_threshold(w, fill)
    c = O.compress(w, thr)
    x32 = rng.standard_normal((m, k)).astype(np.float32)
    x32[::3] *= 8
    xb = x32.astype(np.float16).view(np.uint16)
    t4, t8 = O.calibrate(xb.view(np.float16).astype(np.float32), 0.6, 0.95)
    op = O.OracleLinear(c, t4, t8)
    y, routed, acc = op.forward(xb)
    d = {"packed_base": c.packed_base, "scale_base": c.scale_base, "delta_row_ptrs": c.delta_row_ptrs,
         "delta_col_indices": c.delta_col_indices, "delta_values": c.delta_values, "delta_scale": c.delta_scale}
    y2, r2, acc2 = R.forward(d, n, k, t4, t8, xb)
    assert np.array_equal(routed, r2)
    assert routed.any() and not routed.all()
    assert np.array_equal(acc.view(np.uint32), acc2.view(np.uint32))
    assert np.array_equal(y, y2)


def test_build_csc_preserves_entries():
    rng = np.random.default_rng(11)
    w = _weights(rng, 30, 48)
    c = O.compress(w, O.percentile_threshold(w, 0.2))
    op = O.OracleLinear(c, 0.0, 0.0)
    ds = np.float32(np.uint16(c.delta_scale).view(np.float16))
    rows = np.repeat(np.arange(30), np.diff(c.delta_row_ptrs.astype(np.int64)))
    csr = sorted(zip(rows.tolist(), c.delta_col_indices.tolist(),
                     (c.delta_values.view(np.int8).astype(np.float32) * ds).tolist()))
    cols = np.repeat(np.arange(48), np.diff(op.col_ptrs.astype(np.int64)))
    csc = sorted(zip(op.csc_rows.tolist(), cols.tolist(), op.csc_vals.tolist()))
    assert csr == csc


def test_bypass_agrees_with_route_always():
    rng = np.random.default_rng(13)
    w = _weights(rng, 32, 96)
    c = O.compress(w, O.percentile_threshold(w, 0.05))
    op = O.OracleLinear(c, -1e30, -1e30)
    xb = rng.standard_normal((4, 96)).astype(np.float16).view(np.uint16)
    _, r, acc_route = op.forward(xb)
    _, _, acc_bypass = op.forward(xb, bypass=True)
    assert r.all()
    # same math (base + dW), different summation order: f32 rounding only
    np.testing.assert_allclose(acc_bypass, acc_route, rtol=0, atol=1e-5 * np.abs(acc_route).max())


def test_empty_token_batch():
    rng = np.random.default_rng(3)
    c = O.compress(_weights(rng, 8, 16), 0.001)
    y, r, _ = O.OracleLinear(c, 0.0, 1.0).forward(np.zeros((0, 16), np.uint16))
    assert y.shape == (0, 8) and r.size == 0
