"""Router masks when every token's score sits inside the f32 error band (the CTA-parallel exact
replay of heuristics.rs's sequential chains), against the oracle's sequential f32 scores.

Rows are RMS-normalised (the inputs of q/k/v and gate/up in a decoder: every variance is within
~1e-3 of 1, far inside the band of K = 18944), and the threshold is set at a token's exact score,
one f32 ulp on either side of it, and 1e-6 / 1e-5 relative away, so most decisions can only be
taken on the exact chain.  Token counts 12 (the 9..16-token router) and 64 (the prefill router);
K 896, 3584, 18944; f16 and bf16 inputs; rows with zeros, huge and tiny values, inf and nan.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import saccade_core
    saccade_core.set_bypass_c_tarq(False)
    return saccade_core


_LAYERS = {}


def layer(sc, k):
    if k not in _LAYERS:
        g = torch.Generator(device="cuda").manual_seed(k)
        w = torch.randn(128, k, device="cuda", generator=g) * 0.02
        blocks = sc.compress_tensor_to_saccade(w, sc.compute_percentile_threshold(w, 0.01))
        _LAYERS[k] = sc.saccade_op_from_compressed(blocks, sc.SaccadeConfig(1.0, 3e38), 128, k, mode="fast")
    return _LAYERS[k]


def rows(k, m, seed, kind):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k))
    if kind == "normed":
        x /= np.sqrt(np.mean(x * x, axis=1, keepdims=True))
    elif kind == "mixed":
        x /= np.sqrt(np.mean(x * x, axis=1, keepdims=True))
        x[0, :] = 0.0                                   # all zeros
        x[1, ::3] = 0.0                                 # many zeros
        x[2] *= np.exp(rng.standard_normal(k) * 3)      # wide dynamic range
        x[3, :7] = 6.0e4                                # huge values first
        x[4] *= 1e-4                                    # tiny values (f16 subnormals)
    return x


def scores(xb):
    return np.array([O.variance(r) for r in xb], dtype=np.float32)


@pytest.mark.parametrize("k", [896, 3584, 18944])
@pytest.mark.parametrize("m", [12, 64])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_masks_equal_sequential_chain_on_threshold(sc, k, m, dtype):
    op = layer(sc, k)
    x = rows(k, m, seed=k + m, kind="normed" if dtype == torch.float16 else "mixed")
    xt = torch.from_numpy(x.astype(np.float32)).to("cuda:0").to(dtype)
    xb = xt.to(torch.float16).cpu().numpy().view(np.uint16)
    s = scores(xb)
    one = np.float32(1)
    picks = [s[m // 2], np.nextafter(s[m // 3], one * 2), np.nextafter(s[m // 4], one * 0),
             np.float32(s[m - 1] * (1 + 1e-6)), np.float32(s[1] * (1 - 1e-5)), np.float32(np.median(s))]
    for t4 in picks:
        op.set_thresholds(float(t4), 3e38)
        _, mask, _, nr = op.forward(xt, return_routing=True)
        got = mask.cpu().numpy()
        want = (s >= t4).astype(np.uint8)
        assert np.array_equal(got, want), (k, m, float(t4), np.nonzero(got != want)[0][:8])
        assert int(nr.item()) == int(want.sum())
    op.check_device()


def test_non_finite_rows(sc):
    op = layer(sc, 3584)
    x = rows(3584, 12, seed=5, kind="normed").astype(np.float32)
    x[2, 100] = np.inf
    x[5, 7] = np.nan
    xt = torch.from_numpy(x).to("cuda:0").to(torch.float16)
    xb = xt.cpu().numpy().view(np.uint16)
    s = scores(xb)
    op.set_thresholds(float(np.median(s[np.isfinite(s)])), 3e38)
    _, mask, _, _ = op.forward(xt, return_routing=True)
    t4 = np.float32(op.config.t4)
    want = ((s >= t4) & ~np.isnan(s)).astype(np.uint8)
    assert np.array_equal(mask.cpu().numpy(), want)
