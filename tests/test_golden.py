"""Golden fixtures (tests/golden, written by tests/golden/make_golden.py from the C oracle).

CPU: the oracle (compressor, router, forward) still reproduces every stored array bit for bit,
and the seeded single-layer configuration and Qwen2-7B q shape still hash to the stored digests.
GPU: the CUDA library reproduces the stored outputs (exact mode bit for bit, fast modes within
the tolerance, device packer bit for bit)."""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from ctarq_cases import assert_fast_close, make_case

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
META = json.load(open(os.path.join(GOLD, "digests.json")))


def load(name):
    z = np.load(os.path.join(GOLD, f"{name}.npz"))
    return {k: z[k] for k in z.files}


def compressed(g, n, k):
    return O.Compressed(g["packed_base"], g["scale_base"], g["delta_row_ptrs"], g["delta_col_indices"],
                        g["delta_values"], int(g["delta_scale"][0]), n, k)


def digest(a):
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


@pytest.mark.parametrize("spec", META["small"], ids=[s["name"] for s in META["small"]])
def test_oracle_reproduces_small_fixture(spec):
    g = load(spec["name"])
    n, k = spec["n"], spec["k"]
    if "w" in g:
        c = O.compress(g["w"], O.percentile_threshold(g["w"], spec["fill"]))
        for key in ("packed_base", "scale_base", "delta_row_ptrs", "delta_col_indices", "delta_values"):
            assert np.array_equal(getattr(c, key), g[key]), key
        assert c.delta_scale == int(g["delta_scale"][0])
    t4, t8 = (float(v) for v in g["thresholds"])
    y, routed, acc = O.OracleLinear(compressed(g, n, k), t4, t8).forward(g["x_bits"])
    assert np.array_equal(y, g["y_bits"])
    assert np.array_equal(routed, g["routed"])
    assert np.array_equal(acc.view(np.uint32), g["acc"].view(np.uint32))


@pytest.mark.parametrize("name", sorted(META["digests"]))
def test_oracle_reproduces_digests(name):
    d = META["digests"][name]
    case = make_case(d["n"], d["k"], d["m"], d["fill"], seed=d["seed"], boost=d["boost"])
    c = case.c
    y, routed, acc = case.oracle().forward(case.x_bits)
    got = {"packed_base": c.packed_base, "scale_base": c.scale_base, "delta_row_ptrs": c.delta_row_ptrs,
           "delta_col_indices": c.delta_col_indices, "delta_values": c.delta_values,
           "delta_scale": np.array([c.delta_scale], dtype=np.uint16), "x_bits": case.x_bits,
           "thresholds": np.array([case.t4, case.t8], dtype=np.float32), "y_bits": y, "routed": routed, "acc": acc}
    for key, want in d["sha256"].items():
        assert digest(got[key]) == want, f"{name}: {key} changed"


# ------------------------------------------------------------------ the CUDA library on the fixtures

@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["exact", "fast", "fast_tc", "fast_tc8"])
@pytest.mark.parametrize("spec", META["small"], ids=[s["name"] for s in META["small"]])
def test_library_on_small_fixture(spec, mode):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import saccade_core as sc
    g = load(spec["name"])
    n, k = spec["n"], spec["k"]
    dev = torch.device("cuda", 0)

    def t(a, dt):
        return torch.from_numpy(np.ascontiguousarray(a).view(dt)).to(dev)

    sp = sc.SparseDeltaMatrix(t(g["delta_row_ptrs"], np.int32), t(g["delta_col_indices"], np.int32),
                              t(g["delta_values"], np.uint8),
                              torch.tensor([int(g["delta_scale"][0])], dtype=torch.int32).to(torch.int16)
                              .view(torch.float16)) if g["delta_values"].size else None
    t4, t8 = (float(v) for v in g["thresholds"])
    op = sc.SaccadeLinearOp(t(g["packed_base"], np.int32), t(g["scale_base"], np.float16), sp,
                            sc.SaccadeConfig(t4, t8), n, k, device=dev, mode=mode)
    x = torch.from_numpy(g["x_bits"].view(np.float16)).to(dev)
    y, mask, _, _ = op.forward(x, return_routing=True)
    torch.cuda.synchronize()
    op.check_device()
    assert np.array_equal(mask.cpu().numpy(), g["routed"])
    yb = y.cpu().numpy().view(np.uint16)
    if mode == "exact":
        assert np.array_equal(yb, g["y_bits"])
    else:
        assert_fast_close(yb, g["y_bits"], f"{spec['name']} {mode}")
    if "w" in g:
        wd = torch.from_numpy(g["w"]).to(dev)
        c = sc.compress_tensor_to_saccade(wd, sc.compute_percentile_threshold(wd, spec["fill"]))
        for key in ("packed_base", "delta_row_ptrs", "delta_col_indices"):
            assert np.array_equal(c[key].view(torch.int32).cpu().numpy().view(np.uint32), g[key]), key
        assert np.array_equal(c["delta_values"].cpu().numpy(), g["delta_values"])
