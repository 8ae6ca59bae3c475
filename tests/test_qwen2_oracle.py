"""CPU checks of the Qwen2 model oracle (oracle/qwen2_oracle.py), the checker of the GPU decoder.

Its steps fix Candle's unknown f32 summation orders to the GPU kernels' orders, so each is checked
here against a plain float64 restatement of the same step of saccade-runner's model (model.rs):
RmsNorm (model.rs:92-98), RotaryEmbedding (model.rs:111-154), causal GQA attention with one and
several 256-key blocks (model.rs:238-257), SiLU (model.rs:295-299).  And the model's KV cache:
decoding a token after a prompt gives the same logits bits as running prompt and token in one pass
(every step is per token apart from attention, which reads the same keys in the same order).
"""
import numpy as np
import pytest

from oracle import oracle as O
from oracle import qwen2_oracle as QO


def rel_err(a, ref):
    return float(np.max(np.abs(a.astype(np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))


@pytest.mark.parametrize("H", [64, 896, 3584, 1000])
def test_rmsnorm_close_to_f64(H):
    rng = np.random.default_rng(H)
    x = (rng.standard_normal((5, H)) * np.array([1, 10, 0.01, 300, 1])[:, None]).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    got = QO.rmsnorm(x, w, 1e-6)
    x64 = x.astype(np.float64)
    ref = x64 / np.sqrt(np.mean(x64 * x64, axis=1, keepdims=True) + 1e-6) * w.astype(np.float64)
    for t in range(5):
        assert rel_err(got[t], ref[t]) < 2e-6


def test_rope_matches_f64_formula():
    rng = np.random.default_rng(1)
    hd, T, heads = 64, 7, 3
    ang = rng.uniform(0, 100, (T, hd // 2))
    cos = np.cos(np.concatenate([ang, ang], 1)).astype(np.float32)
    sin = np.sin(np.concatenate([ang, ang], 1)).astype(np.float32)
    x = rng.standard_normal((T, heads, hd)).astype(np.float32)
    got = QO.rope(x, cos, sin)
    x64 = x.astype(np.float64)
    rot = np.concatenate([-x64[..., hd // 2:], x64[..., :hd // 2]], -1)
    ref = x64 * cos[:, None, :].astype(np.float64) + rot * sin[:, None, :].astype(np.float64)
    assert rel_err(got, ref) < 1e-6


@pytest.mark.parametrize("L,positions", [(40, [39, 5, 0]), (600, [599, 300, 256, 255, 10])])
def test_attention_close_to_plain_softmax(L, positions):
    """GQA (4 query heads over 2 KV heads), causal, one block of keys and three blocks."""
    rng = np.random.default_rng(L)
    nh, nkv, hd = 4, 2, 64
    pos = np.array(positions)
    q = rng.standard_normal((len(pos), nh, hd)).astype(np.float32)
    K = rng.standard_normal((L, nkv, hd)).astype(np.float32)
    V = rng.standard_normal((L, nkv, hd)).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(hd))
    got = QO.attention(q, K, V, pos, scale)
    G = nh // nkv
    for t, p in enumerate(pos):
        for h in range(nh):
            s = K[:p + 1, h // G].astype(np.float64) @ q[t, h].astype(np.float64) * float(scale)
            e = np.exp(s - s.max())
            ref = (e / e.sum()) @ V[:p + 1, h // G].astype(np.float64)
            assert rel_err(got[t, h], ref) < 2e-5, (t, h)


def test_silu_close_to_f64():
    """Three f32 roundings (exp, 1 + e, the quotient): within 3 ulp of the f64 value."""
    g = np.linspace(-30, 30, 4001).astype(np.float32)
    got = QO.silu(g)
    g64 = g.astype(np.float64)
    ref = g64 / (1 + np.exp(-g64))
    assert np.all(np.abs(got - ref) <= 3 * np.spacing(np.abs(ref).astype(np.float32)) + 1e-38)


def _tiny_oracle(seed=3, max_pos=64):
    from saccade_core.qwen2 import PROJ, Qwen2Config, rope_tables
    cfg = Qwen2Config(hidden=128, intermediate=256, layers=2, heads=4, kv_heads=2, head_dim=32, vocab=300)
    rng = np.random.default_rng(seed)
    layers = []
    for _ in range(cfg.layers):
        L = {}
        for name in PROJ:
            n, k = cfg.proj_shape(name)
            w = (rng.standard_normal((n, k)) * 0.05).astype(np.float32)
            c = O.compress(w, O.percentile_threshold(w, 0.05))
            # thresholds inside the range of scores, so that some tokens route and some do not
            L[name] = O.OracleLinear(c, 0.9, 3e38)
        L["bias"] = {name: (rng.standard_normal(cfg.proj_shape(name)[0]) * 0.01).astype(np.float32)
                     for name in ("q", "k", "v")}
        L["norm_in"] = (1 + 0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32)
        L["norm_post"] = (1 + 0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32)
        layers.append(L)
    embed = rng.standard_normal((cfg.vocab, cfg.hidden)).astype(np.float16).astype(np.float32)
    cos, sin = rope_tables(cfg, max_pos)
    final = (1 + 0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32)
    return QO.Qwen2Oracle(cfg, layers, final, embed, embed, cos, sin)


def test_decode_after_prompt_equals_one_pass():
    ids = np.random.default_rng(9).integers(0, 300, 13)
    inc = _tiny_oracle()
    inc.forward(ids[:12])
    logits_inc = inc.forward(ids[12:])
    routed_inc = [r for (_, _, r) in inc.routed]
    full = _tiny_oracle()
    logits_full = full.forward(ids)
    assert np.array_equal(logits_inc.view(np.uint32), logits_full.view(np.uint32))
    # the last token's routing is the same either way, and the thresholds route some tokens
    routed_full = [r[-1:] for (_, _, r) in full.routed]
    assert all(np.array_equal(a, b) for a, b in zip(routed_inc, routed_full))
    assert any(r.any() for (_, _, r) in full.routed) and not all(r.all() for (_, _, r) in full.routed)


def test_greedy_is_deterministic_and_feeds_its_tokens():
    prompt = np.random.default_rng(4).integers(0, 300, 6)
    a, gaps = _tiny_oracle().greedy(prompt, 5)
    b, _ = _tiny_oracle().greedy(prompt, 5)
    assert np.array_equal(a, b) and len(a) == 5 and np.all(gaps >= 0)
    # the same tokens from one pass over prompt + the first four greedy tokens
    o = _tiny_oracle()
    logits = o.forward(np.concatenate([prompt, a[:4]]))
    assert int(np.argmax(logits)) == a[4]
