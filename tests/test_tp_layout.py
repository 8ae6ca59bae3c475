"""The tensor-parallel layout of the Qwen2 decoder on the CPU: every rank's query and KV heads, its
intermediate slice and its vocabulary slice, at 1, 2, 4 and 8 ranks, for the Qwen2-0.5B, -7B and
-72B shapes.  The slices must tile the whole, respect the library's shard granularity (whole heads;
multiples of 64 columns for row shards, 16 rows for column shards), and give every query head the
KV head the model assigns it (head h reads KV head h // (heads / kv_heads))."""
import pytest

torch = pytest.importorskip("torch")

from saccade_core import qwen2 as Q  # noqa: E402

CONFIGS = [Q.Qwen2Config.qwen2_0_5b(), Q.Qwen2Config.qwen2_7b(), Q.Qwen2Config.qwen2_72b()]


@pytest.mark.parametrize("cfg", CONFIGS, ids=["0.5b", "7b", "72b"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_slices_tile_the_model(cfg, world):
    if world > cfg.kv_heads and world % cfg.kv_heads:
        pytest.skip("KV heads do not split over this many ranks")
    G = cfg.heads // cfg.kv_heads
    heads, inter, vocab = [], [], []
    for r in range(world):
        q0, q1, k0, k1 = Q.head_split(cfg, r, world)
        assert 0 <= q0 < q1 <= cfg.heads and 0 <= k0 < k1 <= cfg.kv_heads
        for h in range(q0, q1):  # the rank's KV heads serve all its query heads
            assert k0 <= h // G < k1
        # local GQA mapping of the attention kernel: local head j reads local KV head j // (nh / nkv)
        nh, nkv = q1 - q0, k1 - k0
        assert nh % nkv == 0
        for j in range(nh):
            assert (q0 + j) // G - k0 == j // (nh // nkv)
        # row-shard columns of o (whole heads) on 64-column boundaries, column-shard rows on 16
        assert (q0 * cfg.head_dim) % 64 == 0 and (k0 * cfg.head_dim) % 16 == 0
        heads.append((q0, q1))
        i0, i1 = Q.inter_split(cfg, r, world)
        assert i0 % 64 == 0 and (i1 % 64 == 0 or i1 == cfg.intermediate) and i1 > i0
        inter.append((i0, i1))
        v0, v1 = Q.vocab_split(cfg, r, world)
        assert v1 > v0
        vocab.append((v0, v1))
    for parts, total in ((heads, cfg.heads), (inter, cfg.intermediate), (vocab, cfg.vocab)):
        assert parts[0][0] == 0 and parts[-1][1] == total
        assert all(parts[i][1] == parts[i + 1][0] for i in range(len(parts) - 1))
    if cfg.heads == 28 and world == 8:  # Qwen2-7B at 8 ranks: each KV head's 7 query heads split 3 + 4
        assert [b - a for a, b in heads] == [3, 4] * 4
