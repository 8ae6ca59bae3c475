"""The row-sharded (tensor-parallel) path on two ranks over gloo, on the CPU.

Whole-token form (sc_forward_partial): each rank takes its slice of the input columns of a
compressed layer (the column ranges a ROWS shard of sc_layer_create keeps: K * r / n rounded up to
64), routes on the whole token, computes its f32 partial with the oracle, and the ranks all-reduce
(sum) the partials.  Slice-only form (sc_forward_split): each rank sees only its slice and
all-reduces one [y_base | y_delta | router sums] vector, then every rank routes on the summed sums
(oracle/split_oracle.py restates the three steps).  Both must match the unsharded oracle within
the fast-path tolerance (only the f32 summation order changes) with identical routing masks."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def column_slice(c, k0, k1):
    """The reference-format layer restricted to input columns [k0, k1) (multiples of 8)."""
    from oracle import oracle as O
    n = c.out_features
    packed = np.ascontiguousarray(c.packed_base[:, k0 // 8:k1 // 8])
    rp = [0]
    cols, vals = [], []
    for r in range(n):
        lo, hi = int(c.delta_row_ptrs[r]), int(c.delta_row_ptrs[r + 1])
        for e in range(lo, hi):
            col = int(c.delta_col_indices[e])
            if k0 <= col < k1:
                cols.append(col - k0)
                vals.append(c.delta_values[e])
        rp.append(len(cols))
    return O.Compressed(packed, c.scale_base, np.array(rp, dtype=np.uint32), np.array(cols, dtype=np.uint32),
                        np.array(vals, dtype=np.uint8), c.delta_scale, n, k1 - k0)


def rows_shard_columns(k, rank, world):
    """Input columns [k0, k1) of ROWS shard `rank` of `world`, as sc_layer_create computes them
    (K * i / n rounded up to a multiple of 64, the last shard ending at K)."""
    def up64(v):
        return (v + 63) // 64 * 64
    k0 = min(k, up64(k * rank // world))
    k1 = k if rank + 1 == world else min(k, up64(k * (rank + 1) // world))
    return k0, k1


def _rank(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.dirname(here))
    from oracle import oracle as O
    from ctarq_cases import make_case
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = make_case(192, 1024, 6, 0.03, seed=77, boost=[1, 4])
        full = case.oracle()
        _, routed_full, _ = full.forward(case.x_bits)
        k0, k1 = rows_shard_columns(case.k, rank, world)
        part = O.OracleLinear(column_slice(case.c, k0, k1), case.t4, case.t8)
        _, routed, acc = part.forward(np.ascontiguousarray(case.x_bits[:, k0:k1]), force_route=routed_full)
        t = torch.from_numpy(acc.copy())
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        masks = [torch.zeros(case.m, dtype=torch.uint8) for _ in range(world)]
        dist.all_gather(masks, torch.from_numpy(routed_full.copy()))
        q.put((rank, t.numpy(), [m.numpy() for m in masks]))
    finally:
        dist.destroy_process_group()


def test_row_shards_all_reduce_two_ranks():
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from ctarq_cases import assert_acc_close, make_case
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    case = make_case(192, 1024, 6, 0.03, seed=77, boost=[1, 4])
    _, rr, acc_ref = case.oracle().forward(case.x_bits)
    for _, acc, masks in results:
        assert_acc_close(acc, acc_ref, "2-rank all-reduce")
        for m in masks:
            assert np.array_equal(m, rr)
    assert np.array_equal(results[0][1], results[1][1]), "every rank holds the same reduced sum"


# ------------------------------------------------------------------ tensor-parallel MLP, two ranks

def row_slice(c, r0, r1):
    """The layer restricted to output rows [r0, r1) (what a COLUMNS shard keeps: rows move with
    their scales and their dW)."""
    from oracle import oracle as O
    lo, hi = int(c.delta_row_ptrs[r0]), int(c.delta_row_ptrs[r1])
    rp = (c.delta_row_ptrs[r0:r1 + 1] - lo).astype(np.uint32)
    return O.Compressed(np.ascontiguousarray(c.packed_base[r0:r1]), np.ascontiguousarray(c.scale_base[r0:r1]), rp,
                        np.ascontiguousarray(c.delta_col_indices[lo:hi]), np.ascontiguousarray(c.delta_values[lo:hi]),
                        c.delta_scale, r1 - r0, c.in_features)


def _silu_mul(g_bits, u_bits):
    """f16(silu(g) * u) in f32: the MLP's step between gate/up and down."""
    g = g_bits.view(np.float16).astype(np.float32)
    u = u_bits.view(np.float16).astype(np.float32)
    return ((g / (np.float32(1.0) + np.exp(-g))) * u).astype(np.float16).view(np.uint16)


def _mlp_layers():
    from oracle import oracle as O
    rng = np.random.default_rng(91)

    def comp(n, k):
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        return O.compress(w, O.percentile_threshold(w, 0.03))

    gate, up, down = comp(384, 256), comp(384, 256), comp(256, 384)
    x = rng.standard_normal((5, 256)).astype(np.float32)
    x[3] *= 8.0
    return gate, up, down, x.astype(np.float16).view(np.uint16)


def _down_threshold():
    """The down router threshold of the MLP case: between the unboosted and the boosted token's
    variance of h (computed on the unsharded oracle, as calibration would)."""
    from oracle import oracle as O
    gate, up, _, xb = _mlp_layers()
    g, _, _ = O.OracleLinear(gate, 8.0, 3e38).forward(xb)
    u, _, _ = O.OracleLinear(up, 8.0, 3e38).forward(xb)
    return _down_route(_silu_mul(g, u))[0]


def _down_route(h_bits):
    """Threshold between the unboosted and the boosted token's variance of h, and the mask."""
    from oracle import oracle as O
    s = np.array([O.variance(h_bits[t]) for t in range(h_bits.shape[0])])
    t4 = float(np.sqrt(np.max(np.delete(s, 3)) * s[3]))
    return t4, (s >= t4).astype(np.uint8)


def _mlp_rank(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.dirname(here))
    from oracle import oracle as O
    from oracle import split_oracle as S
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gate, up, down, xb = _mlp_layers()
        inter = gate.out_features
        r0, r1 = rows_shard_columns(inter, rank, world)  # down's ROWS shard; gate/up keep the same rows
        # column-parallel gate and up: this rank's rows, x replicated, no exchange
        g, _, _ = O.OracleLinear(row_slice(gate, r0, r1), 8.0, 3e38).forward(xb)
        u, _, _ = O.OracleLinear(row_slice(up, r0, r1), 8.0, 3e38).forward(xb)
        h_part = _silu_mul(g, u)
        # row-parallel down on this rank's slice of h only: one all-reduce of the exchange vector,
        # then the routing decision on the summed router sums (no gather of h)
        t4 = _down_threshold()
        ex = torch.from_numpy(S.split_exchange(column_slice(down, r0, r1), h_part))
        dist.all_reduce(ex, op=dist.ReduceOp.SUM)
        y, routed, undecided = S.split_finalize(ex.numpy(), h_part.shape[0], down.out_features, inter, world,
                                                t4, 3e38)
        q.put((rank, g, u, h_part, routed, y, undecided))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_mlp_two_ranks():
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from oracle import oracle as O
    from ctarq_cases import assert_acc_close, assert_fast_close
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mlp_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=120) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gate, up, down, xb = _mlp_layers()
    g, rg, _ = O.OracleLinear(gate, 8.0, 3e38).forward(xb)
    u, _, _ = O.OracleLinear(up, 8.0, 3e38).forward(xb)
    assert rg.tolist() == [0, 0, 0, 1, 0]
    h = _silu_mul(g, u)
    t4, routed = _down_route(h)
    y, rd, acc_ref = O.OracleLinear(down, t4, 3e38).forward(h)
    assert rd.tolist() == [0, 0, 0, 1, 0]
    inter = gate.out_features
    for rank, g_r, u_r, h_r, routed_r, y_r, undecided in results:
        r0, r1 = rows_shard_columns(inter, rank, world)
        assert np.array_equal(g_r, g[:, r0:r1]) and np.array_equal(u_r, u[:, r0:r1]), "rows are independent"
        assert np.array_equal(h_r, h[:, r0:r1])
        assert undecided == 0 and np.array_equal(routed_r, rd), "routed on the summed sums as on whole tokens"
        assert_fast_close(y_r, y, f"tp mlp rank {rank} y")
    assert np.array_equal(results[0][5], results[1][5]), "every rank holds the same output"


def _split_rank(rank, world, port, q, bypass):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    sys.path.insert(0, os.path.dirname(here))
    from oracle import split_oracle as S
    from ctarq_cases import make_case
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        case = make_case(160, 1280, 9, 0.02, seed=78, boost=[0, 5, 6], thresholds=(8.0, 3e38))
        k0, k1 = rows_shard_columns(case.k, rank, world)
        ex = torch.from_numpy(S.split_exchange(S.slice_columns(case.c, k0, k1),
                                               np.ascontiguousarray(case.x_bits[:, k0:k1])))
        dist.all_reduce(ex, op=dist.ReduceOp.SUM)
        q.put((rank,) + S.split_finalize(ex.numpy(), case.m, case.n, case.k, world, case.t4, case.t8, bypass))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,bypass", [(2, False), (3, False), (2, True)])
def test_split_exchange_ranks(world, bypass):
    """The three-step exchange over gloo ranks equals the unsharded oracle: same routing mask, y
    within the fast-path tolerance, every rank the same result, no undecided token."""
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, here)
    from ctarq_cases import assert_fast_close, make_case
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_split_rank, args=(r, world, port, q, bypass)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted([q.get(timeout=120) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    case = make_case(160, 1280, 9, 0.02, seed=78, boost=[0, 5, 6], thresholds=(8.0, 3e38))
    y_ref, r_ref, _ = case.oracle().forward(case.x_bits, bypass=bypass)
    if bypass:  # the dense path: every token takes base + dW (the library reports them all routed)
        r_ref = np.ones(case.m, dtype=np.uint8)
    else:
        assert r_ref.tolist() == [1, 0, 0, 0, 0, 1, 1, 0, 0]
    for _, y, routed, undecided in results:
        assert undecided == 0
        assert np.array_equal(routed, r_ref)
        assert_fast_close(y, y_ref, f"split exchange over {world} ranks")
    for r in results[1:]:
        assert np.array_equal(r[1], results[0][1])
