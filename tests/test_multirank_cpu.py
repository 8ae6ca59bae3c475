"""The row-sharded (tensor-parallel) path on two ranks over gloo, on the CPU.

Each rank takes its slice of the input columns of a compressed layer (the column ranges a
ROWS shard of sc_layer_create keeps: K * r / n rounded to 64), routes on the whole token as every
shard must, computes its f32 partial with the oracle, and the ranks all-reduce (sum) the
partials -- the exchange step of the sharded layer.  The sum must match the unsharded oracle
within the fast-path tolerance (only the f32 summation order changes) and the routing masks must
be identical on every rank."""
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
        kb = case.k // 64
        k0 = (kb * rank // world) * 64
        k1 = (kb * (rank + 1) // world) * 64 if rank + 1 < world else case.k
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
