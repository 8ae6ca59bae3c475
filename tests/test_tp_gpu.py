"""Tensor parallelism on two GPUs over NCCL (skipped with fewer than two devices).

1. One C-TARQ layer row-sharded over the two GPUs, both ways the library offers:
   - slice only (sc_forward_split): each rank gets its half of the columns of every token, one NCCL
     all-reduce of the [y_base | y_delta | router sums] buffer, sc_finalize_split;
   - whole token (sc_forward_partial): each rank gets all of x, routes on it, one all-reduce of the
     f32 partial sums, sc_finalize;
   against the unsharded oracle (sampled rows, fast tolerance, identical routing masks).
2. A small Qwen2 model (hidden 256, 4 query / 2 KV heads, intermediate 704, 3 layers, every linear
   C-TARQ) at tensor-parallel 2: column-sharded q/k/v/gate/up, row-sharded o/down through the
   exchange, vocab-parallel lm_head; its greedy tokens (each step a CUDA graph holding the NCCL
   calls) equal the CPU oracle's.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.multiprocessing as mp  # noqa: E402

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    import datetime
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (here, os.path.dirname(here), os.path.join(os.path.dirname(here), "saccade-x2_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                         world_size=world, timeout=datetime.timedelta(seconds=120))


def _layer_rank(rank, world, port, q):
    _init(rank, world, port)
    dist = torch.distributed
    try:
        import saccade_core as sc
        from ctarq_cases import make_case
        case = make_case(384, 2048, 12, 0.02, seed=31, boost=[2, 7, 11], thresholds=(8.0, 3e38))
        dev = torch.device("cuda", rank)
        blocks = {
            "packed_base": torch.from_numpy(case.c.packed_base.view(np.int32)).to(dev),
            "scale_base": torch.from_numpy(case.c.scale_base.view(np.float16)).to(dev),
            "delta_row_ptrs": torch.from_numpy(case.c.delta_row_ptrs.view(np.int32)).to(dev),
            "delta_col_indices": torch.from_numpy(case.c.delta_col_indices.view(np.int32)).to(dev),
            "delta_values": torch.from_numpy(case.c.delta_values).to(dev),
            "delta_scale": torch.from_numpy(np.array([case.c.delta_scale], np.uint16).view(np.float16)),
        }
        k0, k1 = (0, 1024) if rank == 0 else (1024, 2048)
        op = sc.saccade_op_from_compressed(blocks, sc.SaccadeConfig(case.t4, case.t8), case.n, case.k,
                                           device=dev, shard=("rows_range", k0, k1))
        x = torch.from_numpy(case.x_bits.view(np.float16)).to(dev)
        # slice only: one all-reduce of the exchange buffer
        ex = op.forward_split(x[:, k0:k1].contiguous())
        dist.all_reduce(ex)
        y_split, mask_split = op.finalize_split(ex, case.m, world, return_routing=True)
        # whole token: one all-reduce of the partial sums
        part, mask_part = op.forward_partial(x, return_routing=True)
        dist.all_reduce(part)
        y_part = sc.finalize(part)
        torch.cuda.synchronize()
        op.check_device()
        q.put((rank, y_split.cpu().numpy().view(np.uint16), mask_split.cpu().numpy(),
               y_part.cpu().numpy().view(np.uint16), mask_part.cpu().numpy(), int(op.undecided.item())))
    finally:
        dist.destroy_process_group()


def _run(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = sorted([q.get(timeout=600) for _ in range(world)], key=lambda r: r[0])
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    return results


@pytest.fixture(scope="module")
def two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")


def test_row_shards_over_nccl_match_unsharded_oracle(two_gpus):
    from ctarq_cases import assert_fast_close, make_case
    results = _run(_layer_rank, 2)
    case = make_case(384, 2048, 12, 0.02, seed=31, boost=[2, 7, 11], thresholds=(8.0, 3e38))
    y_ref, r_ref, _ = case.oracle().forward(case.x_bits)
    assert r_ref.tolist() == [0, 0, 1, 0, 0, 0, 0, 1, 0, 0, 0, 1]
    for rank, y_split, m_split, y_part, m_part, undecided in results:
        assert undecided == 0
        assert np.array_equal(m_split, r_ref) and np.array_equal(m_part, r_ref)
        assert_fast_close(y_split, y_ref, f"slice-only exchange, rank {rank}")
        assert_fast_close(y_part, y_ref, f"whole-token partials, rank {rank}")
    assert np.array_equal(results[0][1], results[1][1]), "both ranks finalize the same sum"


def _model_rank(rank, world, port, q, steps):
    _init(rank, world, port)
    dist = torch.distributed
    try:
        from saccade_core import qwen2 as Q
        from qwen2_cases import oracle_model
        cfg = Q.Qwen2Config(hidden=256, intermediate=704, layers=3, heads=4, kv_heads=2, head_dim=64, vocab=4096)
        dev = torch.device("cuda", rank)
        ck = Q.random_checkpoint(cfg, seed=7, fill=0.01, device=dev)
        rng = np.random.default_rng(7)
        calib = torch.from_numpy(rng.integers(0, cfg.vocab, (1, 24))).to(dev)
        Q.calibrate(ck, calib, device=dev, max_pos=24 + steps)
        th = torch.tensor([ck.thresholds[li][n] for li in range(cfg.layers) for n in Q.PROJ], device=dev)
        dist.broadcast(th, 0)
        th = th.cpu().numpy().reshape(cfg.layers, len(Q.PROJ), 2)
        for li in range(cfg.layers):
            for j, n in enumerate(Q.PROJ):
                ck.thresholds[li][n] = (float(th[li, j, 0]), float(th[li, j, 1]))
        prompt = rng.integers(0, cfg.vocab, 24)
        model = Q.Qwen2Model(ck, dev, max_batch=1, max_pos=24 + steps, tp=(rank, world, dist.group.WORLD))
        dec = Q.GreedyDecoder(model, 1)
        toks = dec.generate(torch.from_numpy(prompt[None]).to(dev), steps)
        torch.cuda.synchronize()
        model.check_device()
        otoks = None
        if rank == 0:
            otoks, _ = oracle_model(ck, 24 + steps).greedy(prompt, steps)
        q.put((rank, toks.cpu().numpy()[0], otoks, model.undecided_routes(), dec.launches_per_step,
               (model.q0, model.q1, model.k0, model.k1, model.i0, model.i1, model.v0, model.v1)))
        del dec
    finally:
        dist.destroy_process_group()


def test_small_model_tensor_parallel_greedy_matches_oracle(two_gpus):
    steps = 16
    results = _run(_model_rank, 2, steps)
    (_, t0, otoks, und0, launches, split0), (_, t1, _, und1, _, split1) = results
    assert split0 == (0, 2, 0, 1, 0, 320, 0, 2048) and split1 == (2, 4, 1, 2, 320, 704, 2048, 4096)
    assert np.array_equal(t0, t1), "both ranks decode the same tokens"
    assert launches > 0
    assert und0 == 0 and und1 == 0
    assert np.array_equal(t0, otoks), (t0, otoks)
