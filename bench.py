#!/usr/bin/env python
"""Qwen2-7B decode tok/s (default workload) and C-TARQ linear effective HBM GB/s (--workload linear).

--workload decode (default): the Qwen2-7B architecture (hidden 3584, intermediate 18944, 28 layers,
28 query / 4 KV heads, head_dim 128, vocab 152064), random init, every linear C-TARQ (1 % dW,
router thresholds calibrated per projection at the 75th / 95th percentile), batch 64, 512-token
random prompts, then greedy decoding.  One step = one decode step of the 64 sequences (64 tokens),
replayed as one CUDA graph; tensor parallel over --gpus N (column-sharded q/k/v/gate/up, row-sharded
o/down with one NCCL all-reduce of [y_base | y_delta | router sums] each, vocab-parallel lm_head).
value = 64 tokens per step / max-over-ranks device time per step.
--model qwen2-72b: the Qwen2-72B architecture (hidden 8192, intermediate 29568, 80 layers, 64 query /
8 KV heads), batch 8, 2048-token prompts (the prefill's device time reported beside), 128 steps;
--route-pct 0.9 / 0.5 places t4 so that ~10 % / ~50 % of the tokens route.

--workload linear: one step = one decode pass of M tokens through every C-TARQ linear of Qwen2-7B
(28 layers x {q 3584->3584, k 3584->512, v 3584->512, o 3584->3584, gate 3584->18944,
up 3584->18944, down 18944->3584}), 1 % dW, a seeded 25 % of the calls routed.
Weights total 3.3 GB, far above L2, so no flush is needed between steps.

Effective bytes per call (the metric's numerator, independent of the device layout):
    2*M*K (x) + N*K/2 (int4 base) + 2*N (f16 scales) + [any token routed]*(3*nnz + 4*(N+1)) + 2*M*N (y)
value = bytes of all calls of all ranks / max-over-ranks device time (CUDA events).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]          # decode tok/s
  python bench.py --model qwen2-72b [--route-pct 0.9|0.5] [--gpus N]                # 72B prefill + decode
  python bench.py --workload linear [--tokens M] [--impl reference]                # linear GB/s
  python bench.py --sweep OUT.md [--sweep-fills 0.005,0.01,0.04]
                                      # single calls: 4 shapes x M 1..4096 x routed 0/10/25/100 %
                                      # x dW densities

--impl reference times the reference's CPU algorithm (the oracle restatement of
saccade-core's op.rs; the Rust reference cannot be built here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "saccade-x2_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

HIDDEN, INTER, LAYERS, KV_DIM = 3584, 18944, 28, 512
PROJ = [("q", 3584, HIDDEN), ("k", KV_DIM, HIDDEN), ("v", KV_DIM, HIDDEN), ("o", HIDDEN, 3584),
        ("gate", INTER, HIDDEN), ("up", INTER, HIDDEN), ("down", HIDDEN, INTER)]  # (name, N, K)

# decode workloads: label, hidden, intermediate, layers, KV width (KV heads x head_dim), and the
# defaults of batch, prompt tokens, decode steps and sequences per prefill pass
DECODE_MODELS = {
    "qwen2-7b": ("Qwen2-7B", 3584, 18944, 28, 512, 64, 512, 256, 16),
    "qwen2-72b": ("Qwen2-72B", 8192, 29568, 80, 1024, 8, 2048, 128, 2),
}


def model_proj(model):
    """(name, N, K) of the seven linears of one decoder layer of `model`."""
    _, h, i, _, kv = DECODE_MODELS[model][:5]
    return [("q", h, h), ("k", kv, h), ("v", kv, h), ("o", h, h), ("gate", i, h), ("up", i, h), ("down", h, i)]
T4_BOOSTED = 8.0        # between the variance of N(0,1) tokens (~1) and x8 tokens (~64)
T8_NEVER = float(np.finfo(np.float32).max)
METRIC = "C-TARQ linear effective HBM GB/s"


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--workload", default="decode", choices=["decode", "linear"])
    ap.add_argument("--steps", type=int, default=None, help="timed steps (decode 100, linear 20)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed steps (decode 5, linear 3)")
    ap.add_argument("--model", default="qwen2-7b", choices=sorted(DECODE_MODELS),
                    help="decode: the architecture (qwen2-72b: batch 8, 2048-token prompts, 128 steps)")
    ap.add_argument("--batch", type=int, default=None, help="decode: sequences (7B 64, 72B 8)")
    ap.add_argument("--prompt", type=int, default=None, help="decode: prompt tokens per sequence (512, 2048)")
    ap.add_argument("--decode-steps", type=int, default=None, help="decode: greedy steps of the workload (256, 128)")
    ap.add_argument("--prefill-chunk", type=int, default=None, help="decode: sequences per prefill pass (16, 2)")
    ap.add_argument("--route-pct", type=float, default=0.75,
                    help="decode: percentile of the calibration scores at t4 (0.75 routes ~25 %% of tokens, "
                         "0.9 ~10 %%, 0.5 ~50 %%); t8 at the 95th (99th above 0.9)")
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--layers", type=int, default=None, help="decoder layers (default: the model's)")
    ap.add_argument("--fill", type=float, default=0.01)
    ap.add_argument("--route-frac", type=float, default=0.25)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="fast", choices=["fast", "fast_tc", "fast_tc8", "exact"])
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--fused-route", default="none", choices=["none", "norm", "all"],
                    help="decode: routers fused into the RMSNorm kernels (norm), also into SiLU * up (all)")
    ap.add_argument("--no-group", action="store_true",
                    help="one launch per projection, the reference's calling pattern (no grouped q/k/v, gate/up)")
    ap.add_argument("--sweep", metavar="PATH",
                    help="instead of the step: time single calls over a grid of shapes x tokens x routed "
                         "fractions (one GPU) and write a markdown table to PATH")
    ap.add_argument("--sweep-fills", default=None, metavar="LIST",
                    help="comma-separated dW densities for --sweep (default: --fill)")
    ap.add_argument("--sweep-tokens", default=None, metavar="LIST",
                    help="comma-separated token counts for --sweep (default: 1,4,16,64,256,1024,4096)")
    ap.add_argument("--sweep-shapes", default=None, metavar="LIST",
                    help="comma-separated shape labels for --sweep (q/o, k/v, gate/up, down; default: all)")
    ap.add_argument("--sweep-routed", default=None, metavar="LIST",
                    help="comma-separated routed fractions for --sweep (default: 0,0.1,0.25,1)")
    a = ap.parse_args(argv)
    _, _, _, layers, _, batch, prompt, dsteps, chunk = DECODE_MODELS[a.model]
    if a.workload != "decode":
        layers = LAYERS
    a.layers = layers if a.layers is None else a.layers
    a.batch = batch if a.batch is None else a.batch
    a.prompt = prompt if a.prompt is None else a.prompt
    a.decode_steps = dsteps if a.decode_steps is None else a.decode_steps
    a.prefill_chunk = chunk if a.prefill_chunk is None else a.prefill_chunk
    if a.steps is None:
        a.steps = 100 if a.workload == "decode" else 20
    if a.warmup is None:
        a.warmup = 5 if a.workload == "decode" else 3
    return a


def launches_per_call(args):
    """Kernels one forward call launches: the router-fused decode kernel for <= 8 tokens in the
    fast modes; otherwise the router, then the exact kernel or the token gather and the GEMM."""
    if args.mode != "exact" and args.tokens <= 8:
        return 1
    return 2 if args.mode == "exact" else 3


def launches_per_step(args, units):
    """Kernels of one step: a group of layers takes one launch when it decodes fused."""
    per = launches_per_call(args)
    return sum(1 if (grp is not None and per == 1) else per * len(idx) for idx, grp in units)


def launch_kind(args):
    if args.mode != "exact" and args.tokens <= 8:
        fast = ("k_ctarq_fused_mma<int8> (router-fused decode, s8 mma.sync on base-256 digits of x)"
                if args.tokens == 1 else "k_ctarq_fused_mma (router-fused decode, f16 mma.sync)")
        return {"fast_tc": "k_ctarq_fused_tc<f16> (router-fused decode, tcgen05)",
                "fast_tc8": "k_ctarq_fused_tc<fp8> (router-fused decode, tcgen05 e4m3)"}.get(args.mode, fast)
    return "k_decode_exact (+ k_router)" if args.mode == "exact" else "k_ctarq_gemm (+ k_router, k_gather_tokens)"


def call_bytes(n, k, m, nnz, routed):
    return 2 * m * k + n * k // 2 + 2 * n + (3 * nnz + 4 * (n + 1) if routed else 0) + 2 * m * n


# Projections reading the same activations in the decoder (model.rs:217-219, 296-297): q, k, v
# take the normed hidden state, gate and up the post-attention normed state.
INPUT_OF = {"q": "attn", "k": "attn", "v": "attn", "o": "o", "gate": "mlp", "up": "mlp", "down": "down"}


def stack_spec(layers, m, route_frac, seed, proj=PROJ):
    """(layer, proj, N, K, boosted-token list) for every call of one step; calls that read the
    same activations share their boosted tokens (each token of each input is boosted with
    probability route_frac)."""
    rng = np.random.default_rng(seed)
    calls = []
    for li in range(layers):
        boosted_of = {}
        for name, n, k in proj:
            inp = INPUT_OF[name]
            if inp not in boosted_of:
                boosted_of[inp] = [t for t in range(m) if rng.random() < route_frac]
            calls.append((li, name, n, k, boosted_of[inp]))
    return calls


def workload_config(args, calls, step_bytes):
    """The workload keys both arms report: the same stack of calls, sizes and routing."""
    return {"workload": "qwen2-7b decoder linear stack, decode", "tokens": args.tokens, "layers": args.layers,
            "calls_per_step": len(calls), "routed_calls_per_step": sum(1 for c in calls if c[4]),
            "dw_fill": args.fill, "route_frac": args.route_frac, "bytes_per_step": step_bytes,
            "weights": "int4 base + i8 dW, f32 accumulation"}


def synth_compressed_np(n, k, fill, rng):
    """Reference-format buffers with the value distributions of a packed N(0, 0.02) matrix."""
    packed = rng.integers(0, 2 ** 32, size=(n, k // 8), dtype=np.uint32)
    scale = (0.02 * (3.0 + np.abs(rng.standard_normal(n)) * 0.5) / 7.0).astype(np.float16)
    nnz = int(round(n * k * fill))
    flat = np.sort(rng.choice(n * k, size=nnz, replace=False))
    rows, cols = flat // k, flat % k
    row_ptrs = np.zeros(n + 1, dtype=np.uint32)
    row_ptrs[1:] = np.cumsum(np.bincount(rows, minlength=n))
    vals = rng.integers(-127, 128, size=nnz).astype(np.int8).view(np.uint8)
    ds = np.float16(0.006 / 127.0)
    return packed, scale, row_ptrs, cols.astype(np.uint32), vals, ds


def make_x(m, k, boosted, rng):
    x = rng.standard_normal((m, k)).astype(np.float32)
    for t in boosted:
        x[t] *= 8.0
    return x.astype(np.float16)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """SM clock and clock-event reasons of this GPU, polled through NVML from a host thread every
    ~2 ms while the timed region runs (the host only waits on the GPU there)."""
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, device):
        self.device = device
        self.samples = []
        self.thread = None
        self.stop_flag = False
        self.err = None

    def _handle(self, nv):
        import torch
        try:
            p = torch.cuda.get_device_properties(self.device)
            bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:  # noqa: BLE001 - fall back to the CUDA ordinal
            return nv.nvmlDeviceGetHandleByIndex(self.device.index or 0)

    def start(self):
        import threading
        try:
            import pynvml as nv
            nv.nvmlInit()
            h = self._handle(nv)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
        except Exception as e:  # noqa: BLE001
            self.err = f"nvml unavailable: {type(e).__name__}"
            return

        def run():
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            while not self.stop_flag:
                try:
                    self.samples.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)), int(get_reasons(h)),
                                         nv.nvmlDeviceGetPowerUsage(h) / 1000.0))
                except Exception:  # noqa: BLE001
                    pass
                time.sleep(0.002)

        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()

    def stop(self):
        if self.thread is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no sampler"]}
        self.stop_flag = True
        self.thread.join(timeout=5)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["no samples"]}
        reasons = sorted({n for _, r, _ in self.samples for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(c for c, _, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples),
                "power_w_median": round(statistics.median(p for _, _, p in self.samples), 1),
                "source": "nvml, 2 ms polling during the timed region"}


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ------------------------------------------------------------------ CPU (oracle) side

def build_oracle_stack(calls, fill, seed, tokens):
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    items = []
    for li, name, n, k, boosted in calls:
        packed, scale, rp, cols, vals, ds = synth_compressed_np(n, k, fill, rng)
        c = O.Compressed(packed, scale.view(np.uint16), rp, cols, vals, int(np.array([ds]).view(np.uint16)[0]), n, k)
        op = O.OracleLinear(c, T4_BOOSTED, T8_NEVER)
        x = make_x(tokens, k, boosted, rng).view(np.uint16)
        items.append((op, x, call_bytes(n, k, tokens, c.nnz, len(boosted) > 0)))
    return items


def time_oracle(items, reps, native=True):
    t0 = time.perf_counter()
    nbytes = 0
    for _ in range(reps):
        for op, x, b in items:
            op.forward(x, native=native)
            nbytes += b
    dt = time.perf_counter() - t0
    return nbytes / dt / 1e9, dt


def cpu_baseline(args):
    """The oracle's op.rs restatement timed on the host cores over a bounded sample."""
    from oracle import oracle as O
    try:
        O.lib(native=True)
        native = True
    except Exception:  # noqa: BLE001 - no compiler on the host: use the portable build
        native = False
    calls = stack_spec(1, args.tokens, args.route_frac, seed=1234)
    items = build_oracle_stack(calls, args.fill, 99, args.tokens)
    _, dt1 = time_oracle(items, 1, native)
    reps = max(1, min(100000, int(args.cpu_seconds / max(dt1, 1e-4))))  # ~cpu_seconds of CPU work
    gbs, dt = time_oracle(items, reps, native)
    cores = os.cpu_count()
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"1 Qwen2-7B decoder layer (7 linears, M={args.tokens}) x {reps} reps, {dt:.1f} s; "
                      f"C restatement of op.rs, OpenMP over rows ({'-march=native' if native else 'x86-64-v3'})"}


def run_reference_linear(args, rank):
    if rank != 0:
        return
    from oracle import oracle as O
    try:
        O.lib(native=True)
        native = True
    except Exception:  # noqa: BLE001
        native = False
    calls = stack_spec(args.layers, args.tokens, args.route_frac, seed=1234)
    items = build_oracle_stack(calls, args.fill, 99, args.tokens)
    step_bytes = sum(b for _, _, b in items)
    config = workload_config(args, calls, step_bytes)
    # one step is bounded: if the whole stack takes too long on this host, time a prefix of it
    _, dt1 = time_oracle(items[: 7], 1, native)
    per_step_est = dt1 * len(items) / 7
    budget = 150.0 / max(1, args.steps + args.warmup)
    if per_step_est > budget:
        keep = max(7, int(len(items) * budget / per_step_est) // 7 * 7)
        items = items[:keep]
        step_bytes = sum(b for _, _, b in items)
    for _ in range(args.warmup):
        time_oracle(items, 1, native)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        time_oracle(items, 1, native)
    dt = time.perf_counter() - t0
    value = step_bytes * args.steps / dt / 1e9
    sample = (f"{len(items)} of {len(calls)} linears per step (Qwen2-7B stack, M={args.tokens}); "
              f"C restatement of op.rs (Rust reference not buildable here), OpenMP over rows")
    out = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
           "config": config,
           "impl": "reference",
           "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                            "sample": sample},
           "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------ GPU side

def run_linear(args, rank, world):
    import torch
    import torch.distributed as dist

    import saccade_core as sc

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    calls = stack_spec(args.layers, args.tokens, args.route_frac, seed=1234 + rank)
    ops, xs, step_bytes, big = [], [], 0, []
    check_src = []
    x_of = {}  # (layer, input) -> activations shared by the calls that read them
    for li, name, n, k, boosted in calls:
        packed = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=torch.int32, device=dev, generator=gen)
        scale = ((0.02 * (3.0 + torch.rand(n, device=dev, generator=gen))) / 7.0).to(torch.float16)
        nnz = int(round(n * k * args.fill))
        flat = torch.randperm(n * k, device=dev, generator=gen)[:nnz].sort().values if n * k < 2 ** 27 else \
            torch.unique(torch.randint(0, n * k, (int(nnz * 1.02) + 16,), device=dev, generator=gen))[:nnz]
        rows, cols = flat // k, flat % k
        rp = torch.zeros(n + 1, dtype=torch.int64, device=dev)
        rp[1:] = torch.cumsum(torch.bincount(rows, minlength=n), 0)
        vals = torch.randint(-127, 128, (flat.numel(),), dtype=torch.int8, device=dev, generator=gen).view(torch.uint8)
        sp = sc.SparseDeltaMatrix(rp.to(torch.int32), cols.to(torch.int32), vals,
                                  torch.tensor([0.006 / 127.0], dtype=torch.float16))
        op = sc.SaccadeLinearOp(packed, scale, sp, sc.SaccadeConfig(T4_BOOSTED, T8_NEVER), n, k, device=dev,
                                mode=args.mode)
        if li == 0 and rank == 0:  # reference-format buffers of the first layer, for the parity check
            check_src.append((len(ops), packed.cpu(), scale.cpu(), rp.to(torch.int32).cpu(), cols.to(torch.int32).cpu(),
                              vals.cpu()))
        del packed, scale, flat, rows, cols, rp, vals
        key = (li, INPUT_OF[name])
        if key not in x_of:
            x = torch.randn((args.tokens, k), device=dev, generator=gen)
            for t in boosted:
                x[t] *= 8.0
            x_of[key] = x.to(torch.float16)
        x = x_of[key]
        b = call_bytes(n, k, args.tokens, op.delta_nnz, len(boosted) > 0)
        ops.append(op)
        xs.append(x)
        step_bytes += b
        if name in ("gate", "up", "down"):
            big.append((len(ops) - 1, b))
    torch.cuda.synchronize()

    ys = [None] * len(ops)
    # launches of one step: a group per input shared by several projections (q,k,v and gate,up),
    # unless --no-group asks for one call per projection (the reference's calling pattern)
    units = []  # (op indices, group or None)
    i = 0
    while i < len(ops):
        j = i
        while j + 1 < len(ops) and calls[j + 1][0] == calls[i][0] and \
                INPUT_OF[calls[j + 1][1]] == INPUT_OF[calls[i][1]]:
            j += 1
        idx = list(range(i, j + 1))
        if len(idx) > 1 and not args.no_group:
            units.append((idx, sc.SaccadeLinearGroup([ops[t] for t in idx])))
        else:
            units.extend(([t], None) for t in idx)
        i = j + 1

    def run_unit(idx, grp, outs=None):
        x = xs[idx[0]]
        if grp is None:
            return [ops[idx[0]].forward(x, out=None if outs is None else outs[0])]
        return grp.forward(x, outs=outs)

    def step():
        for idx, grp in units:
            for t, y in zip(idx, run_unit(idx, grp)):
                ys[t] = y

    big_set = {i for i, _ in big}
    big_units = [(idx, grp) for idx, grp in units if idx[0] in big_set]

    def big_step():
        for idx, grp in big_units:
            for t, y in zip(idx, run_unit(idx, grp)):
                ys[t] = y

    g_step = sc.CapturedStep(step, dev)
    g_big = sc.CapturedStep(big_step, dev)

    # end to end through the public API: every call's input from one pinned host buffer (one
    # host->device copy), every output into one device buffer read back by one device->host copy
    first_of = {}
    for t, x in enumerate(xs):
        first_of.setdefault(id(x), t)
    uniq = sorted(first_of.values())
    xsz = [xs[t].numel() for t in uniq]
    ysz = [args.tokens * op.out_features for op in ops]
    x_host = torch.cat([xs[t].reshape(-1) for t in uniq]).cpu().pin_memory()
    y_host = torch.empty(sum(ysz), dtype=torch.float16).pin_memory()
    x_dev = torch.empty_like(x_host, device=dev)
    y_dev = torch.empty(sum(ysz), dtype=torch.float16, device=dev)
    x_views_u = dict(zip(uniq, torch.split(x_dev, xsz)))
    x_views = [x_views_u[first_of[id(x)]] for x in xs]
    y_views = list(torch.split(y_dev, ysz))

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        for idx, grp in units:
            x = x_views[idx[0]].view(args.tokens, ops[idx[0]].in_features)
            outs = [y_views[t].view(args.tokens, ops[t].out_features) for t in idx]
            if grp is None:
                ops[idx[0]].forward(x, out=outs[0])
            else:
                grp.forward(x, outs=outs)
        y_host.copy_(y_dev, non_blocking=True)

    g_e2e = sc.CapturedStep(e2e_step, dev)
    h2d = x_host.numel() * 2
    d2h = y_host.numel() * 2

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(graph, steps, sync_each=False):
        for _ in range(args.warmup):
            graph.replay()
        graph.synchronize()
        barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(graph.stream):
            s.record()
            for _ in range(steps):
                graph.replay()
                if sync_each:
                    graph.synchronize()
            e.record()
        graph.synchronize()
        barrier()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / steps
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    clocks = ClockSampler(dev)
    clocks.start()
    ms = timed(g_step, args.steps)
    clk = clocks.stop()
    ms_big = timed(g_big, args.steps)
    ms_e2e = timed(g_e2e, args.steps, sync_each=True)

    # correctness guard on the timed configuration: no device-side error recorded, and the first
    # layer's seven outputs of the last timed step equal the oracle's on a sample of rows
    for op in ops[:7]:
        op.check_device()
    parity = check_against_oracle(check_src, ops, xs, ys, calls) if rank == 0 else None

    # bytes of one step over all ranks (their routed tokens, hence their dW bytes, differ)
    total_bytes = float(step_bytes)
    if world > 1:
        tb = torch.tensor([total_bytes], device=dev, dtype=torch.float64)
        dist.all_reduce(tb, op=dist.ReduceOp.SUM)
        total_bytes = float(tb.item())
    value = total_bytes / (ms / 1e3) / 1e9
    big_bytes = sum(b for _, b in big)
    achieved = big_bytes / (ms_big / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    # DRAM traffic of the dominant launch from the committed ncu capture (profiles/): the gate+up
    # group of one layer; reported with that launch's algorithmic bytes for comparison
    traffic = traffic_alg = None
    tp = os.path.join(ROOT, "profiles", "decode_fused_traffic.json")
    if os.path.exists(tp):
        try:
            tj = json.load(open(tp))
            traffic, traffic_alg = tj.get("dram_bytes_per_launch"), tj.get("algorithmic_bytes_per_launch")
        except ValueError:
            pass
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {**workload_config(args, calls, step_bytes), "mode": args.mode,
                   "l2": "inputs > L2 (3.3 GB of weights)",
                   "parallelism": f"replicas{world}", "graph": "one CUDA graph per step",
                   "launch_units": "q,k,v and gate,up grouped (sc_forward_group)" if not args.no_group
                   else "one launch per projection", "launches_per_step": launches_per_step(args, units)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "traffic_note": None if traffic is None else
                     f"ncu DRAM bytes of one gate+up group launch (algorithmic {traffic_alg})",
                     "kernel": launch_kind(args) + f" on the gate/up/down calls ({len(big_units)} launches per step)",
                     "peak_kind": f"{peak_kind} hbm copy"},
        "clocks": clk,
        "e2e": {"value": round(total_bytes / (ms_e2e / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "how": f"one pinned host->device copy of all inputs, the {len(ops)} calls, one device->host copy "
                       "of all outputs; captured step, host sync each step"},
        "gpu_launches": launches_per_step(args, units) * args.steps,
        "parity_check": parity,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(args)
    if rank == 0:
        print(json.dumps(out), flush=True)


# ------------------------------------------------------------------ Qwen2-7B decode

DECODE_PROJ = ("q", "k", "v", "o", "gate", "up", "down")


def decode_metric(args):
    return f"{DECODE_MODELS[args.model][0]} decode tok/s"


def route_pct(args):
    """Percentiles of the calibration scores where t4 and t8 sit."""
    p = args.route_pct
    return p, (0.95 if p < 0.9 else 0.99)


def decode_config(args, world):
    p4, p8 = route_pct(args)
    return {"workload": f"{args.model} batched greedy decode",
            "model": f"{args.model} (random init, every linear C-TARQ)",
            "layers": args.layers, "global_batch": args.batch, "prompt_tokens": args.prompt,
            "decode_steps": args.decode_steps, "dw_fill": args.fill,
            "thresholds": f"per projection at the {p4 * 100:g}th / {p8 * 100:g}th percentile of a "
                          f"{args.prompt}-token calibration prompt",
            "parallelism": f"tp{world}" if world > 1 else "tp1", "fused_route": args.fused_route}


def decode_step_bytes(cfg, model, batch, pos):
    """Algorithmic HBM bytes of one decode step on one rank at cache length `pos`: every C-TARQ call
    (call_bytes, dW counted: some of the 64 tokens route in every call), the lm_head slice (f16),
    the KV cache read (f32 K and V of `pos` keys per sequence and KV head) and written."""
    total = 0
    for L in model.layers:
        for name in DECODE_PROJ:
            op = L[name]
            total += call_bytes(op.out_features, op.in_features, batch, op.delta_nnz, True)
    total += (model.v1 - model.v0) * cfg.hidden * 2
    total += len(model.layers) * batch * model.nkv * cfg.head_dim * 4 * 2 * (pos + 1)
    return total


def build_decode(args, rank, world, dev, group):
    import torch

    from saccade_core import qwen2 as Q
    cfg = (Q.Qwen2Config.qwen2_72b if args.model == "qwen2-72b" else Q.Qwen2Config.qwen2_7b)(layers=args.layers)
    ck = Q.random_checkpoint(cfg, seed=42, fill=args.fill, device=dev)
    g = torch.Generator()
    g.manual_seed(7)
    calib = torch.randint(0, cfg.vocab, (1, args.prompt), generator=g)
    Q.calibrate(ck, calib.to(dev), pct=route_pct(args), device=dev, max_pos=args.prompt)
    if world > 1:  # every rank calibrates the same model; rank 0's thresholds are the ones used
        import torch.distributed as dist
        th = torch.tensor([ck.thresholds[li][n] for li in range(len(ck.blocks)) for n in DECODE_PROJ],
                          dtype=torch.float32, device=dev)
        dist.broadcast(th, 0, group=group)
        th = th.cpu().numpy().reshape(len(ck.blocks), len(DECODE_PROJ), 2)
        for li in range(len(ck.blocks)):
            for j, n in enumerate(DECODE_PROJ):
                ck.thresholds[li][n] = (float(th[li, j, 0]), float(th[li, j, 1]))
    need = 1 + 2 * (args.warmup + args.steps) + 3
    max_pos = args.prompt + max(args.decode_steps, need)
    model = Q.Qwen2Model(ck, dev, max_batch=args.batch, max_pos=max_pos, mode=args.mode,
                         tp=(rank, world, group) if world > 1 else None, fused_route=args.fused_route)
    # reference-format buffers of the last layer's gate and up for the parity check, then free the rest
    last = {n: {k: v.cpu() for k, v in ck.blocks[-1][n].items()} for n in ("gate", "up")}
    last_thr = {n: ck.thresholds[-1][n] for n in ("gate", "up")}
    del ck
    torch.cuda.empty_cache()
    return cfg, model, last, last_thr


def check_decode_against_oracle(model, last, last_thr, batch, rows_per_call=128):
    """The last layer's gate and up outputs of the last step (this rank's rows) against the oracle on
    the same input rows (fast-mode tolerance 1e-3 * RMS + one f16 ulp; router masks identical)."""
    import torch

    from oracle import oracle as O
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from qwen2_cases import to_compressed
    cfg = model.cfg
    x16 = model._bufs[("x16", batch)]
    outs = {"gate": model._bufs[("g16", batch)], "up": model._bufs[("u16", batch)]}
    xb = x16.cpu().numpy().view(np.uint16)
    worst = 0.0
    for name in ("gate", "up"):
        full = to_compressed(last[name], cfg.intermediate, cfg.hidden)
        rng = np.random.default_rng(5)
        local = np.sort(rng.choice(model.i1 - model.i0, size=min(rows_per_call, model.i1 - model.i0), replace=False))
        rows = local + model.i0
        rp = full.delta_row_ptrs.astype(np.int64)
        sel = [np.arange(rp[r], rp[r + 1]) for r in rows]
        ent = np.concatenate(sel) if sel else np.zeros(0, np.int64)
        ptrs = np.concatenate([[0], np.cumsum([len(e) for e in sel])]).astype(np.uint32)
        c = O.Compressed(np.ascontiguousarray(full.packed_base[rows]), np.ascontiguousarray(full.scale_base[rows]),
                         ptrs, full.delta_col_indices[ent].copy(), full.delta_values[ent].copy(), full.delta_scale,
                         len(rows), cfg.hidden)
        yr, routed, _ = O.OracleLinear(c, *last_thr[name]).forward(xb)
        yg = outs[name].cpu().numpy().view(np.uint16)[:, local]
        a, b = yg.view(np.float16).astype(np.float32), yr.view(np.float16).astype(np.float32)
        rms = float(np.sqrt(np.mean(b.astype(np.float64) ** 2)))
        tol = 1e-3 * rms + np.spacing(np.abs(b).astype(np.float16)).astype(np.float32)
        ratio = float(np.max(np.abs(a - b) / tol))
        worst = max(worst, ratio)
        if ratio > 1.0:
            raise AssertionError(f"bench parity: last layer {name} differs from the oracle ({ratio:.3f} of tolerance)")
    return {"calls": "last layer gate and up of the last timed step", "rows_per_call": rows_per_call,
            "routed_tokens": int(np.count_nonzero(routed)), "max_err_over_tol": round(worst, 4),
            "tolerance": "1e-3 * RMS(ref) + 1 f16 ulp", "ok": True}


def run_decode(args, rank, world):
    import torch
    import torch.distributed as dist

    import saccade_core as sc
    from saccade_core import qwen2 as Q
    from saccade_core._lib import LIB

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    group = dist.group.WORLD if world > 1 else None
    t_setup = time.perf_counter()
    cfg, model, last, last_thr = build_decode(args, rank, world, dev, group)
    B, S = args.batch, args.prompt
    g = torch.Generator()
    g.manual_seed(11)
    prompts = torch.randint(0, cfg.vocab, (B, S), generator=g)
    dec = Q.GreedyDecoder(model, B)
    prompts = prompts.to(dev)
    pf0, pf1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(dec.stream):
        pf0.record()
        dec.prefill(prompts, chunk=args.prefill_chunk)
        pf1.record()
    dec.stream.synchronize()
    prefill_ms_rank = pf0.elapsed_time(pf1)
    dec.capture()
    setup_s = time.perf_counter() - t_setup

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # the timed region: K back-to-back step graphs (each feeds its argmax to the next)
    for _ in range(args.warmup):
        dec.step()
    dec.stream.synchronize()
    barrier()
    torch.cuda.synchronize()
    pos0 = int(dec.pos[0].item())
    clocks = ClockSampler(dev)
    clocks.start()
    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("decode_steps")
    with torch.cuda.stream(dec.stream):
        s_ev.record()
        for _ in range(args.steps):
            dec.graph.replay()
        e_ev.record()
    torch.cuda.nvtx.range_pop()
    dec.stream.synchronize()
    clk = clocks.stop()
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(s_ev.elapsed_time(e_ev) / args.steps)
    prefill_ms = max_over_ranks(prefill_ms_rank)

    # end to end: token ids from pinned host memory in, next ids to pinned host memory out, every step
    ids_host = torch.empty(B, dtype=torch.int64).pin_memory()
    out_host = torch.empty(B, dtype=torch.int64).pin_memory()
    ids_host.copy_(dec.next.cpu())
    e2e_steps = args.steps

    def e2e_step():
        nxt = dec.step(ids_host)
        with torch.cuda.stream(dec.stream):
            out_host.copy_(nxt, non_blocking=True)
        dec.stream.synchronize()
        ids_host.copy_(out_host)

    for _ in range(2):
        e2e_step()
    barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(dec.stream)
    for _ in range(e2e_steps):
        e2e_step()
    e2.record(dec.stream)
    dec.stream.synchronize()
    barrier()
    ms_e2e = max_over_ranks(s2.elapsed_time(e2) / e2e_steps)
    model.check_device()
    undecided = model.undecided_routes()
    parity = check_decode_against_oracle(model, last, last_thr, B) if rank == 0 else None

    # the dominant kernel: each layer's gate+up call (one grouped C-TARQ launch unit) at M = 64 on
    # the last step's post-attention normed state, replayed over all layers (weights >> L2)
    x16 = model._bufs[("x16", B)]
    gbuf, ubuf = model._bufs[("g16", B)].clone(), model._bufs[("u16", B)].clone()

    def gateup_all():
        for L in model.layers:
            L["gateup"].forward(x16, outs=[gbuf, ubuf])

    n0 = int(LIB.sc_launch_count())
    cap = sc.CapturedStep(gateup_all, dev)  # one eager call, one captured
    gu_launches = (int(LIB.sc_launch_count()) - n0) // (2 * len(model.layers))
    for _ in range(3):
        cap.replay()
    cap.synchronize()
    reps = 10
    s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(cap.stream):
        s3.record()
        for _ in range(reps):
            cap.replay()
        e3.record()
    cap.synchronize()
    us_gu = s3.elapsed_time(e3) * 1e3 / (reps * len(model.layers))
    gu_bytes = sum(call_bytes(L[n].out_features, L[n].in_features, B, L[n].delta_nnz, True)
                   for n in ("gate", "up") for L in model.layers[:1])
    achieved = gu_bytes / (us_gu * 1e-6) / 1e9
    peak, peak_kind = measured_peak()

    pos_mid = pos0 + args.steps // 2
    step_bytes = decode_step_bytes(cfg, model, B, pos_mid)
    total_bytes = step_bytes
    if world > 1:
        tb = torch.tensor([float(step_bytes)], device=dev, dtype=torch.float64)
        dist.all_reduce(tb, op=dist.ReduceOp.SUM)
        total_bytes = float(tb.item())
    value = B / (ms / 1e3)
    traffic = None
    tp = os.path.join(ROOT, "profiles", "decode_gateup_m64_traffic.json")
    if args.model == "qwen2-7b" and B == 64 and os.path.exists(tp):  # the capture's workload
        try:
            traffic = json.load(open(tp)).get("dram_bytes_per_launch_unit")
        except ValueError:
            pass
    out = {
        "metric": decode_metric(args), "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (random-init weights, random prompt ids)",
        "config": {**decode_config(args, world), "mode": args.mode, "positions_timed": [pos0, pos0 + args.steps],
                   "l2": "inputs > L2 (weights and KV cache of one step far above 126 MB)",
                   "graph": "one CUDA graph per decode step",
                   "collectives_per_step": (2 * len(model.layers) + 1) if world > 1 else 0,
                   "bytes_per_step_all_ranks": int(total_bytes),
                   "step_hbm_frac": round(total_bytes / world / (ms / 1e3) / 1e9 / peak, 4),
                   "setup_s": round(setup_s, 1)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "kernel": f"gate+up C-TARQ call unit at M={B} ({gu_launches} launches: "
                               + ("k_mid_route, then k_ctarq_mid (tcgen05, routed tokens' dW folded into a second A)"
                                  if 9 <= B <= 64 else
                                  "the router-fused decode kernel, gate and up in one launch" if B <= 8 else
                                  "router, token gather, prefill tcgen05 GEMM")
                               + f"), {us_gu:.1f} us per layer, {gu_bytes} algorithmic bytes",
                     "peak_kind": f"{peak_kind} hbm copy"},
        "clocks": clk,
        "e2e": {"value": round(B / (ms_e2e / 1e3), 1), "unit": "tok/s", "h2d_bytes_per_step": B * 8,
                "d2h_bytes_per_step": B * 8,
                "how": "per step: token ids from pinned host memory, the step graph, next ids to pinned host "
                       "memory, host synchronisation"},
        "prefill": {"tokens": B * S, "ms": round(prefill_ms, 2), "tok_s": round(B * S / (prefill_ms / 1e3), 1),
                    "sequences_per_pass": args.prefill_chunk,
                    "how": "device time of the process's first prefill (CUDA events, max over ranks): includes "
                           "workspace allocation and one-time kernel setup"},
        "gpu_launches": dec.launches_per_step * args.steps,
        "undecided_split_routes": undecided,
        "parity_check": parity,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline_decode(args)
    if rank == 0:
        print(json.dumps(out), flush=True)


def decode_layer_items(args, tokens):
    """One decoder layer's seven linears of the model on the oracle (synthetic reference-format
    weights), `tokens` tokens with a seeded 25 % boosted over the router threshold."""
    calls = stack_spec(1, tokens, args.route_frac, seed=4321, proj=model_proj(args.model))
    return build_oracle_stack(calls, args.fill, 98, tokens)


def cpu_decode_rate(args, seconds):
    from oracle import oracle as O
    try:
        O.lib(native=True)
        native = True
    except Exception:  # noqa: BLE001
        native = False
    items = decode_layer_items(args, 1)
    _, dt1 = time_oracle(items, 1, native)
    reps = max(1, int(seconds / max(dt1, 1e-4)))
    _, dt = time_oracle(items, reps, native)
    per_layer = dt / reps
    return 1.0 / (per_layer * args.layers), reps, dt, native


def cpu_baseline_decode(args):
    """The oracle's op.rs restatement on the host cores, per layer (the seven linears of one decoder
    layer, one token), scaled to the model's layers: tokens per second of the linears alone."""
    rate, reps, dt, native = cpu_decode_rate(args, args.cpu_seconds)
    label = DECODE_MODELS[args.model][0]
    return {"value": round(rate, 3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"1 {label} decoder layer (7 C-TARQ linears, 1 token) x {reps} reps in {dt:.1f} s, scaled "
                      f"x{args.layers} layers (linears only: no attention, norms or lm_head); C restatement of op.rs, "
                      f"OpenMP over rows ({'-march=native' if native else 'x86-64-v3'})"}


def run_reference_decode(args, rank):
    """--impl reference: the reference's CPU algorithm for the decode step's linears (the oracle's
    op.rs restatement; the Rust reference cannot be built here), per layer, scaled to the model's layers."""
    if rank != 0:
        return
    from oracle import oracle as O
    try:
        O.lib(native=True)
        native = True
    except Exception:  # noqa: BLE001
        native = False
    items = decode_layer_items(args, 1)
    _, dt1 = time_oracle(items, 1, native)
    budget = min(150.0, 10.0 * args.cpu_seconds) / max(1, args.steps + args.warmup)  # seconds per step
    reps = max(1, int(budget / max(dt1, 1e-4)))
    for _ in range(args.warmup):
        time_oracle(items, reps, native)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        time_oracle(items, reps, native)
    dt = time.perf_counter() - t0
    per_layer = dt / (args.steps * reps)
    value = 1.0 / (per_layer * args.layers)
    sample = (f"each step: 1 {DECODE_MODELS[args.model][0]} decoder layer (7 C-TARQ linears, 1 token) x {reps}, "
              f"scaled x{args.layers} layers "
              f"(linears only); C restatement of op.rs (Rust reference not buildable here), OpenMP over rows")
    out = {"metric": decode_metric(args), "value": round(value, 3), "unit": "tok/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_layer * args.layers * 1e3, 3),
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
           "data": "synthetic", "config": decode_config(args, args.gpus), "impl": "reference",
           "cpu_baseline": {"value": round(value, 3), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                            "sample": sample},
           "e2e": {"value": round(value, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def check_against_oracle(check_src, ops, xs, ys, calls, rows_per_call=96):
    """Compares sampled output rows of the given calls with the oracle on the same inputs (fast-mode
    tolerance: 1e-3 * RMS + one f16 ulp, router masks identical).  Raises on a mismatch."""
    import torch

    from oracle import oracle as O
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    worst = 0.0
    for idx, packed, scale, rp, cols, vals in check_src:
        n, k = ops[idx].out_features, ops[idx].in_features
        rng = np.random.default_rng(idx)
        rows = np.sort(rng.choice(n, size=min(rows_per_call, n), replace=False))
        rpn = rp.numpy().astype(np.int64)
        sel = [np.arange(rpn[r], rpn[r + 1]) for r in rows]
        ent = np.concatenate(sel) if sel else np.zeros(0, np.int64)
        ptrs = np.concatenate([[0], np.cumsum([len(e) for e in sel])]).astype(np.uint32)
        c = O.Compressed(np.ascontiguousarray(packed.numpy().view(np.uint32)[rows]),
                         np.ascontiguousarray(scale.numpy().view(np.uint16)[rows]), ptrs,
                         cols.numpy().view(np.uint32)[ent].copy(), vals.numpy()[ent].copy(),
                         int(np.array([0.006 / 127.0], dtype=np.float16).view(np.uint16)[0]), len(rows), k)
        xb = xs[idx].cpu().numpy().view(np.uint16)
        yr, _, _ = O.OracleLinear(c, T4_BOOSTED, T8_NEVER).forward(xb)
        yg = ys[idx].cpu().numpy().view(np.uint16)[:, rows]
        a, b = yg.view(np.float16).astype(np.float32), yr.view(np.float16).astype(np.float32)
        rms = float(np.sqrt(np.mean(b.astype(np.float64) ** 2)))
        tol = 1e-3 * rms + np.spacing(np.abs(b).astype(np.float16)).astype(np.float32)
        ratio = float(np.max(np.abs(a - b) / tol))
        worst = max(worst, ratio)
        if ratio > 1.0:
            raise AssertionError(f"bench parity: call {calls[idx][:4]} differs from the oracle "
                                 f"(max error / tolerance {ratio:.3f})")
    return {"calls": len(check_src), "rows_per_call": rows_per_call, "max_err_over_tol": round(worst, 4),
            "tolerance": "1e-3 * RMS(ref) + 1 f16 ulp", "ok": True}


SWEEP_SHAPES = [("q/o", 3584, 3584), ("k/v", 512, 3584), ("gate/up", 18944, 3584), ("down", 3584, 18944)]
SWEEP_TOKENS = [1, 4, 16, 64, 256, 1024, 4096]
SWEEP_ROUTED = [0.0, 0.10, 0.25, 1.0]
SWEEP_POOL_BYTES = 512 * 2 ** 20  # round-robin over >= 4x L2 of distinct layers


def run_sweep(args):
    """Single-call times over dW densities x shapes x tokens x routed fractions: every point replays a
    CUDA graph of one call on each layer of a pool of distinct copies of the layer (>= 512 MB of
    weights, so each call reads its weights from HBM), and reports the algorithmic bytes and
    flops per call against the measured HBM and bf16 peaks."""
    import torch

    import saccade_core as sc

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    hbm, _ = measured_peak()
    tc = 1617.5
    try:
        tc = float(json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["bf16_tflops"])
    except (OSError, ValueError, KeyError):
        pass
    fills = [float(v) for v in args.sweep_fills.split(",")] if args.sweep_fills else [args.fill]
    tokens = [int(v) for v in args.sweep_tokens.split(",")] if args.sweep_tokens else SWEEP_TOKENS
    shapes = [sh for sh in SWEEP_SHAPES if not args.sweep_shapes or sh[0] in args.sweep_shapes.split(",")]
    routed = [float(v) for v in args.sweep_routed.split(",")] if args.sweep_routed else SWEEP_ROUTED
    rows = []
    for fill, (label, n, k) in [(f, sh) for f in fills for sh in shapes]:
        packed = torch.randint(-2 ** 31, 2 ** 31 - 1, (n, k // 8), dtype=torch.int32, device=dev, generator=gen)
        scale = ((0.02 * (3.0 + torch.rand(n, device=dev, generator=gen))) / 7.0).to(torch.float16)
        nnz = int(round(n * k * fill))
        flat = torch.unique(torch.randint(0, n * k, (int(nnz * 1.02) + 16,), device=dev, generator=gen))[:nnz]
        rr, cc = flat // k, flat % k
        rp = torch.zeros(n + 1, dtype=torch.int64, device=dev)
        rp[1:] = torch.cumsum(torch.bincount(rr, minlength=n), 0)
        vals = torch.randint(-127, 128, (flat.numel(),), dtype=torch.int8, device=dev, generator=gen).view(torch.uint8)
        sp = sc.SparseDeltaMatrix(rp.to(torch.int32), cc.to(torch.int32), vals,
                                  torch.tensor([0.006 / 127.0], dtype=torch.float16))
        wbytes = n * k // 2
        pool = max(4, min(1024, -(-SWEEP_POOL_BYTES // wbytes)))
        ops = [sc.SaccadeLinearOp(packed, scale, sp, sc.SaccadeConfig(T4_BOOSTED, T8_NEVER), n, k, device=dev,
                                  mode=args.mode) for _ in range(pool)]
        real_nnz = ops[0].delta_nnz
        del packed, scale, flat, rr, cc, rp, vals, sp
        for m in tokens:
            y = torch.empty((m, n), dtype=torch.float16, device=dev)
            for frac in routed:
                r = int(round(frac * m))
                x = torch.randn((m, k), device=dev, generator=gen)
                if r:
                    x[torch.randperm(m, device=dev, generator=gen)[:r]] *= 8.0
                x = x.to(torch.float16)

                def one_pass():
                    for op in ops:
                        op.forward(x, out=y)

                g = sc.CapturedStep(one_pass, dev)
                for _ in range(2):
                    g.replay()
                g.synchronize()
                reps = 1
                while True:
                    s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    with torch.cuda.stream(g.stream):
                        s_ev.record()
                        for _ in range(reps):
                            g.replay()
                        e_ev.record()
                    g.synchronize()
                    ms = s_ev.elapsed_time(e_ev)
                    if ms >= 20.0 or reps >= 64:
                        break
                    reps *= 4
                us = ms * 1e3 / (reps * pool)
                ops[0].check_device()
                b = call_bytes(n, k, m, real_nnz, r > 0)
                fl = 2.0 * m * n * k + 2.0 * real_nnz * r
                t_hbm, t_tc = b / (hbm * 1e3), fl / (tc * 1e6)  # microseconds
                rows.append((fill, label, n, k, m, frac, us, b / us / 1e3, fl / us / 1e6,
                             "hbm" if t_hbm >= t_tc else "tensor", max(t_hbm, t_tc) / us, pool))
                del g
            del y
        del ops
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
    with open(args.sweep, "w") as f:
        f.write(f"# C-TARQ linear: single-call sweep ({args.mode} mode, f16 x)\n\n")
        f.write("Command: `python bench.py --sweep " + args.sweep + (f" --mode {args.mode}" if args.mode != "fast" else "")
                + (f" --sweep-fills {args.sweep_fills}" if args.sweep_fills else "")
                + (f" --sweep-tokens {args.sweep_tokens}" if args.sweep_tokens else "")
                + (f" --sweep-shapes {args.sweep_shapes}" if args.sweep_shapes else "")
                + (f" --sweep-routed {args.sweep_routed}" if args.sweep_routed else "")
                + (f" --fill {args.fill}" if not args.sweep_fills and args.fill != 0.01 else "") + "`\n\n")
        f.write(f"Peaks: HBM {hbm} GB/s, bf16 dense {tc} TFLOP/s (MEASURED_PEAKS.json). `bound` is the larger of "
                "bytes/HBM and flops/tensor; `frac` = that bound time / measured time. Routed = fraction of "
                "the tokens boosted x8 (their variance clears t4 = 8). Each point replays one call on every "
                "layer of a pool of distinct copies (>= 512 MB of weights).\n\n")
        f.write("| dW | shape | N x K | M | routed | us / call | GB/s | TFLOP/s | bound | frac | pool |\n")
        f.write("|---|---|---|---|---|---|---|---|---|---|---|\n")
        for (fill, label, n, k, m, frac, us, gbs, tfl, bound, fr, pool) in rows:
            f.write(f"| {fill:.1%} | {label} | {n}x{k} | {m} | {frac:.0%} | {us:.2f} | {gbs:.0f} | {tfl:.1f} | "
                    f"{bound} | {fr:.3f} | {pool} |\n")
    print(json.dumps({"sweep": args.sweep, "points": len(rows)}), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.sweep:
        if rank == 0:
            run_sweep(args)
        return
    if args.impl == "reference":
        if args.workload == "decode":
            run_reference_decode(args, rank)
        else:
            run_reference_linear(args, rank)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    try:
        if args.workload == "decode":
            run_decode(args, rank, world)
        else:
            run_linear(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
