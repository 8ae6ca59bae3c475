"""bench.py on the CPU: the byte accounting of the metric, the workload both arms report, and the
reference arm (the oracle's C restatement of op.rs on the host cores) end to end."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402

REQUIRED = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
            "vs_baseline", "dtype", "data", "config", "impl", "cpu_baseline", "e2e"}


def test_call_bytes_worked_examples():
    # 2MK + NK/2 + 2N + [routed](3 nnz + 4(N+1)) + 2MN
    assert bench.call_bytes(4864, 896, 16, 43581, True) == 2523323       # single layer, 16 tokens, 1 % dW
    assert bench.call_bytes(18944, 3584, 1, 678953, True) == 36143231    # Qwen2-7B gate, one token
    assert bench.call_bytes(18944, 3584, 1, 678953, False) == 36143231 - 3 * 678953 - 4 * 18945


def test_decode_stack_workload():
    calls = bench.stack_spec(28, 1, 0.25, seed=1234)
    assert len(calls) == 196
    assert [c[1] for c in calls[:7]] == ["q", "k", "v", "o", "gate", "up", "down"]
    # calls that read the same activations route the same tokens
    for li in range(28):
        layer = [c for c in calls if c[0] == li]
        assert layer[0][4] == layer[1][4] == layer[2][4] and layer[4][4] == layer[5][4]


def _run(cmd, env=None):
    e = dict(os.environ)
    e.update(env or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py")] + cmd, capture_output=True, text=True,
                          timeout=600, env=e, cwd=ROOT)


def test_reference_arm_json_line():
    r = _run(["--workload", "linear", "--impl", "reference", "--steps", "2", "--warmup", "1", "--layers", "1"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    d = json.loads(lines[-1])
    assert REQUIRED <= set(d)
    assert d["impl"] == "reference" and d["unit"] == "GB/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 1
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    calls = bench.stack_spec(1, 1, 0.25, seed=1234)
    want = bench.workload_config(bench.parse(["--workload", "linear", "--layers", "1"]), calls,
                                 d["config"]["bytes_per_step"])
    assert d["config"] == want


def test_reference_arm_decode_json_line():
    """The default workload's reference arm: Qwen2-7B decode tok/s of the CPU algorithm, per layer."""
    r = _run(["--impl", "reference", "--steps", "2", "--warmup", "1", "--cpu-seconds", "0.3"])
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads([ln for ln in r.stdout.splitlines() if ln.strip()][-1])
    assert REQUIRED <= set(d)
    assert d["metric"] == "Qwen2-7B decode tok/s" and d["unit"] == "tok/s" and d["impl"] == "reference"
    assert d["value"] > 0 and d["steps"] == 2 and d["warmup"] == 1 and d["scaling"] == "strong"
    assert d["config"] == bench.decode_config(bench.parse([]), 1)
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "0", "--layers", "1"],
             env={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0 and r.stdout.strip() == ""


@pytest.mark.parametrize("flags", [["--sweep-fills", "0.005,0.04"], ["--sweep-tokens", "1,4"]])
def test_sweep_flags_parse(flags):
    a = bench.parse(["--sweep", "out.md"] + flags)
    assert a.sweep == "out.md"
    assert (a.sweep_fills or a.sweep_tokens)


def test_decode_model_options():
    """--model picks the architecture and its workload defaults; --route-pct places t4 (and t8)."""
    a = bench.parse(["--model", "qwen2-72b", "--route-pct", "0.5"])
    assert (a.layers, a.batch, a.prompt, a.decode_steps, a.prefill_chunk) == (80, 8, 2048, 128, 2)
    assert bench.decode_metric(a) == "Qwen2-72B decode tok/s"
    assert bench.route_pct(a) == (0.5, 0.95)
    assert bench.route_pct(bench.parse(["--route-pct", "0.9"])) == (0.9, 0.99)
    proj = {n: (N, K) for n, N, K in bench.model_proj("qwen2-72b")}
    assert proj == {"q": (8192, 8192), "k": (1024, 8192), "v": (1024, 8192), "o": (8192, 8192),
                    "gate": (29568, 8192), "up": (29568, 8192), "down": (8192, 29568)}
    assert bench.model_proj("qwen2-7b") == bench.PROJ
    d = bench.parse([])
    assert (d.model, d.layers, d.batch, d.prompt, d.decode_steps) == ("qwen2-7b", 28, 64, 512, 256)
    assert bench.parse(["--workload", "linear"]).layers == bench.LAYERS
