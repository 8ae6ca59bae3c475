#!/usr/bin/env python
"""Generates the golden fixtures of tests/test_golden.py from the C oracle.

The Rust reference cannot be built here and ships no golden vectors, so these fixtures pin the
oracle itself (and through it the CUDA library): any change to the restated arithmetic of
compress.rs, calibration.rs, heuristics.rs or op.rs shows up as a fixture mismatch.

  python tests/golden/make_golden.py     # rewrites tests/golden/*.npz and digests.json

Small cases store every array (packed buffers, activations, outputs; the f32 weights too when
they are small).  The
single-layer configuration (4864 x 896, 16 tokens, 1 % dW) and the Qwen2-7B q/o shape at one
token are stored as SHA-256 digests of their arrays; the test regenerates them from the seed.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))           # tests/
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))  # repo root

from ctarq_cases import make_case  # noqa: E402

SMALL = [
    # name, n, k, m, fill, seed, boost
    ("ragged_33x136_m9", 33, 136, 9, 0.10, 101, [2, 5]),
    ("k8_256x8_m3", 256, 8, 3, 0.30, 102, [1]),
    ("tile_160x192_m8", 160, 192, 8, 0.05, 103, [0, 7]),
]
DIGEST = [
    # name, n, k, m, fill, seed, boost
    ("config0_4864x896_m16", 4864, 896, 16, 0.01, 42, [1, 6, 9, 14]),
    ("qwen2_7b_q_3584x3584_m1", 3584, 3584, 1, 0.01, 7, [0]),
]


def arrays(case):
    c = case.c
    y, routed, acc = case.oracle().forward(case.x_bits)
    return {
        "packed_base": c.packed_base, "scale_base": c.scale_base, "delta_row_ptrs": c.delta_row_ptrs,
        "delta_col_indices": c.delta_col_indices, "delta_values": c.delta_values,
        "delta_scale": np.array([c.delta_scale], dtype=np.uint16), "x_bits": case.x_bits,
        "thresholds": np.array([case.t4, case.t8], dtype=np.float32), "y_bits": y, "routed": routed, "acc": acc,
    }


def digest(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).hexdigest()


def main():
    meta = {"small": [], "digests": {}}
    for name, n, k, m, fill, seed, boost in SMALL:
        case = make_case(n, k, m, fill, seed=seed, boost=boost)
        arr = arrays(case)
        if n * k <= 10000:  # small enough to store the f32 weights too (compressor input)
            arr["w"] = case.w
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arr)
        meta["small"].append({"name": name, "n": n, "k": k, "m": m, "fill": fill, "seed": seed, "boost": boost,
                              "nnz": int(case.c.nnz)})
    for name, n, k, m, fill, seed, boost in DIGEST:
        case = make_case(n, k, m, fill, seed=seed, boost=boost)
        meta["digests"][name] = {"n": n, "k": k, "m": m, "fill": fill, "seed": seed, "boost": boost,
                                 "nnz": int(case.c.nnz),
                                 "sha256": {key: digest(v) for key, v in arrays(case).items()}}
    with open(os.path.join(HERE, "digests.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print("wrote", len(SMALL), "fixtures and", len(DIGEST), "digest sets")


if __name__ == "__main__":
    main()
