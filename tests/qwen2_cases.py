"""Shared helpers of the Qwen2 model tests: a GPU checkpoint as CPU oracle ops."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O
from oracle import qwen2_oracle as QO


def to_compressed(blocks: dict, n: int, k: int) -> O.Compressed:
    """A compress_tensor_to_saccade() dict (device tensors) as the oracle's reference-format buffers."""
    def u32(t):
        return np.ascontiguousarray(t.view(torch.int32).cpu().numpy().view(np.uint32))

    packed = u32(blocks["packed_base"]).reshape(n, k // 8)
    scale = blocks["scale_base"].cpu().numpy().view(np.uint16)
    if "delta_row_ptrs" in blocks:
        rp = u32(blocks["delta_row_ptrs"])
        ci = u32(blocks["delta_col_indices"])
        cv = blocks["delta_values"].cpu().numpy().astype(np.uint8)
        ds = int(blocks["delta_scale"].view(torch.int16).item()) & 0xFFFF
    else:
        rp, ci, cv, ds = np.zeros(n + 1, np.uint32), np.zeros(0, np.uint32), np.zeros(0, np.uint8), 0
    return O.Compressed(packed, scale, rp, ci, cv, ds, n, k)


def oracle_model(ck, max_pos: int) -> QO.Qwen2Oracle:
    """The checkpoint's model on the CPU oracle (thresholds and every buffer copied from the GPU)."""
    from saccade_core.qwen2 import PROJ, rope_tables
    cfg = ck.cfg
    layers = []
    for li, lb in enumerate(ck.blocks):
        L = {}
        for name in PROJ:
            n, k = cfg.proj_shape(name)
            t4, t8 = ck.thresholds[li][name]
            L[name] = O.OracleLinear(to_compressed(lb[name], n, k), t4, t8)
        L["bias"] = {name: ck.biases[li][name].float().cpu().numpy() for name in ("q", "k", "v")}
        L["norm_in"] = ck.norms[li]["input"].float().cpu().numpy()
        L["norm_post"] = ck.norms[li]["post"].float().cpu().numpy()
        layers.append(L)
    embed = ck.embed.float().cpu().numpy()
    lm = embed if ck.lm_head is None else ck.lm_head.float().cpu().numpy()
    cos, sin = rope_tables(cfg, max_pos)
    return QO.Qwen2Oracle(cfg, layers, ck.final_norm.float().cpu().numpy(), embed, lm, cos, sin)
