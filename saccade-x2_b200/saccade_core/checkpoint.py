"""Compiled checkpoints with the reference's key schema, in the safetensors container.

    read_safetensors / write_safetensors  the container: u64 little-endian header length, a JSON
                                          header {name: {dtype, shape, data_offsets}, optional
                                          "__metadata__"}, then the raw little-endian tensor bytes
    compile_mlp_checkpoint                saccade-runner/src/bin/compile.rs:158-205 (phase 4: the
                                          MLP projections become saccade_* keys, per-layer
                                          saccade_t4/t8, every other tensor copied unchanged)
    extract_scalar_f32                    saccade-core/src/engine.rs:14-19
    saccade_blocks                        saccade-runner/src/model.rs:470-492 (the keys one op reads)
    build_saccade_op                      saccade-runner/src/model.rs:470-495
    load_mlp / load_saccade_checkpoint    saccade-runner/src/model.rs:437-468 and 379-432 (the
                                          C-TARQ part: every layer's three MLP projections)

Keys (compress.rs:113-127 under the prefix `model.layers.{i}.mlp.{gate,up,down}_proj`):
`saccade_packed_base` u32 [N, K/8], `saccade_scale_base` f16 [N] and, when dW kept any
coordinate, `saccade_delta_row_ptrs` u32 [N+1], `saccade_delta_col_indices` u32 [nnz],
`saccade_delta_values` u8 [nnz], `saccade_delta_scale` f16 [1]; thresholds
`model.layers.{i}.saccade_t4` / `saccade_t8` f32 [1].  A layer is compressed when its
`down_proj.saccade_packed_base` exists (model.rs:438-439).

Reading is host-only (numpy copy-on-write maps of the file); building the ops copies the blocks
into the device layouts of libsaccade_ctarq.so.
"""
from __future__ import annotations

import json
import os
import struct
import sys
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np
import torch

# safetensors dtype tag -> (numpy storage dtype, torch dtype); BF16 is stored as u16 bits
_DTYPES = {
    "F64": (np.float64, torch.float64),
    "F32": (np.float32, torch.float32),
    "F16": (np.float16, torch.float16),
    "BF16": (np.uint16, torch.bfloat16),
    "I64": (np.int64, torch.int64),
    "I32": (np.int32, torch.int32),
    "I16": (np.int16, torch.int16),
    "I8": (np.int8, torch.int8),
    "U64": (np.uint64, torch.uint64),
    "U32": (np.uint32, torch.uint32),
    "U16": (np.uint16, torch.uint16),
    "U8": (np.uint8, torch.uint8),
    "BOOL": (np.bool_, torch.bool),
}
_TAGS = {tdt: tag for tag, (_, tdt) in _DTYPES.items()}

MLP_PROJS = ("gate_proj", "up_proj", "down_proj")  # compile.rs:158
BLOCK_SUFFIXES = ("packed_base", "scale_base", "delta_row_ptrs", "delta_col_indices", "delta_values", "delta_scale")
_MAX_HEADER = 100 * 1024 * 1024


def _check_le():
    if sys.byteorder != "little":
        raise RuntimeError("safetensors data is little-endian; this host is not")


def read_safetensors(path: str) -> Tuple[Dict[str, torch.Tensor], Dict[str, str]]:
    """All tensors of a safetensors file as CPU torch tensors (views of a copy-on-write map of the
    file where the offsets are aligned, copies otherwise) and the header's `__metadata__`.

    Raises ValueError for a malformed file: a header that is not JSON, an unknown dtype, a shape
    whose byte size differs from its offsets, or offsets outside the data or overlapping."""
    _check_le()
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: shorter than the 8-byte header length")
        (hlen,) = struct.unpack("<Q", head)
        if hlen > _MAX_HEADER or 8 + hlen > size:
            raise ValueError(f"{path}: header length {hlen} exceeds the file")
        try:
            header = json.loads(f.read(hlen).decode("utf-8"))
        except (UnicodeDecodeError, json.JSONDecodeError) as e:
            raise ValueError(f"{path}: header is not JSON ({e})") from None
    if not isinstance(header, dict):
        raise ValueError(f"{path}: header is not a JSON object")
    meta = header.pop("__metadata__", None) or {}
    if not isinstance(meta, dict):
        raise ValueError(f"{path}: __metadata__ is not an object")
    base = 8 + hlen
    nbytes = size - base
    spans = []
    for name, ent in header.items():
        if not isinstance(ent, dict) or set(ent) != {"dtype", "shape", "data_offsets"}:
            raise ValueError(f"{path}: entry {name!r} needs exactly dtype, shape and data_offsets")
        tag = ent["dtype"]
        if tag not in _DTYPES:
            raise ValueError(f"{path}: {name}: unsupported dtype {tag!r}")
        shape, offs = ent["shape"], ent["data_offsets"]
        if (not isinstance(shape, list) or not all(isinstance(d, int) and d >= 0 for d in shape)
                or not isinstance(offs, list) or len(offs) != 2 or not all(isinstance(o, int) for o in offs)):
            raise ValueError(f"{path}: {name}: shape {shape!r} or data_offsets {offs!r} malformed")
        b, e = offs
        if not 0 <= b <= e <= nbytes:
            raise ValueError(f"{path}: {name}: offsets [{b}, {e}) outside the {nbytes} B of data")
        itemsize = np.dtype(_DTYPES[tag][0]).itemsize
        if int(np.prod(shape, dtype=np.int64)) * itemsize != e - b:
            raise ValueError(f"{path}: {name}: shape {shape} x {itemsize} B != {e - b} B of data")
        spans.append((b, e, name))
    spans.sort()
    for (b0, e0, n0), (b1, e1, n1) in zip(spans, spans[1:]):
        if b1 < e0:
            raise ValueError(f"{path}: {n0} and {n1} overlap")
    mm = np.memmap(path, dtype=np.uint8, mode="c") if size > 0 else np.zeros(0, np.uint8)
    out = {}
    for b, e, name in spans:
        ent = header[name]
        npdt, tdt = _DTYPES[ent["dtype"]]
        raw = mm[base + b: base + e]
        if (base + b) % np.dtype(npdt).itemsize:
            raw = np.array(raw)  # unaligned: copy
        arr = raw.view(npdt).reshape(ent["shape"])
        t = torch.from_numpy(arr)
        out[name] = t.view(torch.bfloat16) if tdt == torch.bfloat16 else t
    return out, {str(k): str(v) for k, v in meta.items()}


def write_safetensors(path: str, tensors: Dict[str, torch.Tensor], metadata: Optional[Dict[str, str]] = None) -> None:
    """Write tensors (any device; copied to the host) in the safetensors container: entries
    ordered by element size (largest first), then name, so every offset is aligned to its
    element; the header is padded with spaces to a multiple of 8 bytes."""
    _check_le()
    items = []
    for name, t in tensors.items():
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name}: expected a torch.Tensor")
        if t.dtype not in _TAGS:
            raise ValueError(f"{name}: unsupported dtype {t.dtype}")
        items.append((name, t.detach().contiguous().cpu()))
    items.sort(key=lambda it: (-it[1].element_size(), it[0]))
    header: Dict[str, object] = {}
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    off = 0
    for name, t in items:
        n = t.numel() * t.element_size()
        header[name] = {"dtype": _TAGS[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + n]}
        off += n
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * (-len(hb) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for _, t in items:
            if t.numel():
                src = t.view(torch.uint16) if t.dtype == torch.bfloat16 else t
                f.write(src.numpy().tobytes())


def extract_scalar_f32(t: Optional[torch.Tensor]) -> float:
    """engine.rs:14-19: the first element of the flattened tensor as f32."""
    if t is None:
        raise KeyError("Missing threshold tensor")
    flat = t.flatten().to(torch.float32)
    if flat.numel() == 0:
        raise ValueError("Empty threshold tensor")
    return float(flat[0])


def is_compressed_layer(tensors: Dict[str, torch.Tensor], layer_idx: int) -> bool:
    """model.rs:438-439: a layer's MLP is compressed when down_proj carries saccade_packed_base."""
    return f"model.layers.{layer_idx}.mlp.down_proj.saccade_packed_base" in tensors


def saccade_blocks(tensors: Dict[str, torch.Tensor], prefix: str) -> Tuple[dict, int, int]:
    """The saccade_* tensors of one projection (model.rs:471-492): the blocks keyed as
    compress_tensor_to_saccade returns them, out_features = scale_base.dim(0) and in_features =
    packed_base.dim(1) * 8.  The delta_* keys are read only when delta_row_ptrs exists; then all
    four must."""
    def get(suffix):
        t = tensors.get(f"{prefix}.saccade_{suffix}")
        if t is None:
            raise KeyError(f"Missing {prefix}.saccade_{suffix}")
        return t

    blocks = {"packed_base": get("packed_base"), "scale_base": get("scale_base")}
    if blocks["packed_base"].dim() != 2 or blocks["scale_base"].dim() != 1:
        raise ValueError(f"{prefix}: packed_base must be 2-D and scale_base 1-D")
    out_features = int(blocks["scale_base"].shape[0])
    in_features = int(blocks["packed_base"].shape[1]) * 8
    if f"{prefix}.saccade_delta_row_ptrs" in tensors:
        for s in ("delta_row_ptrs", "delta_col_indices", "delta_values", "delta_scale"):
            blocks[s] = get(s)
    return blocks, out_features, in_features


def build_saccade_op(tensors: Dict[str, torch.Tensor], prefix: str, config, **kw):
    """model.rs:470-495: SaccadeLinearOp of one projection (kw: device, mode, shard)."""
    from .compress import saccade_op_from_compressed

    blocks, n, k = saccade_blocks(tensors, prefix)
    return saccade_op_from_compressed(blocks, config, n, k, **kw)


@dataclass
class SaccadeMlp:
    """Mlp::from_saccade (model.rs:287-299): gate and up read the same x, so they run as one
    grouped launch; forward = down(silu(gate(x)) * up(x)).  Each op takes and returns f16
    (model.rs:55-62); silu and the product run in f32, the reference model's dtype
    (model.rs:381), and round to f16 once for down."""
    gate_proj: object
    up_proj: object
    down_proj: object
    gate_up: object = None

    def forward(self, xs: torch.Tensor) -> torch.Tensor:
        orig = xs.dtype
        x16 = xs if orig == torch.float16 else xs.to(torch.float16)  # model.rs:58-61
        if self.gate_up is not None:
            gate, up = self.gate_up.forward(x16)
        else:
            gate, up = self.gate_proj.forward(x16), self.up_proj.forward(x16)
        h = torch.nn.functional.silu(gate.float()) * up.float()
        y = self.down_proj.forward(h.to(torch.float16))
        return y if orig == torch.float16 else y.to(orig)

    __call__ = forward


def load_mlp(tensors: Dict[str, torch.Tensor], layer_idx: int, *, device=None, mode: str = "fast",
             group: bool = True) -> Optional[SaccadeMlp]:
    """model.rs:437-451: the layer's three C-TARQ projections with the layer's thresholds, or
    None when the layer is stored uncompressed (the caller keeps its dense weights)."""
    from .op import SaccadeConfig, SaccadeLinearGroup

    if not is_compressed_layer(tensors, layer_idx):
        return None
    t4 = extract_scalar_f32(tensors.get(f"model.layers.{layer_idx}.saccade_t4"))
    t8 = extract_scalar_f32(tensors.get(f"model.layers.{layer_idx}.saccade_t8"))
    cfg = SaccadeConfig(t4, t8)
    prefix = f"model.layers.{layer_idx}.mlp"
    ops = [build_saccade_op(tensors, f"{prefix}.{p}", cfg, device=device, mode=mode) for p in MLP_PROJS]
    gate_up = None
    if group and ops[0].in_features == ops[1].in_features:
        gate_up = SaccadeLinearGroup(ops[:2])
    return SaccadeMlp(ops[0], ops[1], ops[2], gate_up)


def load_saccade_checkpoint(source, num_layers: Optional[int] = None, *, device=None, mode: str = "fast",
                            group: bool = True) -> Tuple[List[Optional[SaccadeMlp]], Dict[str, torch.Tensor]]:
    """The C-TARQ part of model.rs:379-432: for each of `num_layers` layers (default: every
    `model.layers.{i}` present) its SaccadeMlp or None, and the tensors no op consumed (attention,
    norms, embeddings and dense MLP weights) for the rest of the model.  `source` is a path or a
    name -> tensor mapping."""
    if isinstance(source, (str, os.PathLike)):
        tensors, _ = read_safetensors(os.fspath(source))
    else:
        tensors = dict(source)
    if num_layers is None:
        parts = (k.split(".") for k in tensors if k.startswith("model.layers."))
        idx = {int(p[2]) for p in parts if len(p) > 2 and p[2].isdigit()}
        num_layers = max(idx) + 1 if idx else 0
    mlps, used = [], set()
    for i in range(num_layers):
        mlp = load_mlp(tensors, i, device=device, mode=mode, group=group)
        mlps.append(mlp)
        if mlp is not None:
            used.update({f"model.layers.{i}.saccade_t4", f"model.layers.{i}.saccade_t8"})
            used.update(f"model.layers.{i}.mlp.{p}.saccade_{s}" for p in MLP_PROJS for s in BLOCK_SUFFIXES)
    rest = {k: v for k, v in tensors.items() if k not in used}
    return mlps, rest


def compile_mlp_checkpoint(tensors: Dict[str, torch.Tensor], num_layers: int, t4: float, t8: float,
                           target_fill: float, *, device=None, projs: Iterable[str] = MLP_PROJS,
                           log=None) -> Dict[str, torch.Tensor]:
    """compile.rs:158-205 (phase 4): every tensor that is not an MLP projection weight is copied
    unchanged; each of the `num_layers` layers gets saccade_t4 / saccade_t8 (f32 [1]); each 2-D
    projection weight with in_features % 8 == 0 becomes its saccade_* blocks, its threshold from
    compute_percentile_threshold at `target_fill`, while one of another shape is kept as is and a
    missing one is skipped with a warning.  Compression runs on the GPU (bit-identical to the
    reference's packer); the outputs are host tensors."""
    from .compress import compress_tensor_to_saccade, compute_percentile_threshold

    projs = tuple(projs)
    warn = log or (lambda msg: print(msg, file=sys.stderr))
    out = {}
    for name, t in tensors.items():
        if not (any(p in name for p in projs) and name.endswith(".weight")):
            out[name] = t
    for i in range(num_layers):
        out[f"model.layers.{i}.saccade_t4"] = torch.tensor([t4], dtype=torch.float32)
        out[f"model.layers.{i}.saccade_t8"] = torch.tensor([t8], dtype=torch.float32)
        for p in projs:
            key = f"model.layers.{i}.mlp.{p}.weight"
            w = tensors.get(key)
            if w is None:
                warn(f"Warning: missing {key}, skipping")
                continue
            if w.dim() != 2 or w.shape[1] % 8:
                warn(f"Warning: {key} has incompatible shape {list(w.shape)}, keeping as-is")
                out[key] = w
                continue
            wd = w if device is None else w.to(device)
            thr = compute_percentile_threshold(wd, target_fill)
            for suffix, blk in compress_tensor_to_saccade(wd, thr).items():
                out[f"model.layers.{i}.mlp.{p}.saccade_{suffix}"] = blk.cpu()
    return out
