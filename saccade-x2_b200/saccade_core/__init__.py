"""saccade_core: the C-TARQ linear on NVIDIA B200, with saccade-core's operator surface.

Compute runs only in libsaccade_ctarq.so (hand-written sm_100a kernels, C ABI in
include/saccade_ctarq.h); this package is the host-side mirror of the reference's
names (saccade-core/src/lib.rs:9-12).
"""
from ._lib import CTarqError, LIB_PATH
from .checkpoint import (SaccadeMlp, build_saccade_op, compile_mlp_checkpoint, extract_scalar_f32,
                         load_mlp, load_saccade_checkpoint, read_safetensors, saccade_blocks,
                         write_safetensors)
from .graph import CapturedStep
from .compress import (ProfileRunner, compress_tensor_to_saccade, compute_percentile_threshold,
                       saccade_op_from_compressed)
from .op import (GroupRouting, SaccadeConfig, SaccadeLinearGroup, SaccadeLinearOp, SparseDeltaMatrix, finalize,
                 is_c_tarq_bypassed, set_bypass_c_tarq, variance_heuristic)

__all__ = [
    "CapturedStep", "CTarqError", "GroupRouting", "LIB_PATH", "ProfileRunner", "SaccadeConfig", "SaccadeLinearGroup", "SaccadeLinearOp",
    "SaccadeMlp", "SparseDeltaMatrix", "build_saccade_op", "compile_mlp_checkpoint", "compress_tensor_to_saccade",
    "compute_percentile_threshold", "extract_scalar_f32", "finalize", "is_c_tarq_bypassed", "load_mlp",
    "load_saccade_checkpoint", "read_safetensors", "saccade_blocks", "saccade_op_from_compressed",
    "set_bypass_c_tarq", "variance_heuristic", "write_safetensors",
]
