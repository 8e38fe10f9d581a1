"""NVFP4 linear-layer path on B200: radiance's ``radiance.nvfp4`` operator surface, re-pointed at
the sm_100a CUDA library (``include/radiance_nvfp4.h``).

Same names and semantics as ``src/radiance/nvfp4/__init__.py`` in jamespa16/radiance for
everything on the hot path; the reference's pure-torch emulation (``quantize_reference`` and the
``ref_*`` helpers) defines the format and stays in radiance.
"""

from .grouped import bmm
from .linear import FP4FeedForward, FP4Linear, FP4Recipe, FP4SwiGLU, refresh_fp4_weights
from .quantize import (
    BLOCK,
    E4M3_MAX,
    FP4_MAX,
    FP4_VALUES,
    TINY,
    NVFP4Tensor,
    blocked_offset,
    col_scale_bytes,
    global_scale_and_column_sums,
    global_scale_of,
    hadamard_matrix,
    interleave_gate_up,
    merge_gate_up,
    mm,
    nvfp4_linear_mm,
    nvfp4_mm,
    nvfp4_supported,
    pack_nibbles,
    quantize,
    quantize_both,
    quantize_into_,
    quantize_supported_shape,
    require_nvfp4,
    row_scale_bytes,
    scale_denominator,
    split_gate_up,
    swiglu_mm,
    unpack_nibbles,
    update_and_global_scale_,
)

__all__ = [
    "BLOCK",
    "E4M3_MAX",
    "FP4_MAX",
    "FP4_VALUES",
    "TINY",
    "NVFP4Tensor",
    "FP4FeedForward",
    "FP4Linear",
    "FP4SwiGLU",
    "FP4Recipe",
    "blocked_offset",
    "bmm",
    "col_scale_bytes",
    "global_scale_and_column_sums",
    "global_scale_of",
    "hadamard_matrix",
    "interleave_gate_up",
    "merge_gate_up",
    "mm",
    "nvfp4_linear_mm",
    "nvfp4_mm",
    "nvfp4_supported",
    "pack_nibbles",
    "quantize",
    "quantize_both",
    "quantize_into_",
    "quantize_supported_shape",
    "refresh_fp4_weights",
    "require_nvfp4",
    "row_scale_bytes",
    "scale_denominator",
    "split_gate_up",
    "swiglu_mm",
    "unpack_nibbles",
    "update_and_global_scale_",
]
