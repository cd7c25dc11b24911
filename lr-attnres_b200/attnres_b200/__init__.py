"""attnres_b200 — B200 (sm_100a) fused block Attention-Residual depth-routing read.

The CUDA kernels live in libattnres_b200.so (C ABI: include/attnres_b200.h);
this package registers the reference-compatible torch.library operators
(attnres::lrid_read_list, attnres::lrid_read_list_backward) plus the general
attnres::lrid_read / attnres::base_read operators, and exposes the reference's
public read functions.
"""
from . import _native
from .ops import (
    attention_residual_block_summary,
    attention_residual_read,
    block_summary,
    block_summary_norm,
    base_read,
    is_fused_attnres_available,
    lrid_attention_residual_read,
    lrid_attention_residual_read_gated,
    lrid_attention_residual_read_key_from_value,
    lrid_block_source,
    lrid_fused_projection_forward,
    lrid_kv_read,
    lrid_read,
    lrid_read_list,
    lrid_read_list_backward,
    source_logit_bias,
)

__all__ = [
    "attention_residual_block_summary",
    "attention_residual_read",
    "block_summary",
    "block_summary_norm",
    "base_read",
    "is_fused_attnres_available",
    "lrid_attention_residual_read",
    "lrid_attention_residual_read_gated",
    "lrid_attention_residual_read_key_from_value",
    "lrid_block_source",
    "lrid_fused_projection_forward",
    "lrid_kv_read",
    "lrid_read",
    "lrid_read_list",
    "lrid_read_list_backward",
    "source_logit_bias",
]
