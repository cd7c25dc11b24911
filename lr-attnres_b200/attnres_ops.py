"""Drop-in replacement for the reference's `attnres_ops` module (jon123boss/LR-AttnRes).

Put this directory on sys.path ahead of the reference checkout and
`from attnres_ops import ...` in model.py resolves here: the same public names
(attnres_ops.py:26-40) with the same signatures, backed by the B200 kernels in
libattnres_b200.so. The fused reads and the phase-2 merges have no CPU path;
the `*_torch` functions are PyTorch by definition in the reference too.
"""
from attnres_b200.ops import (  # noqa: F401
    attention_residual_average_read,
    attention_residual_phase1_from_logits,
    attention_residual_phase2,
    attention_residual_phase2_from_logit,
    attention_residual_read,
    is_fused_attnres_available,
    lrid_attention_residual_read,
    lrid_attention_residual_read_gated,
    lrid_attention_residual_phase2,
    lrid_attention_residual_read_key_from_value,
)
from attnres_b200.torch_ref import (  # noqa: F401
    attention_residual_phase1,
    attention_residual_phase2_torch,
    attention_residual_read_torch,
    lrid_attention_residual_phase2_torch,
    lrid_attention_residual_read_torch,
)

__all__ = [
    "attention_residual_average_read",
    "attention_residual_phase1",
    "attention_residual_phase1_from_logits",
    "attention_residual_phase2",
    "attention_residual_phase2_from_logit",
    "attention_residual_phase2_torch",
    "attention_residual_read",
    "attention_residual_read_torch",
    "is_fused_attnres_available",
    "lrid_attention_residual_phase2",
    "lrid_attention_residual_phase2_torch",
    "lrid_attention_residual_read",
    "lrid_attention_residual_read_torch",
]
