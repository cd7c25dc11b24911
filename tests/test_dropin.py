"""The drop-in module exposes every name the reference's model.py imports
(model.py:9-19) and the reference's full __all__ (attnres_ops.py:26-40)."""
import importlib
import inspect
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

MODEL_IMPORTS = [
    "attention_residual_average_read", "attention_residual_phase1_from_logits", "attention_residual_phase2",
    "attention_residual_phase2_torch", "attention_residual_phase2_from_logit", "attention_residual_read",
    "lrid_attention_residual_phase2", "lrid_attention_residual_phase2_torch", "lrid_attention_residual_read",
]
REFERENCE_ALL = MODEL_IMPORTS + [
    "attention_residual_phase1", "attention_residual_read_torch", "is_fused_attnres_available",
    "lrid_attention_residual_read_torch",
]


def test_dropin_exports_reference_api():
    mod = importlib.import_module("attnres_ops")
    assert os.path.dirname(os.path.abspath(mod.__file__)) == os.path.join(ROOT, "lr-attnres_b200")
    for name in REFERENCE_ALL:
        assert callable(getattr(mod, name)), name
    assert set(REFERENCE_ALL) <= set(mod.__all__)


@pytest.mark.parametrize("name,params", [
    ("lrid_attention_residual_read", ["values", "keys", "query", "num_heads", "logit_scale", "key_norm",
                                      "force_triton", "normalize_output", "source_counts", "source_logit_biases"]),
    ("attention_residual_read", ["values", "query", "key_norm", "force_triton", "normalize_output",
                                 "source_counts", "source_logit_biases"]),
    ("attention_residual_phase1_from_logits", ["values", "logits", "force_triton", "normalize_output"]),
    ("attention_residual_average_read", ["values", "normalize_output", "force_triton"]),
])
def test_dropin_signatures_match_reference(name, params):
    mod = importlib.import_module("attnres_ops")
    assert list(inspect.signature(getattr(mod, name)).parameters) == params


def test_fused_reads_reject_cpu_tensors():
    import torch

    mod = importlib.import_module("attnres_ops")
    v = [torch.randn(1, 2, 8) for _ in range(3)]
    with pytest.raises(RuntimeError, match="CUDA"):
        mod.attention_residual_read(v, torch.randn(8), True)
    with pytest.raises(RuntimeError, match="CUDA"):
        mod.attention_residual_phase1_from_logits(v, torch.randn(2, 3, 1, 2))


def test_torch_reference_functions_match_oracle_on_cpu():
    """The PyTorch reference functions (not the fused path) agree with the oracle."""
    import numpy as np
    import torch

    from oracle import oracle

    mod = importlib.import_module("attnres_ops")
    rng = np.random.default_rng(3)
    v = rng.standard_normal((4, 6, 32)).astype(np.float32)
    k = rng.standard_normal((4, 6, 16)).astype(np.float32)
    q = rng.standard_normal((2, 8)).astype(np.float32)
    out = mod.lrid_attention_residual_read_torch(torch.tensor(v).reshape(4, 1, 6, 32), torch.tensor(k).reshape(4, 1, 6, 16),
                                                torch.tensor(q), 2, 0.5, True)
    ref = oracle.lrid_forward(v, k, 2, 0.5, True, query=q)[0]
    np.testing.assert_allclose(out.reshape(6, 32).numpy(), ref, rtol=1e-5, atol=1e-5)
