"""The recorded reference-model calls (tests/golden/model_calls) on the CPU:
every call model.py made into the op API binds to the drop-in attnres_ops
function of the same name, with the same arguments, and the fixtures cover
the call sites the drop-in must serve."""
import inspect

import pytest

import attnres_ops
from model_calls import FILES, IDS, call_args, load


@pytest.mark.parametrize("path", FILES, ids=IDS)
def test_recorded_calls_bind_to_the_drop_in(path):
    d, meta = load(path)
    assert meta["calls"], "no call recorded"
    for call in meta["calls"]:
        fn = getattr(attnres_ops, call["fn"])
        _, args, kwargs = call_args(d, call)
        inspect.signature(fn).bind(*args, **kwargs)
        if meta["train"] and any(lf["requires_grad"] for lf in call["leaves"]):
            assert "grad_outs" in call and call["grad_in"], f"{call['fn']}: no gradients recorded"


def test_fixtures_cover_the_model_call_sites():
    seen = set()
    for path in FILES:
        _, meta = load(path)
        seen.update(c["fn"] for c in meta["calls"])
    assert {
        "lrid_attention_residual_read", "attention_residual_read", "attention_residual_phase1_from_logits",
        "lrid_attention_residual_phase2", "lrid_attention_residual_phase2_torch", "attention_residual_phase2",
        "attention_residual_phase2_torch",
        "lrid_attention_residual_read_gated", "lrid_attention_residual_read_key_from_value",
    } <= seen
