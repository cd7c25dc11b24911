"""GPU parity of the base AttnRes read (forward + backward) against the CPU oracle.

Mirrors test_fused_base_attnres_matches_torch (reference
tests/test_attnres_ops.py:884-895) and BASELINE config 1.
"""
import numpy as np
import pytest
import torch

from cases import CASES, case_inputs
from gpu_helpers import RMS_EPS, assert_close, dev_rows, rounded, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


def run_base(inp, B, T, key_norm, dtype, normalize_output=False, bias=False):
    import attnres_b200 as ops

    values = [dev_rows(v, B, T, dtype) for v in inp["values"]]
    q = torch.tensor(inp["query"], device="cuda", dtype=torch.float32, requires_grad=True)
    biases = None
    if bias:
        biases = [torch.tensor(float(b), device="cuda", requires_grad=True) for b in inp["logit_bias"]]
    out = ops.attention_residual_read(values, q, key_norm, normalize_output=normalize_output,
                                      source_logit_biases=biases)
    out.backward(dev_rows(inp["grad_output"], B, T, dtype, requires_grad=False))
    torch.cuda.synchronize()
    res = {"out": to_np(out).reshape(B * T, -1),
           "dV": np.stack([to_np(v.grad).reshape(B * T, -1) for v in values]),
           "dq": to_np(q.grad).reshape(-1)}
    if biases:
        res["dbias"] = np.array([b.grad.item() for b in biases])
    return res


def oracle_base(inp, key_norm, dtype, normalize_output, bias):
    eps = RMS_EPS
    vals = rounded(inp["values"], dtype)
    q = rounded(inp["query"], dtype)
    b = inp["logit_bias"] if bias else None
    norm = oracle.NORM_ROW if normalize_output else oracle.NORM_NONE
    out = oracle.base_forward(vals, q, key_norm, b, norm, key_eps=eps, output_eps=eps)[0]
    grads = oracle.base_backward(vals, q, key_norm, rounded(inp["grad_output"], dtype), b, norm,
                                 key_eps=eps, output_eps=eps)
    grads["out"] = out
    return grads


BASE_CASES = [c for c in CASES if c["kind"] == "base"]


@pytest.mark.parametrize("case", BASE_CASES, ids=[c["name"] for c in BASE_CASES])
def test_base_golden_cases_fp32(case):
    inp = case_inputs(case)
    B, T = case["B"], case["T"]
    res = run_base(inp, B, T, case["key_norm"], torch.float32, case.get("normalize_output", False),
                   case.get("bias", False))
    ref = oracle_base(inp, case["key_norm"], torch.float32, case.get("normalize_output", False),
                      case.get("bias", False))
    assert_close("out", res["out"], ref["out"], torch.float32)
    assert_close("dV", res["dV"], ref["dV"], torch.float32)
    assert_close("dq", res["dq"], ref["dq"], torch.float32, sum_terms=B * T)
    if "dbias" in ref:
        assert_close("dbias", res["dbias"], ref["dbias"], torch.float32, sum_terms=B * T)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [256, 1024, 2048, 100])
def test_base_dtypes_and_widths(dtype, D):
    rng = np.random.default_rng(D)
    S, B, T = 6, 1, 45
    inp = {"values": rng.standard_normal((S, B * T, D)).astype(np.float32),
           "query": (rng.standard_normal(D) * 0.02).astype(np.float32),
           "logit_bias": rng.standard_normal(S).astype(np.float32),
           "grad_output": rng.standard_normal((B * T, D)).astype(np.float32)}
    res = run_base(inp, B, T, True, dtype, normalize_output=True, bias=True)
    ref = oracle_base(inp, True, dtype, True, True)
    assert_close("out", res["out"], ref["out"], dtype)
    assert_close("dV", res["dV"], ref["dV"], dtype)
    assert_close("dq", res["dq"], ref["dq"], dtype, sum_terms=B * T)
