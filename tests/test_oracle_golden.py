"""The CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by tests/golden/make_golden.py, which runs the
reference's PyTorch path (attnres_ops.py) in fp32 with autograd. The oracle is
double precision, so agreement is at fp32 rounding level.
"""
import os

import numpy as np
import pytest

from cases import CASES, case_inputs
from oracle import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
F32_EPS = float(np.finfo(np.float32).eps)


def oracle_case(case):
    inp = case_inputs(case)
    norm = oracle.NORM_NONE
    if case.get("normalize_output") and case["kind"] not in ("phase1", "phase2"):
        if case["kind"] == "base":
            norm = oracle.NORM_ROW
        else:
            norm = oracle.NORM_PER_HEAD if case["H"] == 1 else oracle.NORM_ROW
    bias = inp["logit_bias"] if case.get("bias") else None
    if case["kind"] == "phase2":
        return oracle_phase2(case, inp)
    if case["kind"] == "phase1":
        nrm = case.get("normalize_output", False)
        out, lse, _, _, _ = oracle.phase1_forward(inp["values"], inp["logits"], nrm)
        grads = oracle.phase1_backward(inp["values"], inp["logits"], inp["grad_output"], inp["grad_lse"], nrm)
        grads["lse"] = lse
        return out, grads
    if case["kind"] == "lrid_kv":
        vn = case.get("value_norm", True)
        args = (inp["values"], inp["key_weight"], case["H"], case["scale"], case["key_norm"])
        out = oracle.lrid_kv_forward(*args, value_norm=vn, query=inp["query"])[0]
        grads = oracle.lrid_kv_backward(*args, inp["grad_output"], value_norm=vn, query=inp["query"])
        return out, grads
    if case["kind"] == "base":
        out, _ = oracle.base_forward(inp["values"], inp["query"], case["key_norm"], bias, norm)
        grads = oracle.base_backward(inp["values"], inp["query"], case["key_norm"], inp["grad_output"], bias, norm)
        return out, grads
    kw = dict(logit_bias=bias, output_norm=norm)
    if case["query"] == "static":
        kw["query"] = inp["query"]
    elif case["query"] == "dynamic":
        kw["query_dynamic"] = inp["query_dynamic"]
    else:
        kw.update(query=inp["query"], gate=inp["gate"], query_dynamic=inp["query_dynamic"])
    args = (inp["values"], inp["keys"], case["H"], case["scale"], case["key_norm"])
    out = oracle.lrid_forward(*args, **kw)[0]
    grads = oracle.lrid_backward(*args, inp["grad_output"], **kw)
    if "dq_dynamic" in grads:
        grads["dq_dynamic"] = grads["dq_dynamic"]
    return out, grads


def phase2_args(case, inp):
    """Keyword arguments of oracle.phase2_forward/backward for a phase-2 case,
    with the reference's eps choices: fp32 eps for the LRID key norm
    (_norm(partial_key.float())), the value dtype's eps (fp32 here) for the
    base key norm and the output norm."""
    mode = {"lrid": oracle.PHASE2_LRID, "base": oracle.PHASE2_BASE, "logit": oracle.PHASE2_LOGIT}[case["mode"]]
    kw = dict(partial_key=inp.get("partial_key"), query=inp.get("query"), partial_logit=inp.get("partial_logit"),
              logit_scale=case.get("scale", 1.0), key_norm=case.get("key_norm", False),
              logit_bias=float(inp["logit_bias"]) if case.get("bias") else 0.0,
              normalize_output=case.get("normalize_output", False))
    return mode, kw


def oracle_phase2(case, inp):
    mode, kw = phase2_args(case, inp)
    base = (inp["partial_value"], inp["interblock_output"], inp["interblock_lse"])
    out, _ = oracle.phase2_forward(mode, *base, **kw)
    grads = oracle.phase2_backward(mode, *base, inp["grad_output"], **kw)
    return out, grads


def _close(name, actual, expected, scale=1.0):
    expected = np.asarray(expected, np.float64)
    tol = 2e-5 * scale * max(1.0, float(np.abs(expected).max(initial=0.0)))
    err = float(np.abs(np.asarray(actual, np.float64) - expected).max(initial=0.0))
    assert err <= tol, f"{name}: max |err| {err:.3e} > {tol:.3e}"


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_golden(case):
    gold = np.load(os.path.join(GOLDEN, case["name"] + ".npz"))
    out, grads = oracle_case(case)
    _close("out", out, gold["out"])
    keep = case.get("keep_tokens")
    for name in ("dV", "dK"):
        if name in gold:
            got = grads[name]
            if keep is not None:
                _close(name + "_sum", got.sum(axis=(1, 2)), gold[name + "_sum"], scale=10.0)
                got = got[:, :keep]
            _close(name, got, gold[name])
    for name in ("d_partial_value", "d_interblock_output", "d_interblock_lse", "d_partial_key", "d_partial_logit"):
        if name in gold:
            _close(name, grads[name], gold[name])
    for name in ("lse", "dlogits"):
        if name in gold:
            _close(name, grads[name], gold[name])
    if "dW" in gold:
        _close("dW", grads["dW"], gold["dW"], scale=4.0)
    for name in ("dq", "dgate", "dq_dynamic", "dbias"):
        if name in gold:
            _close(name, np.asarray(grads[name]).reshape(gold[name].shape), gold[name], scale=4.0)


def test_count_prior_zero_query_is_count_weighted_mean():
    """Known answer from the reference (tests/test_attnres_ops.py:479-512): with a
    zero query and log-count logit biases the read is the count-weighted mean."""
    emb = np.full((1, 2, 8), 2.0, np.float32)
    blk = np.full((1, 2, 8), 10.0, np.float32)
    keys = np.zeros((2, 2, 4), np.float32)
    bias = np.log(np.array([1.0, 3.0], np.float32))
    out = oracle.lrid_forward(np.concatenate([emb, blk]), keys, 1, 1.0, False,
                              query=np.zeros((1, 4), np.float32), logit_bias=bias)[0]
    np.testing.assert_allclose(out, (emb[0] + 3 * blk[0]) / 4, rtol=1e-7, atol=1e-7)
    out_b = oracle.base_forward(np.stack([np.full((2, 4), 1.0, np.float32), np.full((2, 4), 7.0, np.float32)]),
                                np.zeros(4, np.float32), False, logit_bias=bias)[0]
    np.testing.assert_allclose(out_b, np.full((2, 4), (1.0 + 21.0) / 4), rtol=1e-7)


def test_oracle_thread_count_does_not_change_results():
    case = CASES[2]
    oracle.set_num_threads(1)
    a = oracle_case(case)
    oracle.set_num_threads(4)
    b = oracle_case(case)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_allclose(a[1]["dq"], b[1]["dq"], rtol=1e-13, atol=1e-13)
