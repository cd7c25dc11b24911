"""GPU parity of the cached-logit block read (phase 1), the mean read and the
drop-in module's phase-2 merge against the oracle / reference formulas."""
import numpy as np
import pytest
import torch

from cases import CASES, case_inputs
from gpu_helpers import RMS_EPS, assert_close, rounded, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


def run_phase1(inp, Q, B, T, dtype, normalize_output, stacked=False):
    import attnres_ops as A

    S, N, D = inp["values"].shape
    vs = torch.tensor(inp["values"].reshape(S, B, T, D), device="cuda").to(dtype).requires_grad_(True)
    lg = torch.tensor(inp["logits"].reshape(Q, S, B, T), device="cuda").requires_grad_(True)
    src = vs if stacked else list(vs.unbind(0))
    out, lse = A.attention_residual_phase1_from_logits(src, lg, normalize_output=normalize_output)
    g = torch.tensor(inp["grad_output"].reshape(Q, B, T, D), device="cuda").to(dtype)
    gl = torch.tensor(inp["grad_lse"].reshape(Q, B, T), device="cuda")
    ((out.float() * g.float()).sum() + (lse * gl).sum()).backward()
    torch.cuda.synchronize()
    return {"out": to_np(out).reshape(Q, N, D), "lse": to_np(lse).reshape(Q, N),
            "dV": to_np(vs.grad).reshape(S, N, D), "dlogits": to_np(lg.grad).reshape(Q, S, N)}


def oracle_phase1(inp, dtype, normalize_output):
    v, g = rounded(inp["values"], dtype), rounded(inp["grad_output"], dtype)
    eps = RMS_EPS
    out, lse, _, _, _ = oracle.phase1_forward(v, inp["logits"], normalize_output, eps)
    res = oracle.phase1_backward(v, inp["logits"], g, inp["grad_lse"], normalize_output, eps)
    res.update(out=out, lse=lse)
    return res


P1_CASES = [c for c in CASES if c["kind"] == "phase1"]


@pytest.mark.parametrize("case", P1_CASES, ids=[c["name"] for c in P1_CASES])
@pytest.mark.parametrize("stacked", [False, True])
def test_phase1_golden_fp32(case, stacked):
    inp = case_inputs(case)
    nrm = case.get("normalize_output", False)
    res = run_phase1(inp, case["Q"], case["B"], case["T"], torch.float32, nrm, stacked)
    ref = oracle_phase1(inp, torch.float32, nrm)
    for k in ("out", "lse", "dV", "dlogits"):
        assert_close(k, res[k], ref[k], torch.float32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("Q,S,D,norm", [(4, 5, 1024, False), (8, 13, 2048, False), (16, 3, 100, True), (1, 9, 256, True)])
def test_phase1_shapes(dtype, Q, S, D, norm):
    rng = np.random.default_rng(Q * 100 + S)
    B, T = 1, 77
    inp = {"values": rng.standard_normal((S, B * T, D)).astype(np.float32),
           "logits": rng.standard_normal((Q, S, B * T)).astype(np.float32),
           "grad_output": rng.standard_normal((Q, B * T, D)).astype(np.float32),
           "grad_lse": rng.standard_normal((Q, B * T)).astype(np.float32)}
    res = run_phase1(inp, Q, B, T, dtype, norm)
    ref = oracle_phase1(inp, dtype, norm)
    for k in ("out", "dV"):
        assert_close(k, res[k], ref[k], dtype)
    assert_close("lse", res["lse"], ref["lse"], torch.float32)
    assert_close("dlogits", res["dlogits"], ref["dlogits"], dtype)


def test_average_read_is_the_mean():
    import attnres_ops as A

    vs = [torch.randn(2, 5, 96, device="cuda", requires_grad=True) for _ in range(4)]
    out = A.attention_residual_average_read(vs)
    ref = torch.stack([v.detach() for v in vs]).mean(0)
    torch.testing.assert_close(out, ref, rtol=1e-6, atol=1e-6)
    out.sum().backward()
    torch.testing.assert_close(vs[0].grad, torch.full_like(vs[0], 0.25), rtol=1e-6, atol=1e-6)


def test_phase1_then_phase2_equals_full_read():
    """Two-phase decomposition used by cached block training (model.py:1808-2000):
    phase 1 over the completed blocks, then the phase-2 merge of the live
    partial block, equals one base read over all sources."""
    import attnres_ops as A

    torch.manual_seed(0)
    S, B, T, D = 5, 2, 33, 128
    vs = [torch.randn(B, T, D, device="cuda") for _ in range(S)]
    q = torch.randn(D, device="cuda") * 0.3
    keys = [torch.nn.functional.rms_norm(v, (D,)) for v in vs]
    logits = torch.stack([(k * q).sum(-1) for k in keys[:-1]])[None]  # [1, S-1, B, T]
    inter, lse = A.attention_residual_phase1_from_logits(vs[:-1], logits)
    merged = A.attention_residual_phase2_torch(vs[-1], q, inter[0], lse[0], True)
    full = A.attention_residual_read(vs, q, True)
    torch.testing.assert_close(merged, full, rtol=1e-5, atol=1e-5)
