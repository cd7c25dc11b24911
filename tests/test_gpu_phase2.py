"""GPU parity of the cached-logit phase 2 (the live partial block merged into
the phase-1 result) against the oracle, pinned by the reference's own golden
vectors: LRID key, base key rms_norm(partial_value) and given logit, with and
without logit bias and output norm, fp32 / bf16 / fp16, ragged widths."""
import numpy as np
import pytest
import torch

from cases import CASES, case_inputs
from gpu_helpers import RMS_EPS, assert_close, rounded, to_np
from oracle import oracle
from test_oracle_golden import phase2_args

pytestmark = pytest.mark.gpu

P2_CASES = [c for c in CASES if c["kind"] == "phase2"]


def run_phase2(case, inp, dtype, bias_as_tensor=True):
    import attnres_ops as A

    N, D = inp["partial_value"].shape
    dev = lambda x, dt=dtype: torch.tensor(np.asarray(x, np.float32), device="cuda").to(dt).requires_grad_(True)  # noqa: E731
    pv = dev(inp["partial_value"].reshape(1, N, D))
    io = dev(inp["interblock_output"].reshape(1, N, D))
    lse = dev(inp["interblock_lse"].reshape(1, N), torch.float32)
    bias = 0.0
    if case.get("bias"):
        bias = dev(inp["logit_bias"], torch.float32) if bias_as_tensor else float(inp["logit_bias"])
    norm = case.get("normalize_output", False)
    extra = {}
    if case["mode"] == "lrid":
        pk = dev(inp["partial_key"].reshape(1, N, -1))
        q = dev(inp["query"], torch.float32)
        out = A.lrid_attention_residual_phase2(pv, pk, q, io, lse, case["scale"], case["key_norm"],
                                               normalize_output=norm, logit_bias=bias)
        extra = {"d_partial_key": pk, "dq": q}
    elif case["mode"] == "base":
        q = dev(inp["query"], torch.float32)
        out = A.attention_residual_phase2(pv, q, io, lse, case["key_norm"], normalize_output=norm, logit_bias=bias)
        extra = {"dq": q}
    else:
        lg = dev(inp["partial_logit"].reshape(1, N), torch.float32)
        out = A.attention_residual_phase2_from_logit(pv, lg, io, lse, normalize_output=norm)
        extra = {"d_partial_logit": lg}
    g = torch.tensor(inp["grad_output"].reshape(1, N, D), device="cuda").to(dtype)
    out.backward(g)
    torch.cuda.synchronize()
    res = {"out": to_np(out).reshape(N, D), "d_partial_value": to_np(pv.grad).reshape(N, D),
           "d_interblock_output": to_np(io.grad).reshape(N, D), "d_interblock_lse": to_np(lse.grad).reshape(N)}
    for k, t in extra.items():
        res[k] = to_np(t.grad).reshape(N, -1) if k == "d_partial_key" else to_np(t.grad).reshape(-1)
    if case.get("bias") and bias_as_tensor:
        res["dbias"] = to_np(bias.grad).reshape(())
    return res


def oracle_phase2(case, inp, dtype, saved_output=None):
    """The oracle on the inputs the GPU sees (rounded to dtype), with the
    dtype's eps where the reference uses it; the output-norm backward uses the
    saved value-dtype output, as the reference's backward does."""
    r = dict(inp)
    for k in ("partial_value", "interblock_output", "partial_key", "grad_output"):
        if k in r:
            r[k] = rounded(r[k], dtype)
    if "query" in r:
        r["query"] = rounded(r["query"], dtype)
    mode, kw = phase2_args(case, r)
    if case["mode"] == "base":
        kw["key_eps"] = RMS_EPS
    kw["output_eps"] = RMS_EPS
    base = (r["partial_value"], r["interblock_output"], r["interblock_lse"])
    out, _ = oracle.phase2_forward(mode, *base, **kw)
    res = oracle.phase2_backward(mode, *base, r["grad_output"], saved_output=saved_output, **kw)
    res["out"] = out
    return res


def compare(case, res, ref, dtype, n):
    for k in ("out", "d_partial_value", "d_interblock_output", "d_interblock_lse", "d_partial_key",
              "d_partial_logit"):
        if k in res:
            assert_close(k, res[k], ref[k], dtype)
    if "dq" in res:
        assert_close("dq", res["dq"], ref["dq"], dtype, sum_terms=n)
    if "dbias" in res:
        assert_close("dbias", res["dbias"], np.asarray(ref["dbias"]), dtype, sum_terms=n)


@pytest.mark.parametrize("case", P2_CASES, ids=[c["name"] for c in P2_CASES])
def test_phase2_golden_fp32(case):
    inp = case_inputs(case)
    res = run_phase2(case, inp, torch.float32)
    ref = oracle_phase2(case, inp, torch.float32)
    compare(case, res, ref, torch.float32, inp["partial_value"].shape[0])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("mode,D,R,key_norm,norm,bias", [
    ("lrid", 1024, 64, True, False, False),   # config-2 row width, default block training
    ("lrid", 2048, 64, False, True, True),
    ("base", 1000, 0, True, True, False),     # width not a multiple of the 16-byte pack
    ("base", 256, 0, False, False, True),
    ("logit", 4096, 0, False, True, False),
])
def test_phase2_shapes(dtype, mode, D, R, key_norm, norm, bias):
    rng = np.random.default_rng(D + R)
    N = 2 * 333
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    inp = {"partial_value": f(N, D), "interblock_output": f(N, D), "interblock_lse": f(N),
           "grad_output": f(N, D), "logit_bias": np.float32(0.3)}
    case = dict(mode=mode, scale=0.125, key_norm=key_norm, normalize_output=norm, bias=bias)
    if mode == "lrid":
        inp["partial_key"] = f(N, R)
        inp["query"] = f(R)
    elif mode == "base":
        inp["query"] = f(D) * np.float32(0.05)
    else:
        inp["partial_logit"] = f(N)
    res = run_phase2(case, inp, dtype)
    ref = oracle_phase2(case, inp, dtype, saved_output=res["out"] if norm else None)
    compare(case, res, ref, dtype, N)


def test_phase2_parameter_grads_are_deterministic():
    import attnres_ops as A

    torch.manual_seed(3)
    N, D, R = 4096, 1024, 64
    pv = torch.randn(2, N // 2, D, device="cuda", dtype=torch.bfloat16)
    io = torch.randn_like(pv)
    lse = torch.randn(2, N // 2, device="cuda")
    pk = torch.randn(2, N // 2, R, device="cuda", dtype=torch.bfloat16)
    g = torch.randn_like(pv)
    grads = []
    for _ in range(2):
        q = torch.randn(R, device="cuda", generator=torch.Generator("cuda").manual_seed(1)).requires_grad_(True)
        b = torch.tensor(0.2, device="cuda", requires_grad=True)
        A.lrid_attention_residual_phase2(pv, pk, q, io, lse, 0.125, True, logit_bias=b).backward(g)
        grads.append((q.grad.clone(), b.grad.clone()))
    for x, y in zip(*grads):
        assert torch.equal(x, y)


def test_phase2_cpu_tensors_fail_loudly():
    import attnres_ops as A

    with pytest.raises(RuntimeError, match="CUDA"):
        A.attention_residual_phase2_from_logit(torch.randn(1, 4, 8), torch.randn(1, 4), torch.randn(1, 4, 8),
                                               torch.randn(1, 4))
