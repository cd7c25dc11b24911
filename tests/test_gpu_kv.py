"""GPU parity of the key-from-value LRID read (BASELINE config 4 family):
keys_s = rms_norm(V_s) @ W^T computed inside the op (tcgen05 tensor cores for
bf16/fp16, CUDA cores otherwise), then the depth read; forward and backward
(values through both paths, the key weight, the query) against the oracle."""
import numpy as np
import pytest
import torch

from cases import CASES, case_inputs
from gpu_helpers import RMS_EPS, assert_close, dev_rows, rounded, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=["auto", "simt"])
def kernel_path(request, monkeypatch):
    monkeypatch.setenv("ATTNRES_B200_PATH", request.param)
    yield request.param
    from attnres_b200 import _native

    assert _native.device_status(reset=True) == 0


def run_kv(inp, B, T, H, scale, key_norm, dtype, value_norm=True, normalize_output=False):
    import attnres_b200 as A

    values = [dev_rows(v, B, T, dtype) for v in inp["values"]]
    w = torch.tensor(inp["key_weight"], device="cuda", dtype=torch.float32).to(dtype).requires_grad_(True)
    q = torch.tensor(inp["query"], device="cuda", dtype=torch.float32, requires_grad=True)
    out = A.lrid_attention_residual_read_key_from_value(values, w, q, H, scale, key_norm, value_norm=value_norm,
                                                        normalize_output=normalize_output)
    out.backward(dev_rows(inp["grad_output"], B, T, dtype, requires_grad=False))
    torch.cuda.synchronize()
    return {"out": to_np(out).reshape(B * T, -1),
            "dV": np.stack([to_np(v.grad).reshape(B * T, -1) for v in values]),
            "dW": to_np(w.grad), "dq": to_np(q.grad).reshape(-1)}


def oracle_kv(inp, H, scale, key_norm, dtype, value_norm=True, normalize_output=False):
    eps = RMS_EPS
    kw = {}
    if normalize_output:
        kw = dict(output_norm=oracle.NORM_PER_HEAD if H == 1 else oracle.NORM_ROW, output_eps=eps)
    v, w = rounded(inp["values"], dtype), rounded(inp["key_weight"], dtype)
    q = rounded(inp["query"], dtype)
    g = rounded(inp["grad_output"], dtype)
    out = oracle.lrid_kv_forward(v, w, H, scale, key_norm, value_norm=value_norm, value_eps=eps, query=q, **kw)[0]
    res = oracle.lrid_kv_backward(v, w, H, scale, key_norm, g, value_norm=value_norm, value_eps=eps, query=q, **kw)
    res["out"] = out
    return res


def compare(res, ref, dtype, n, out_norm=False):
    """out_norm: the 16-bit backward reads the saved 16-bit normed output, so
    dV's absolute floor scales with dV (as in test_gpu_lrid.compare)."""
    assert_close("out", res["out"], ref["out"], dtype)
    assert_close("dV", res["dV"], ref["dV"], dtype, scaled_atol=out_norm)
    assert_close("dW", res["dW"], ref["dW"], dtype, sum_terms=n)
    assert_close("dq", res["dq"], ref["dq"], dtype, sum_terms=n)


KV_CASES = [c for c in CASES if c["kind"] == "lrid_kv"]


@pytest.mark.parametrize("case", KV_CASES, ids=[c["name"] for c in KV_CASES])
def test_kv_golden_cases_fp32(case):
    inp = case_inputs(case)
    vn = case.get("value_norm", True)
    res = run_kv(inp, case["B"], case["T"], case["H"], case["scale"], case["key_norm"], torch.float32, vn)
    ref = oracle_kv(inp, case["H"], case["scale"], case["key_norm"], torch.float32, vn)
    compare(res, ref, torch.float32, case["B"] * case["T"])


def make(S, N, D, R, H, seed):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    return {"values": f(S, N, D), "key_weight": (f(R, D) / np.sqrt(D)).astype(np.float32),
            "query": (f(H, R // H) * 0.5).astype(np.float32), "grad_output": f(N, D)}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("S,N,D,R,value_norm", [
    (3, 300, 256, 64, True),     # partial last 128-row tile
    (17, 260, 2048, 64, True),   # BASELINE config-4 row shape (S=17, d=2048, R=64)
    (4, 129, 128, 32, False),    # no value norm, R=32
    (2, 1000, 512, 128, True),   # R=128, several tiles per source
])
def test_key_projection_matches_oracle(dtype, S, N, D, R, value_norm):
    """The projection alone: keys and the value inv-rms it saves."""
    from attnres_b200.ops import _kv_project

    inp = make(S, N, D, R, 1, seed=S * 7 + R)
    v = [torch.tensor(x, device="cuda").to(dtype) for x in inp["values"]]
    w = torch.tensor(inp["key_weight"], device="cuda").to(dtype)
    keys, inv = _kv_project(v, w, value_norm)
    torch.cuda.synchronize()
    ref_keys, ref_inv, _ = oracle._kv_keys(rounded(inp["values"], dtype), rounded(inp["key_weight"], dtype),
                                           value_norm, RMS_EPS)
    assert_close("keys", to_np(keys), ref_keys, dtype)
    if value_norm:
        assert_close("inv_rms", to_np(inv), ref_inv[..., 0], torch.float32)


@pytest.mark.parametrize("S,N,D,R,H", [(17, 150, 2048, 64, 1), (5, 200, 256, 64, 2)])
def test_kv_read_bf16(S, N, D, R, H):
    inp = make(S, N, D, R, H, seed=N)
    res = run_kv(inp, 1, N, H, 1.0 / np.sqrt(R // H), True, torch.bfloat16)
    ref = oracle_kv(inp, H, 1.0 / np.sqrt(R // H), True, torch.bfloat16)
    compare(res, ref, torch.bfloat16, N)


@pytest.mark.parametrize("H", [1, 2])
def test_kv_read_output_norm_bf16(H):
    """With the output normalised the read backward writes dV itself and the
    projection backward adds into it (read-modify-write path)."""
    inp = make(5, 150, 256, 64, H, seed=9 + H)
    res = run_kv(inp, 1, 150, H, 0.25, True, torch.bfloat16, normalize_output=True)
    ref = oracle_kv(inp, H, 0.25, True, torch.bfloat16, normalize_output=True)
    compare(res, ref, torch.bfloat16, 150, out_norm=True)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("S,N,D,H,value_norm", [
    (17, 300, 2048, 1, True),    # config-4 row shape, ragged last token tile
    (3, 1000, 256, 2, True),     # two heads, several token tiles per slice
    (4, 129, 384, 1, False),     # no value norm (coef = 0), three column slices
])
def test_kv_fused_projection_backward_matches_oracle(kernel_path, monkeypatch, dtype, S, N, D, H, value_norm):
    """The tensor-core projection backward (dn = dKs @ W in TMEM, dV written
    once, dW accumulated in TMEM) against the oracle, and against the cuBLAS
    dn + combine path it replaces."""
    if kernel_path != "auto":
        pytest.skip("one kernel path is enough for the projection backward")
    R = 64
    inp = make(S, N, D, R, H, seed=N + D)
    scale = 1.0 / np.sqrt(R // H)
    res = run_kv(inp, 1, N, H, scale, True, dtype, value_norm=value_norm)
    ref = oracle_kv(inp, H, scale, True, dtype, value_norm=value_norm)
    compare(res, ref, dtype, N)
    monkeypatch.setenv("ATTNRES_KV_BWD", "gemm")
    res_gemm = run_kv(inp, 1, N, H, scale, True, dtype, value_norm=value_norm)
    assert_close("dV (fused vs gemm)", res["dV"], res_gemm["dV"], dtype)
    assert_close("dW (fused vs gemm)", res["dW"], res_gemm["dW"], dtype, sum_terms=N)


def test_kv_fused_projection_backward_is_deterministic():
    import attnres_b200 as A

    S, B, T, D, R = 5, 2, 700, 512, 64
    torch.manual_seed(3)
    values = [torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    w = (torch.randn(R, D, device="cuda") / D ** 0.5).to(torch.bfloat16)
    q = torch.randn(1, R, device="cuda") * 0.02
    g = torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16)
    grads = []
    for _ in range(2):
        vs = [v.clone().requires_grad_(True) for v in values]
        ww = w.clone().requires_grad_(True)
        A.lrid_attention_residual_read_key_from_value(vs, ww, q, 1, 0.125, True).backward(g)
        grads.append((ww.grad.clone(), vs[2].grad.clone()))
    for a, b in zip(*grads):
        assert torch.equal(a, b)


@pytest.mark.parametrize("S,N,D,H,bias,dtype", [
    (17, 1000, 2048, 1, False, torch.bfloat16),   # config-4 rows: clusters of 4
    (32, 77, 1024, 4, False, torch.bfloat16),     # 32 sources, clusters of 2, ragged tile
    (5, 33, 2048, 2, True, torch.bfloat16),       # logit biases, one partial tile
    (3, 301, 4096, 2, True, torch.float16),       # clusters of 8, ragged last tile
])
def test_kv_one_kernel_forward_matches_two_pass(kernel_path, monkeypatch, S, N, D, H, bias, dtype):
    """The one-kernel key-from-value forward (projection, softmax and weighted
    sum with V read once) against the projection kernel followed by the read
    kernel: out, the saved keys, value inverse rms and softmax weights. The
    one-kernel call is made directly, so a shape it refused would fail here
    instead of silently comparing the two-kernel path with itself."""
    if kernel_path != "auto":
        pytest.skip("one kernel path is enough")
    from attnres_b200 import _native, ops as O

    torch.manual_seed(S + N)
    values = [torch.randn(1, N, D, device="cuda", dtype=dtype) for _ in range(S)]
    w = (torch.randn(64, D, device="cuda") / D ** 0.5).to(dtype)
    q = (torch.randn(H, 64 // H, device="cuda") * 0.5).to(dtype)
    b = torch.randn(S, device="cuda") if bias else None
    _native.device_status(reset=True)
    monkeypatch.setenv("ATTNRES_KV_FWD", "one")
    fused = O._kv_fused_forward(values, w, q, b, H, 0.25, True, True)
    assert fused is not None, "the one-kernel forward refused a shape it supports"
    o1, k1, i1, a1 = fused
    torch.cuda.synchronize()
    assert _native.device_status(reset=True) == 0
    monkeypatch.setenv("ATTNRES_KV_FWD", "twopass")
    o2, _, k2, i2, a2 = torch.ops.attnres.lrid_kv_read(values, w, q, None, None, b, H, 0.25, True, 0, True)
    torch.cuda.synchronize()
    assert_close("out", to_np(o1), to_np(o2), dtype)
    assert_close("keys", to_np(k1), to_np(k2), dtype)
    torch.testing.assert_close(i1, i2, rtol=1e-5, atol=0)
    # each path's weights are the softmax of its own saved keys (tight) ...
    for keys, alpha in ((k1, a1), (k2, a2)):
        torch.testing.assert_close(alpha, _alpha_from_keys(keys, q, b, H, 0.25), rtol=1e-4, atol=1e-6)
    # ... and the keys of the two paths may differ by one bf16 ulp (fp32 partial
    # sums added in another order), which moves a weight by up to ~0.5 %
    torch.testing.assert_close(a1, a2, rtol=1e-2, atol=1e-5)


def _alpha_from_keys(keys, q, bias, H, scale):
    """Softmax over sources of the per-head key-normed logits, in fp32, from
    saved keys [S, ..., R] -> [N, H, S]."""
    S, R = keys.size(0), keys.size(-1)
    k = keys.float().reshape(S, -1, H, R // H)
    k = k * torch.rsqrt(k.square().mean(-1, keepdim=True) + RMS_EPS)
    logits = (k * q.float().reshape(1, 1, H, R // H)).sum(-1) * scale
    if bias is not None:
        logits = logits + bias.float().reshape(S, 1, 1)
    return torch.softmax(logits, dim=0).permute(1, 2, 0)


@pytest.mark.parametrize("S,N,D,H,dtype,value_norm,bias", [
    (17, 300, 2048, 1, torch.bfloat16, True, False),   # config-4 row shape, ragged last token tile
    (6, 2500, 1024, 2, torch.float16, True, True),     # two heads, several tiles per slice group, biases
    (3, 513, 512, 1, torch.bfloat16, False, False),    # no value norm (coef = 0), two column slices
    (5, 700, 1024, 4, torch.bfloat16, True, True),     # four heads of 256 columns
    (4, 257, 2048, 8, torch.float16, True, False),     # eight heads
])
def test_kv_one_pass_backward_matches_oracle(kernel_path, monkeypatch, S, N, D, H, dtype, value_norm, bias):
    """The one-pass key-from-value backward (partial dots exchanged between the
    column slices of a token tile, dKs formed in-kernel, dV/dW on tcgen05)
    against the oracle, and against the read backward + projection backward it
    replaces (same saved forward tensors)."""
    if kernel_path != "auto":
        pytest.skip("one kernel path is enough for the one-pass backward")
    import attnres_b200  # noqa: F401

    ops = torch.ops.attnres
    R = 64
    inp = make(S, N, D, R, H, seed=S * N + D + H)
    scale = 1.0 / np.sqrt(R // H)
    vals = [dev_rows(v, 1, N, dtype, requires_grad=False) for v in inp["values"]]
    w = torch.tensor(inp["key_weight"], device="cuda").to(dtype)
    q = torch.tensor(inp["query"], device="cuda").to(dtype)
    g = dev_rows(inp["grad_output"], 1, N, dtype, requires_grad=False)
    b = torch.log(torch.arange(1, S + 1, device="cuda", dtype=torch.float32)) * 0.7 if bias else None
    out, oinv, keys, vinv, alpha = ops.lrid_kv_read(vals, w, q, None, None, b, H, scale, True, 0, value_norm)

    def bwd(path):
        monkeypatch.setenv("ATTNRES_KV_BWD", path)
        r = ops.lrid_kv_read_backward(vals, w, keys, vinv, alpha, q, None, None, b, g, out, oinv, H, scale, True,
                                      0, value_norm)
        torch.cuda.synchronize()
        return {"dV": np.stack([to_np(x).reshape(N, D) for x in r[0]]), "dW": to_np(r[1]),
                "dq": to_np(r[2]).reshape(-1), "dbias": to_np(r[5]) if bias else None}

    one, two = bwd("one"), bwd("tc")
    kw = {"logit_bias": to_np(b)} if bias else {}
    v, wr = rounded(inp["values"], dtype), rounded(inp["key_weight"], dtype)
    ref = oracle.lrid_kv_backward(v, wr, H, scale, True, rounded(inp["grad_output"], dtype), value_norm=value_norm,
                                  value_eps=RMS_EPS, query=rounded(inp["query"], dtype), **kw)
    assert_close("dV", one["dV"], ref["dV"], dtype)
    assert_close("dW", one["dW"], ref["dW"], dtype, sum_terms=N)
    assert_close("dq", one["dq"], ref["dq"], dtype, sum_terms=N)
    assert_close("dV (one pass vs two kernels)", one["dV"], two["dV"], dtype)
    assert_close("dW (one pass vs two kernels)", one["dW"], two["dW"], dtype, sum_terms=N)
    assert_close("dq (one pass vs two kernels)", one["dq"], two["dq"], dtype, sum_terms=N)
    if bias:
        assert_close("dbias", one["dbias"], ref["dbias"], dtype, sum_terms=N)
        assert_close("dbias (one pass vs two kernels)", one["dbias"], two["dbias"], dtype, sum_terms=N)
