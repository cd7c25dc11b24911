"""GPU parity of the LRID read (forward + backward) against the CPU oracle.

Mirrors the reference's CUDA parity tests (tests/test_attnres_ops.py:898-1030)
and extends them to the BASELINE configurations, the gated hybrid query,
logit biases, output norms, S > 16 and ragged/edge layouts.
"""
import numpy as np
import pytest
import torch

from cases import CASES, case_inputs
from gpu_helpers import RMS_EPS, assert_close, dev_rows, rounded, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True, params=["auto", "simt"])
def kernel_path(request, monkeypatch):
    """Run every LRID test on both kernels: `auto` picks the streaming warp
    pipeline (bulk copies into per-warp rings) where the row layout allows it,
    `simt` forces the register-streaming kernel that serves every layout."""
    monkeypatch.setenv("ATTNRES_B200_PATH", request.param)
    yield request.param
    if request.param != "simt":
        from attnres_b200 import _native

        assert _native.device_status(reset=True) == 0, "a pipeline kernel abandoned a bounded wait"


def _ops():
    import attnres_b200

    return attnres_b200


def _norm_mode(case):
    if not case.get("normalize_output"):
        return oracle.NORM_NONE
    return oracle.NORM_PER_HEAD if case["H"] == 1 else oracle.NORM_ROW


def run_lrid(inp, B, T, H, scale, key_norm, query_kind, dtype, normalize_output=False, bias=False,
             api="public"):
    """Forward + backward of the CUDA path; returns numpy out and grads."""
    ops = _ops()
    S = inp["values"].shape[0]
    values = [dev_rows(v, B, T, dtype) for v in inp["values"]]
    keys = [dev_rows(k, B, T, dtype) for k in inp["keys"]]
    g = dev_rows(inp["grad_output"], B, T, dtype, requires_grad=False)
    res = {}
    biases = None
    if bias:
        biases = [torch.tensor(float(b), device="cuda", requires_grad=True) for b in inp["logit_bias"]]
    if query_kind == "static":
        q = torch.tensor(inp["query"], device="cuda", dtype=torch.float32, requires_grad=True)
        out = ops.lrid_attention_residual_read(values, keys, q, H, scale, key_norm,
                                               normalize_output=normalize_output,
                                               source_logit_biases=biases)
        params = [("dq", q)]
    elif query_kind == "dynamic":
        q = torch.tensor(inp["query_dynamic"].reshape(B, T, H, -1), device="cuda", dtype=dtype,
                         requires_grad=True)
        out = ops.lrid_attention_residual_read(values, keys, q, H, scale, key_norm,
                                               normalize_output=normalize_output,
                                               source_logit_biases=biases)
        params = [("dq", q)]
    else:
        qs = torch.tensor(inp["query"], device="cuda", dtype=torch.float32, requires_grad=True)
        gate = torch.tensor(inp["gate"], device="cuda", dtype=torch.float32, requires_grad=True)
        qd = torch.tensor(inp["query_dynamic"].reshape(B, T, H, -1), device="cuda", dtype=dtype,
                          requires_grad=True)
        out = ops.lrid_attention_residual_read_gated(values, keys, qs, gate, qd, H, scale, key_norm,
                                                     normalize_output=normalize_output,
                                                     source_logit_biases=biases)
        params = [("dq", qs), ("dgate", gate), ("dq_dynamic", qd)]
    out.backward(g)
    torch.cuda.synchronize()
    res["out"] = to_np(out).reshape(B * T, -1)
    res["dV"] = np.stack([to_np(v.grad).reshape(B * T, -1) for v in values])
    res["dK"] = np.stack([to_np(k.grad).reshape(B * T, -1) for k in keys])
    for name, p in params:
        gr = to_np(p.grad)
        res[name] = gr.reshape(B * T, -1) if (name == "dq_dynamic" or query_kind == "dynamic") else gr.reshape(-1)
    if biases is not None:
        res["dbias"] = np.array([b.grad.item() for b in biases])
    return res


def oracle_lrid(inp, H, scale, key_norm, query_kind, dtype, norm, bias):
    vals = rounded(inp["values"], dtype)
    keys = rounded(inp["keys"], dtype)
    g = rounded(inp["grad_output"], dtype)
    kw = dict(output_norm=norm, logit_bias=inp["logit_bias"] if bias else None,
              output_eps=RMS_EPS)
    if query_kind == "static":
        kw["query"] = rounded(inp["query"], dtype)
    elif query_kind == "dynamic":
        kw["query_dynamic"] = rounded(inp["query_dynamic"], dtype)
    else:
        kw.update(query=rounded(inp["query"], dtype), gate=rounded(inp["gate"], dtype),
                  query_dynamic=rounded(inp["query_dynamic"], dtype))
    out = oracle.lrid_forward(vals, keys, H, scale, key_norm, **kw)[0]
    grads = oracle.lrid_backward(vals, keys, H, scale, key_norm, g, **kw)
    grads["out"] = out
    if query_kind == "dynamic":
        grads["dq"] = grads["dq"]
    return grads


def compare(res, ref, dtype, n_tokens, out_norm=False):
    """With the output normalised, the 16-bit backward reads the saved 16-bit
    normed output (as the reference's fused backward does), so dV / dK carry an
    error proportional to their own scale: their absolute floor scales too."""
    assert_close("out", res["out"], ref["out"], dtype)
    assert_close("dV", res["dV"], ref["dV"], dtype, scaled_atol=out_norm)
    assert_close("dK", res["dK"], ref["dK"], dtype, scaled_atol=out_norm)
    for name in ("dq", "dgate", "dq_dynamic", "dbias"):
        if name in ref:
            summed = name in ("dq", "dgate", "dbias") and ref[name].ndim == 1
            assert_close(name, res[name].reshape(ref[name].shape), ref[name], dtype,
                         sum_terms=n_tokens if summed else 1)


LRID_CASES = [c for c in CASES if c["kind"] == "lrid"]


@pytest.mark.parametrize("case", LRID_CASES, ids=[c["name"] for c in LRID_CASES])
def test_lrid_golden_cases_fp32(case):
    inp = case_inputs(case)
    B, T = case["B"], case["T"]
    res = run_lrid(inp, B, T, case["H"], case["scale"], case["key_norm"], case["query"], torch.float32,
                   case.get("normalize_output", False), case.get("bias", False))
    ref = oracle_lrid(inp, case["H"], case["scale"], case["key_norm"], case["query"], torch.float32,
                      _norm_mode(case), case.get("bias", False))
    compare(res, ref, torch.float32, B * T)


def make_inputs(S, N, D, R, H, seed, query_std=1.0):
    rng = np.random.default_rng(seed)
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    return {
        "values": f(S, N, D), "keys": f(S, N, R), "query": f(H, R // H) * np.float32(query_std),
        "query_dynamic": f(N, H, R // H), "gate": np.full(H, 0.1, np.float32),
        "logit_bias": rng.standard_normal(S).astype(np.float32), "grad_output": f(N, D),
    }


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("query_kind", ["static", "dynamic", "gated"])
def test_lrid_dtypes_and_query_modes(dtype, query_kind):
    S, B, T, D, R, H = 7, 2, 37, 256, 64, 2
    seed = 100 + 10 * [torch.bfloat16, torch.float16, torch.float32].index(dtype) + ["static", "dynamic", "gated"].index(query_kind)
    inp = make_inputs(S, B * T, D, R, H, seed=seed)
    res = run_lrid(inp, B, T, H, 0.125, True, query_kind, dtype, bias=True)
    ref = oracle_lrid(inp, H, 0.125, True, query_kind, dtype, oracle.NORM_NONE, True)
    compare(res, ref, dtype, B * T)


@pytest.mark.parametrize("name,S,D,R,H,scale,query_kind,norm", [
    ("config2_lrid_h1", 9, 1024, 64, 1, 1 / 8, "static", False),
    ("config2_lrid_h1_outnorm", 9, 1024, 64, 1, 1 / 8, "static", True),
    ("config3_gated_h4", 13, 2048, 64, 4, 1 / 4, "gated", False),
    ("config3_gated_h4_outnorm", 13, 2048, 64, 4, 1 / 4, "gated", True),
    ("model_h2_outnorm", 13, 1024, 64, 2, 1 / 4, "static", True),
    ("sources17", 17, 512, 64, 2, 0.25, "static", True),
    ("sources64", 64, 128, 32, 1, 0.25, "static", False),
    ("heads3", 5, 96, 24, 3, 0.5, "static", True),
    ("dk512", 3, 1024, 512, 1, 1.0, "static", False),
    ("odd_width", 4, 100, 20, 2, 0.5, "dynamic", True),
])
def test_lrid_shapes_bf16(name, S, D, R, H, scale, query_kind, norm):
    B, T = 1, 67
    inp = make_inputs(S, B * T, D, R, H, seed=len(name) * 7 + S, query_std=0.02 if "config" in name else 1.0)
    res = run_lrid(inp, B, T, H, scale, True, query_kind, torch.bfloat16, normalize_output=norm)
    ref = oracle_lrid(inp, H, scale, True, query_kind, torch.bfloat16,
                      (oracle.NORM_PER_HEAD if H == 1 else oracle.NORM_ROW) if norm else oracle.NORM_NONE, False)
    compare(res, ref, torch.bfloat16, B * T, out_norm=norm)


def test_lrid_config3_many_tokens_per_cta():
    """BASELINE config-3 row shape with enough tokens that every persistent CTA
    walks its stage ring several times (single-token stages of 57 KB leave
    only a few stages, fewer than the consumer warps a CTA could run)."""
    S, B, T, D, R, H = 13, 1, 1500, 2048, 64, 4
    inp = make_inputs(S, B * T, D, R, H, seed=77, query_std=0.02)
    res = run_lrid(inp, B, T, H, 0.25, True, "gated", torch.bfloat16)
    ref = oracle_lrid(inp, H, 0.25, True, "gated", torch.bfloat16, oracle.NORM_NONE, False)
    compare(res, ref, torch.bfloat16, B * T)


def test_lrid_strided_and_misaligned_sources():
    """Keys as a column slice of a wider row (output-tail keys,
    tests/test_attnres_ops.py:934-972) and values offset by one element, which
    forces the element-wise (unpacked) layout."""
    ops = _ops()
    S, B, T, D, R, H = 5, 2, 9, 128, 32, 2
    rng = np.random.default_rng(5)
    wide = torch.tensor(rng.standard_normal((S, B, T, D + 1)), dtype=torch.float32, device="cuda")
    values = [wide[s, :, :, 1:] for s in range(S)]  # misaligned by 4 bytes, row stride D+1
    keys = [wide[s, :, :, -R:] for s in range(S)]
    q = torch.tensor(rng.standard_normal((H, R // H)), dtype=torch.float32, device="cuda")
    out = ops.lrid_attention_residual_read(values, keys, q, H, 0.25, True)
    torch.cuda.synchronize()
    v = np.stack([to_np(x).reshape(B * T, D) for x in values])
    k = np.stack([to_np(x).reshape(B * T, R) for x in keys])
    ref = oracle.lrid_forward(v, k, H, 0.25, True, query=to_np(q))[0]
    assert_close("out", to_np(out).reshape(B * T, D), ref, torch.float32)


@pytest.mark.parametrize("N", [1, 2, 3, 255, 257])
def test_lrid_ragged_token_counts(N):
    S, D, R, H = 6, 256, 64, 1
    inp = make_inputs(S, N, D, R, H, seed=N)
    res = run_lrid(inp, 1, N, H, 0.125, True, "static", torch.bfloat16)
    ref = oracle_lrid(inp, H, 0.125, True, "static", torch.bfloat16, oracle.NORM_NONE, False)
    compare(res, ref, torch.bfloat16, N)


def test_lrid_zero_tokens_and_single_source():
    ops = _ops()
    v = [torch.zeros(0, 0, 64, device="cuda", requires_grad=True) for _ in range(3)]
    k = [torch.zeros(0, 0, 16, device="cuda", requires_grad=True) for _ in range(3)]
    q = torch.randn(1, 16, device="cuda", requires_grad=True)
    out = ops.lrid_attention_residual_read(v, k, q, 1, 0.25, True)
    out.sum().backward()
    assert out.shape == (0, 0, 64)
    assert torch.all(q.grad == 0)
    one = torch.randn(2, 3, 64, device="cuda")
    assert ops.lrid_attention_residual_read([one], [torch.randn(2, 3, 16, device="cuda")], q, 1, 0.25, True) is one


def test_lrid_too_many_sources_raises():
    ops = _ops()
    v = [torch.randn(1, 2, 32, device="cuda") for _ in range(65)]
    k = [torch.randn(1, 2, 8, device="cuda") for _ in range(65)]
    with pytest.raises(RuntimeError, match="64"):
        ops.lrid_attention_residual_read(v, k, torch.randn(1, 8, device="cuda"), 1, 1.0, True)


def test_lrid_cpu_tensors_fail_loudly():
    ops = _ops()
    v = [torch.randn(1, 2, 32) for _ in range(3)]
    k = [torch.randn(1, 2, 8) for _ in range(3)]
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.lrid_attention_residual_read(v, k, torch.randn(1, 8), 1, 1.0, True)


def test_lrid_backward_is_deterministic():
    ops = _ops()
    S, B, T, D, R, H = 9, 4, 1000, 1024, 64, 1
    torch.manual_seed(0)
    values = [torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    keys = [torch.randn(B, T, R, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    q = torch.randn(H, R // H, device="cuda") * 0.02
    g = torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16)
    outs = []
    for _ in range(2):
        vs = [v.clone().requires_grad_(True) for v in values]
        ks = [k.clone().requires_grad_(True) for k in keys]
        qq = q.clone().requires_grad_(True)
        ops.lrid_attention_residual_read(vs, ks, qq, H, 0.125, True).backward(g)
        outs.append((qq.grad.clone(), vs[3].grad.clone(), ks[5].grad.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_lrid_query_grad_is_additive_over_token_shards():
    """Size-independent property at the full BASELINE config-2 size: the fp32
    query gradient of the whole batch equals the sum over token shards (each
    shard run on its own), and the per-token outputs equal the oracle on a
    slice at each end of the batch. Calls the attnres::lrid_read ops directly,
    so dq is compared before the cast to the bf16 query dtype."""
    ops = torch.ops.attnres
    _ops()
    S, B, T, D, R, H = 9, 8, 2048, 1024, 64, 1
    torch.manual_seed(1)
    values = [torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    keys = [torch.randn(B, T, R, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    q0 = (torch.randn(H, R // H, device="cuda") * 0.02).to(torch.bfloat16)
    g = torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16)

    def run(sl):
        vs = [v[sl] for v in values]
        ks = [k[sl] for k in keys]
        out, inv = ops.lrid_read(vs, ks, q0, None, None, None, H, 0.125, True, 0)
        res = ops.lrid_read_backward(vs, ks, q0, None, None, None, g[sl], out, inv, H, 0.125, True, 0)
        return out, res[2].double()

    out_full, dq_full = run(slice(0, B))
    dq_sum = sum(run(slice(i, i + 2))[1] for i in range(0, B, 2))
    # fp32 partial sums over 16384 tokens x 9 sources: allow 1e-5 of the scale
    torch.testing.assert_close(dq_full, dq_sum, rtol=1e-5, atol=1e-5 * float(dq_full.abs().max()))
    for sl in (slice(0, 1), slice(B - 1, B)):
        v = np.stack([to_np(x[sl]).reshape(-1, D) for x in values])
        k = np.stack([to_np(x[sl]).reshape(-1, R) for x in keys])
        ref = oracle.lrid_forward(v, k, H, 0.125, True, query=to_np(q0))[0]
        assert_close("out", to_np(out_full[sl]).reshape(-1, D), ref, torch.bfloat16)


def test_reference_library_op_with_aux_and_output_norm():
    """attnres::lrid_read_list / _backward with the reference's schema
    (attnres_ops.py:4636-4847): per-head output norm, saved alpha / key inv-rms."""
    S, B, T, D, R, H = 6, 2, 7, 128, 32, 1
    inp = make_inputs(S, B * T, D, R, H, seed=3)
    values = [dev_rows(v, B, T, torch.float32) for v in inp["values"]]
    keys = [dev_rows(k, B, T, torch.float32) for k in inp["keys"]]
    q = torch.tensor(inp["query"], device="cuda", requires_grad=True)
    out, inv, alpha, kinv = torch.ops.attnres.lrid_read_list(values, keys, q, H, 0.25, True, True, True)
    g = dev_rows(inp["grad_output"], B, T, torch.float32, requires_grad=False)
    out.backward(g)
    torch.cuda.synchronize()
    r_out, r_inv, r_alpha, r_kinv = oracle.lrid_forward(inp["values"], inp["keys"], H, 0.25, True,
                                                        query=inp["query"], output_norm=oracle.NORM_PER_HEAD)
    assert_close("out", to_np(out).reshape(B * T, D), r_out, torch.float32)
    assert_close("inv", to_np(inv), r_inv, torch.float32)
    assert_close("alpha", to_np(alpha), r_alpha, torch.float32)
    assert_close("kinv", to_np(kinv), r_kinv, torch.float32)
    grads = oracle.lrid_backward(inp["values"], inp["keys"], H, 0.25, True, inp["grad_output"],
                                 query=inp["query"], output_norm=oracle.NORM_PER_HEAD)
    assert_close("dq", to_np(q.grad).reshape(-1), grads["dq"], torch.float32, sum_terms=B * T)
    assert_close("dV0", to_np(values[0].grad).reshape(B * T, D), grads["dV"][0], torch.float32)
    assert_close("dK2", to_np(keys[2].grad).reshape(B * T, R), grads["dK"][2], torch.float32)


def test_lrid_forward_token_schedule_static_equals_dynamic(kernel_path, monkeypatch):
    """The streaming forward claims tokens from a global counter (dynamic
    schedule); its rows must match the static round-robin schedule bit for bit,
    across repeated launches (the counter rewinds itself) and graph replays."""
    if kernel_path != "auto":
        pytest.skip("schedule applies to the streaming kernel (auto path)")
    ops = _ops()
    S, B, T, D, R, H = 9, 3, 2731, 1024, 64, 1
    torch.manual_seed(1)
    values = [torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    keys = [torch.randn(B, T, R, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    q = torch.randn(H, R // H, device="cuda") * 0.02

    def fwd():
        return ops.lrid_attention_residual_read(values, keys, q, H, 0.125, True)

    monkeypatch.setenv("ATTNRES_STREAM_SCHEDULE", "static")
    ref = fwd()
    monkeypatch.setenv("ATTNRES_STREAM_SCHEDULE", "dynamic")
    for _ in range(3):
        assert torch.equal(fwd(), ref)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        fwd()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        out = fwd()
    for _ in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


def test_lrid_graph_replays_and_eager_launches_on_two_streams(kernel_path):
    """Forward and backward captured in a CUDA graph replay on one stream while
    eager launches of other inputs run on a second stream, many times over:
    each captured launch owns its token / CTA counters, so neither side skips
    or repeats rows. Results must equal the launches run alone, bit for bit
    (the backward's parameter-gradient sums have a fixed order)."""
    if kernel_path != "auto":
        pytest.skip("counter slots belong to the streaming kernels (auto path)")
    ops = torch.ops.attnres
    _ops()
    S, N, D, R, H = 9, 5000, 1024, 64, 1
    torch.manual_seed(7)

    def make():
        v = [torch.randn(1, N, D, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
        k = [torch.randn(1, N, R, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
        g = torch.randn(1, N, D, device="cuda", dtype=torch.bfloat16)
        return v, k, g

    q = (torch.randn(H, R // H, device="cuda") * 0.02).to(torch.bfloat16)
    a, b = make(), make()

    def step(x):
        v, k, g = x
        out, inv = ops.lrid_read(v, k, q, None, None, None, H, 0.125, True, 0)
        res = ops.lrid_read_backward(v, k, q, None, None, None, g, out, inv, H, 0.125, True, 0)
        return out, res[2], res[0][4]

    ref_a, ref_b = step(a), step(b)
    sa, sb = torch.cuda.Stream(), torch.cuda.Stream()
    with torch.cuda.stream(sa):
        step(a)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=sa):
        got_a = step(a)
    torch.cuda.synchronize()
    for _ in range(40):
        with torch.cuda.stream(sa):
            graph.replay()
        with torch.cuda.stream(sb):
            got_b = step(b)
        torch.cuda.synchronize()
        for x, y in zip(got_a, ref_a):
            assert torch.equal(x, y)
        for x, y in zip(got_b, ref_b):
            assert torch.equal(x, y)


def test_lrid_output_norm_read_matches_the_unnormed_read_then_rms_norm(kernel_path):
    """The model's default read (normalize_output with H == 1, model.py:2238-2244)
    against the composition it fuses: the plain read, then F.rms_norm of the
    value-dtype output, at the config-2 row shape."""
    ops = _ops()
    S, B, T, D, R, H = 9, 2, 1500, 1024, 64, 1
    torch.manual_seed(11)
    values = [torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    keys = [torch.randn(B, T, R, device="cuda", dtype=torch.bfloat16) for _ in range(S)]
    q = torch.randn(H, R // H, device="cuda") * 0.02
    g = torch.randn(B, T, D, device="cuda", dtype=torch.bfloat16)
    grads = []
    for fused in (True, False):
        vs = [v.clone().requires_grad_(True) for v in values]
        ks = [k.clone().requires_grad_(True) for k in keys]
        qq = q.clone().requires_grad_(True)
        if fused:
            out = ops.lrid_attention_residual_read(vs, ks, qq, H, 0.125, True, normalize_output=True)
        else:
            out = ops.lrid_attention_residual_read(vs, ks, qq, H, 0.125, True)
            out = torch.nn.functional.rms_norm(out.float(), (D,), eps=RMS_EPS)
        out.float().backward(g.float())
        grads.append((out.float(), qq.grad.float(), vs[2].grad.float(), ks[6].grad.float()))
    for name, x, y in zip(("out", "dq", "dV2", "dK6"), *grads):
        assert_close(name, to_np(x), to_np(y), torch.bfloat16, sum_terms=B * T if name == "dq" else 1)
