"""Parity at the full BASELINE sizes of configs 3 and 4 (bf16).

The per-token outputs do not depend on the batch size, but the parameter
gradients do: dq / d(gate) (config 3) and dW_k / dq (config 4) are fp32 sums
over every token row (2.2 million rows x sources for dW_k), reduced per CTA and
then in a fixed order. At these sizes (32768 and 131072 tokens) they are
compared with a float64 PyTorch composition of the same read, computed in
token chunks on the GPU, at the bf16 tolerance (rtol 2e-2, atol 1e-2 of the
largest entry), and out / dV / dK (config 3) and out / dV (config 4) on token
slices at both ends of the batch against the fp64 oracle.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import RMS_EPS, assert_close, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu

CHUNK = 4096  # tokens per float64 reference chunk (about 1 GB of values at config 4)


def _slices(n):
    return (slice(0, 64), slice(n - 64, n))


def _read64(V, K, q, H, scale, gate=None, qd=None):
    """float64 LRID read of one token chunk: V [S, n, d], K [S, n, R], static
    query q [H, dk] (+ gate [H] * dynamic query [n, H, dk]); key rms norm with
    the fp32 eps (F.rms_norm's for 16-bit inputs)."""
    S, n, d = V.shape
    dk = K.shape[-1] // H
    Kh = K.reshape(S, n, H, dk)
    Kh = Kh * torch.rsqrt(Kh.pow(2).mean(-1, keepdim=True) + RMS_EPS)
    qq = q.reshape(1, H, dk) + (gate.reshape(1, H, 1) * qd if qd is not None else 0)
    logits = (Kh * qq.unsqueeze(0)).sum(-1) * scale  # [S, n, H]
    a = torch.softmax(logits, dim=0)
    return torch.einsum("snh,snhe->nhe", a, V.reshape(S, n, H, d // H)).reshape(n, d)


def test_config3_full_size_gated_read():
    ops = torch.ops.attnres
    import attnres_b200  # noqa: F401

    S, N, D, R, H, scale = 13, 32768, 2048, 64, 4, 0.25
    g_ = torch.Generator(device="cuda").manual_seed(31)
    bf = torch.bfloat16
    values = [torch.randn(1, N, D, device="cuda", dtype=bf, generator=g_) for _ in range(S)]
    keys = [torch.randn(1, N, R, device="cuda", dtype=bf, generator=g_) for _ in range(S)]
    qs = (torch.randn(H, R // H, device="cuda", generator=g_) * 0.02).to(bf)
    gate = torch.full((H,), 0.1, device="cuda", dtype=bf)
    qd = torch.randn(1, N, H, R // H, device="cuda", dtype=bf, generator=g_)
    g = torch.randn(1, N, D, device="cuda", dtype=bf, generator=g_)

    def run(sl):
        vs = [v[:, sl] for v in values]
        ks = [k[:, sl] for k in keys]
        out, inv = ops.lrid_read(vs, ks, qs, gate, qd[:, sl], None, H, scale, True, 0)
        r = ops.lrid_read_backward(vs, ks, qs, gate, qd[:, sl], None, g[:, sl], out, inv, H, scale, True, 0)
        return out, r

    out, (dV, dK, dq, dgate, dqd, _) = run(slice(0, N))
    q64 = qs.double().requires_grad_(True)
    g64 = gate.double().requires_grad_(True)
    for c in range(0, N, CHUNK):
        sl = slice(c, c + CHUNK)
        V = torch.stack([v[0, sl] for v in values]).double()
        K = torch.stack([k[0, sl] for k in keys]).double()
        o = _read64(V, K, q64, H, scale, g64, qd[0, sl].double())
        (o * g[0, sl].double()).sum().backward()
    assert_close("dq", to_np(dq).reshape(-1), to_np(q64.grad).reshape(-1), bf, sum_terms=N)
    assert_close("dgate", to_np(dgate).reshape(-1), to_np(g64.grad).reshape(-1), bf, sum_terms=N)
    for sl in _slices(N):
        v = np.stack([to_np(x[0, sl]) for x in values])
        k = np.stack([to_np(x[0, sl]) for x in keys])
        kw = dict(query=to_np(qs), gate=to_np(gate), query_dynamic=to_np(qd[0, sl]))
        ref_out = oracle.lrid_forward(v, k, H, scale, True, **kw)[0]
        ref = oracle.lrid_backward(v, k, H, scale, True, to_np(g[0, sl]), **kw)
        assert_close("out", to_np(out[0, sl]), ref_out, bf)
        assert_close("dV", np.stack([to_np(x[0, sl]) for x in dV]), ref["dV"], bf)
        assert_close("dK", np.stack([to_np(x[0, sl]) for x in dK]), ref["dK"], bf)
        assert_close("dq_dynamic", to_np(dqd.reshape(N, R)[sl]), ref["dq_dynamic"], bf)


def test_config4_full_size_key_from_value_read():
    ops = torch.ops.attnres
    import attnres_b200  # noqa: F401

    S, N, D, R, H, scale = 17, 131072, 2048, 64, 1, 0.125
    g_ = torch.Generator(device="cuda").manual_seed(41)
    bf = torch.bfloat16
    values = [torch.randn(1, N, D, device="cuda", dtype=bf, generator=g_) for _ in range(S)]
    w = (torch.randn(R, D, device="cuda", generator=g_) / D ** 0.5).to(bf)
    q = (torch.randn(H, R // H, device="cuda", generator=g_) * 0.02).to(bf)
    g = torch.randn(1, N, D, device="cuda", dtype=bf, generator=g_)

    def run(sl):
        vs = [v[:, sl] for v in values]
        out, inv, keys, vinv, alpha = ops.lrid_kv_read(vs, w, q, None, None, None, H, scale, True, 0, True)
        r = ops.lrid_kv_read_backward(vs, w, keys, vinv, alpha, q, None, None, None, g[:, sl], out, inv, H, scale,
                                      True, 0, True)
        return out, r

    out, r = run(slice(0, N))
    dV, dW, dq = r[0], r[1], r[2]
    w64 = w.double().requires_grad_(True)
    q64 = q.double().requires_grad_(True)
    for c in range(0, N, CHUNK):
        sl = slice(c, c + CHUNK)
        V = torch.stack([v[0, sl] for v in values]).double()
        nhat = V * torch.rsqrt(V.pow(2).mean(-1, keepdim=True) + RMS_EPS)
        o = _read64(V, nhat @ w64.t(), q64, H, scale)
        (o * g[0, sl].double()).sum().backward()
        del V, nhat, o
    assert_close("dW_k", to_np(dW), to_np(w64.grad), bf, sum_terms=N)
    assert_close("dq", to_np(dq).reshape(-1), to_np(q64.grad).reshape(-1), bf, sum_terms=N)
    eps = RMS_EPS
    for sl in _slices(N):
        v = np.stack([to_np(x[0, sl]) for x in values])
        kw = dict(query=to_np(q))
        ref_out = oracle.lrid_kv_forward(v, to_np(w), H, scale, True, value_eps=eps, **kw)[0]
        ref = oracle.lrid_kv_backward(v, to_np(w), H, scale, True, to_np(g[0, sl]), value_eps=eps, **kw)
        assert_close("out", to_np(out[0, sl]), ref_out, bf)
        assert_close("dV", np.stack([to_np(x[0, sl]) for x in dV]), ref["dV"], bf)
