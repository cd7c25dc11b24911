"""Parity at the full BASELINE sizes of configs 3 and 4 (bf16).

The per-token outputs do not depend on the batch size, but the parameter
gradients do: dq / d(gate) (config 3) and dW_k / dq (config 4) are fp32 sums
over every token row, reduced per CTA and then in a fixed order. At these
sizes (32768 and 131072 tokens) the tests check a size-independent property of
those sums -- the whole batch equals the fp64 sum of its token shards, each
run on its own -- and compare out / dV / dK (config 3) and out / dV (config 4)
on token slices at both ends of the batch against the fp64 oracle.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import assert_close, to_np
from oracle import oracle

pytestmark = pytest.mark.gpu

# fp32 sums over ~10^5 - 10^6 terms, accumulated per CTA in a different order
# for the whole batch and for each shard: allow 2e-5 of the largest entry
SUM_RTOL, SUM_ATOL_REL = 1e-5, 2e-5


def _slices(n):
    return (slice(0, 64), slice(n - 64, n))


def _assert_additive(name, full, shards):
    total = sum(shards)
    torch.testing.assert_close(full, total, rtol=SUM_RTOL, atol=SUM_ATOL_REL * float(full.abs().max()),
                               msg=lambda m: f"{name}: {m}")


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
    shards = [run(slice(i, i + N // 4))[1] for i in range(0, N, N // 4)]
    _assert_additive("dq", dq.double(), [r[2].double() for r in shards])
    _assert_additive("dgate", dgate.double(), [r[3].double() for r in shards])
    for sl in _slices(N):
        v = np.stack([to_np(x[0, sl]) for x in values])
        k = np.stack([to_np(x[0, sl]) for x in keys])
        kw = dict(query=to_np(qs), gate=to_np(gate), query_dynamic=to_np(qd[0, sl]))
        ref_out = oracle.lrid_forward(v, k, H, scale, True, **kw)[0]
        ref = oracle.lrid_backward(v, k, H, scale, True, to_np(g[0, sl]), **kw)
        assert_close("out", to_np(out[0, sl]), ref_out, bf)
        assert_close("dV", np.stack([to_np(x[0, sl]) for x in dV]), ref["dV"], bf)
        assert_close("dK", np.stack([to_np(x[0, sl]) for x in dK]), ref["dK"], bf)
        assert_close("dq_dynamic", to_np(dqd.reshape(N, H, R // H)[sl]), ref["dq_dynamic"], bf)


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
    shard_dW, shard_dq = [], []
    for i in range(0, N, N // 4):
        rs = run(slice(i, i + N // 4))[1]
        shard_dW.append(rs[1].double())
        shard_dq.append(rs[2].double())
    _assert_additive("dW_k", dW.double(), shard_dW)
    _assert_additive("dq", dq.double(), shard_dq)
    eps = float(torch.finfo(bf).eps)
    for sl in _slices(N):
        v = np.stack([to_np(x[0, sl]) for x in values])
        kw = dict(query=to_np(q))
        ref_out = oracle.lrid_kv_forward(v, to_np(w), H, scale, True, value_eps=eps, **kw)[0]
        ref = oracle.lrid_kv_backward(v, to_np(w), H, scale, True, to_np(g[0, sl]), value_eps=eps, **kw)
        assert_close("out", to_np(out[0, sl]), ref_out, bf)
        assert_close("dV", np.stack([to_np(x[0, sl]) for x in dV]), ref["dV"], bf)
