"""attnres_lrid_backward_noalloc against attnres_lrid_backward, through the C ABI.

The no-alloc entry point serves callers that cannot allocate device memory or
pass a workspace (allocator callbacks, plugins handed fixed buffers, runtimes
that pre-reserve all device memory): it keeps the backward's scratch in a
static device array instead. This file is named to be collected last, so a
run that stops at the first failure has already run every other test; it also
passes when run alone in a fresh process.
"""
import ctypes

import pytest
import torch

from gpu_helpers import RMS_EPS, assert_close
from attnres_b200 import _native as N

pytestmark = pytest.mark.gpu

F32_EPS = float(torch.finfo(torch.float32).eps)


def _inputs(S=9, n=3000, d=1024, R=64, H=1, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    values = [torch.randn(n, d, device="cuda", dtype=dtype, generator=g) for _ in range(S)]
    keys = [torch.randn(n, R, device="cuda", dtype=dtype, generator=g) for _ in range(S)]
    query = (torch.randn(H, R // H, device="cuda", generator=g) * 0.02).to(dtype)
    grad = torch.randn(n, d, device="cuda", dtype=dtype, generator=g)
    bias = torch.randn(S, device="cuda", generator=g)
    return values, keys, query, grad, bias


def _call(noalloc, values, keys, query, grad, bias, H, scale=0.125):
    """One backward through the C ABI; returns (dV list, dK list, dq, dbias)."""
    L = N.load()
    S, n, d, R = len(values), values[0].shape[0], values[0].shape[1], keys[0].shape[1]
    dt = {torch.float32: N.DTYPE_F32, torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16}[values[0].dtype]
    dV = [torch.empty_like(v) for v in values]
    dK = [torch.empty_like(k) for k in keys]
    dq = torch.empty(H, R // H, device="cuda", dtype=torch.float32)
    db = torch.empty(S, device="cuda", dtype=torch.float32)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    common = [
        S, n, d, R, H, dt,
        N.ptr_array([v.data_ptr() for v in values]), N.i64_array([d] * S),
        N.ptr_array([k.data_ptr() for k in keys]), N.i64_array([R] * S),
        N.QUERY_STATIC, p(query), None, None, scale, 1, F32_EPS, p(bias), N.NORM_NONE,
        RMS_EPS, p(grad), None, None,
        N.ptr_array([t.data_ptr() for t in dV]), N.ptr_array([t.data_ptr() for t in dK]),
        p(dq), None, None, p(db),
    ]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = L.attnres_lrid_backward_noalloc(*common, stream)
        N.check(rc, "attnres_lrid_backward_noalloc")
    else:
        ws_bytes = L.attnres_lrid_backward_workspace_bytes(S, n, d, R, H, dt)
        ws = torch.empty(ws_bytes, device="cuda", dtype=torch.uint8)
        rc = L.attnres_lrid_backward(*common, p(ws), ws_bytes, stream)
        N.check(rc, "attnres_lrid_backward")
    torch.cuda.synchronize()
    return dV, dK, dq, db


def _compare(a, b, dtype):
    for x, y in zip(a[0], b[0]):
        assert_close("dV", x.float().cpu().numpy(), y.float().cpu().numpy(), dtype)
    for x, y in zip(a[1], b[1]):
        assert_close("dK", x.float().cpu().numpy(), y.float().cpu().numpy(), dtype)
    assert_close("dq", a[2].cpu().numpy(), b[2].cpu().numpy(), torch.float32, sum_terms=a[0][0].shape[0])
    assert_close("dbias", a[3].cpu().numpy(), b[3].cpu().numpy(), torch.float32, sum_terms=a[0][0].shape[0])


@pytest.mark.parametrize("dtype,H", [(torch.bfloat16, 1), (torch.float32, 2)])
def test_noalloc_backward_matches_workspace_backward_twice(dtype, H):
    """Two calls in a row: the static scratch keeps the previous call's
    partial sums, which must not leak into the next result."""
    x1 = _inputs(dtype=dtype, H=H, seed=1)
    x2 = _inputs(dtype=dtype, H=H, seed=2, n=1777)
    for x in (x1, x2):
        ref = _call(False, *x, H=H)
        got = _call(True, *x, H=H)
        _compare(got, ref, dtype)


def test_noalloc_rejects_geometries_beyond_the_static_scratch():
    L = N.load()
    cap = L.attnres_noalloc_scratch_bytes()
    assert cap == 4 << 20
    n = 1 << 20
    # wide key ranks give long partial rows (R + H + S floats per CTA)
    for S, d, R, H in [(64, 2048, 4096, 8), (64, 1024, 4096, 8), (64, 4096, 4096, 8)]:
        need = L.attnres_lrid_backward_workspace_bytes(S, n, d, R, H, N.DTYPE_BF16)
        if need > cap:
            break
    else:
        pytest.fail("no candidate geometry needs more than the static scratch")
    one = torch.zeros(16, device="cuda", dtype=torch.bfloat16)
    ptrs = N.ptr_array([one.data_ptr()] * S)
    rc = L.attnres_lrid_backward_noalloc(
        S, n, d, R, H, N.DTYPE_BF16, ptrs, N.i64_array([d] * S), ptrs, N.i64_array([R] * S),
        N.QUERY_STATIC, ctypes.c_void_p(one.data_ptr()), None, None, 1.0, 1, F32_EPS, None,
        N.NORM_NONE, 1e-2, ctypes.c_void_p(one.data_ptr()), None, None, ptrs, ptrs,
        ctypes.c_void_p(one.data_ptr()), None, None, None, None)
    assert rc == 2
    assert "static scratch" in L.attnres_last_error().decode()


def test_noalloc_accepts_calls_that_use_no_scratch():
    """A per-token (dynamic) query without a logit-bias gradient sums no
    parameter gradient, so the call uses no scratch: a geometry whose
    workspace would exceed the static array still runs, and matches the
    workspace entry point (which needs no workspace for it either)."""
    L = N.load()
    S, d, R, H = 64, 512, 4096, 8  # key heads of 512: the widest the kernels take
    cap = L.attnres_noalloc_scratch_bytes()
    for n in (256, 1024, 4096, 16384):
        if L.attnres_lrid_backward_workspace_bytes(S, n, d, R, H, N.DTYPE_BF16) > cap:
            break
    else:
        pytest.fail("no token count up to 16384 needs more than the static scratch")
    g = torch.Generator(device="cuda").manual_seed(3)
    values = [torch.randn(n, d, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(S)]
    keys = [torch.randn(n, R, device="cuda", dtype=torch.bfloat16, generator=g) for _ in range(S)]
    qdyn = torch.randn(n, R, device="cuda", dtype=torch.bfloat16, generator=g)
    grad = torch.randn(n, d, device="cuda", dtype=torch.bfloat16, generator=g)
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    results = []
    for noalloc in (False, True):
        dV = [torch.empty_like(v) for v in values]
        dK = [torch.empty_like(k) for k in keys]
        dq = torch.empty_like(qdyn)
        common = [
            S, n, d, R, H, N.DTYPE_BF16,
            N.ptr_array([v.data_ptr() for v in values]), N.i64_array([d] * S),
            N.ptr_array([k.data_ptr() for k in keys]), N.i64_array([R] * S),
            N.QUERY_DYNAMIC, None, None, p(qdyn), 0.125, 1, F32_EPS, None, N.NORM_NONE,
            RMS_EPS, p(grad), None, None,
            N.ptr_array([t.data_ptr() for t in dV]), N.ptr_array([t.data_ptr() for t in dK]),
            p(dq), None, None, None,
        ]
        if noalloc:
            N.check(L.attnres_lrid_backward_noalloc(*common, stream), "attnres_lrid_backward_noalloc")
        else:
            N.check(L.attnres_lrid_backward(*common, None, 0, stream), "attnres_lrid_backward")
        torch.cuda.synchronize()
        results.append((dV, dK, dq))
    (dV0, dK0, dq0), (dV1, dK1, dq1) = results
    for x, y in zip(dV1 + dK1 + [dq1], dV0 + dK0 + [dq0]):
        assert_close("grad", x.float().cpu().numpy(), y.float().cpu().numpy(), torch.bfloat16)
