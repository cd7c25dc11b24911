"""GPU parity of LRIDFusedProjection.forward (model.py:363-388, fused-key
layout) against the reference's own composition -- one linear projection, the
output columns split off, the key columns normalised per head by
_norm_lrid_key (model.py:33-36), the query columns split off -- evaluated in
float64 from the same (rounded) inputs: forward and the gradients of x and of
the projection weight. fp32 is held to 1e-5 (the weight gradient, a sum over
all tokens, to 1e-5 of its scale); 16-bit to the output rounding."""
import pytest
import torch

from gpu_helpers import RMS_EPS
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _ref(x, w, d, R, H, key_norm, Rq):
    projected = F.linear(x, w)
    out = projected[..., :d].contiguous()
    key = projected[..., d:d + R]
    if key_norm:
        ks = key.shape
        # F.rms_norm's default eps for fp32 / 16-bit inputs, which the model uses
        key = F.rms_norm(key.reshape(*ks[:-1], H, ks[-1] // H), (ks[-1] // H,), eps=RMS_EPS).reshape(ks)
    query = projected[..., d + R:d + R + Rq] if Rq else None
    return out, key, query


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d,R,H,key_norm,Rq", [(256, 64, 1, True, 0), (512, 64, 4, True, 64), (192, 32, 2, False, 32)])
def test_fused_projection_matches_reference(dtype, d, R, H, key_norm, Rq):
    import attnres_b200 as A

    torch.manual_seed(d + R + Rq)
    B, T, din = 2, 97, 384
    x = torch.randn(B, T, din, device="cuda", dtype=dtype, requires_grad=True)
    w = (torch.randn(d + R + Rq, din, device="cuda") / din ** 0.5).to(dtype).requires_grad_(True)
    res = A.lrid_fused_projection_forward(x, w, d, R, H, key_norm, Rq)
    x64 = x.detach().double().requires_grad_(True)
    w64 = w.detach().double().requires_grad_(True)
    ref = _ref(x64, w64, d, R, H, key_norm, Rq)
    if dtype == torch.float32:
        tol, wtol = dict(rtol=1e-5, atol=1e-5), dict(rtol=1e-5, atol=1e-5 * (B * T) ** 0.5)
    else:
        tol, wtol = dict(rtol=2e-2, atol=2e-2), dict(rtol=2e-2, atol=2e-2 * (B * T) ** 0.5)
    for a, b in zip(res, ref):
        torch.testing.assert_close(a.double(), b, **tol)
    grads = [torch.randn_like(t, dtype=dtype) for t in ref if t is not None]
    torch.autograd.backward([t for t in res], grads)
    torch.autograd.backward([t for t in ref if t is not None], [g.double() for g in grads])
    torch.testing.assert_close(x.grad.double(), x64.grad, **tol)
    # the weight gradient sums over all B*T tokens: its rounding grows like sqrt(B*T)
    torch.testing.assert_close(w.grad.double(), w64.grad, **wtol)


def test_head_rms_norm_reads_a_strided_key_slice():
    """The key norm reads the key columns in place (row stride of the
    projection's key/query buffer) and matches F.rms_norm per head."""
    from attnres_b200 import _native as N
    import ctypes

    torch.manual_seed(0)
    n, R, H = 1000, 64, 4
    kq = torch.randn(n, 2 * R, device="cuda", dtype=torch.bfloat16)
    y = torch.empty(n, R, device="cuda", dtype=torch.bfloat16)
    inv = torch.empty(n, H, device="cuda")
    rc = N.load().attnres_head_rms_norm_forward(n, R, H, 2, ctypes.c_void_p(kq.data_ptr()), kq.stride(0),
                                                RMS_EPS, ctypes.c_void_p(y.data_ptr()),
                                                ctypes.c_void_p(inv.data_ptr()), None)
    N.check(rc, "head norm")
    torch.cuda.synchronize()
    # against fp32 math (bf16 tolerance), as the other bf16 parity checks
    xk = kq[:, :R].float().reshape(n, H, R // H)
    want = (xk * torch.rsqrt(xk.pow(2).mean(-1, keepdim=True) + RMS_EPS)).reshape(n, R)
    torch.testing.assert_close(y.float(), want, rtol=2e-2, atol=1e-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,din,R,H,Rq,key_norm", [(300, 384, 64, 2, 32, True), (1000, 1024, 64, 1, 0, True),
                                                   (129, 256, 32, 2, 0, True), (257, 512, 64, 4, 64, False)])
def test_fused_key_projection_tensor_core_epilogue(dtype, n, din, R, H, Rq, key_norm):
    """attnres_lrid_fused_key_projection (tcgen05 GEMM, per-head key norm in
    the epilogue) through the C ABI: the pre-norm key/query columns against a
    float64 GEMM of the same rounded inputs, the normalised key and its inverse
    rms against F.rms_norm per head of the kernel's own rounded columns, and a
    strided input row (x a column slice of a wider tensor)."""
    from attnres_b200 import _native as N
    import ctypes

    torch.manual_seed(n + din + R)
    code = {torch.bfloat16: 2, torch.float16: 1}[dtype]
    wide = torch.randn(n, din + 64, device="cuda", dtype=dtype)
    x = wide[:, 32:32 + din]  # row stride din + 64, 64-byte offset
    d_out = 128
    w = (torch.randn(d_out + R + Rq, din, device="cuda") / din ** 0.5).to(dtype)
    wk = w[d_out:]
    kq = torch.empty(n, R + Rq, device="cuda", dtype=dtype)
    key = torch.empty(n, R, device="cuda", dtype=dtype)
    inv = torch.empty(n, H, device="cuda")
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = N.load().attnres_lrid_fused_key_projection(n, din, R, Rq, H, code, vp(x), x.stride(0), vp(wk), wk.stride(0),
                                                     int(key_norm), RMS_EPS, vp(kq), vp(key), vp(inv), None)
    N.check(rc, "attnres_lrid_fused_key_projection")
    torch.cuda.synchronize()
    ref = x.double() @ wk.double().t()
    torch.testing.assert_close(kq.double(), ref, rtol=1e-2, atol=1e-2)
    if key_norm:
        kr = kq[:, :R].double().reshape(n, H, R // H)
        want_inv = torch.rsqrt(kr.pow(2).mean(-1) + RMS_EPS)
        torch.testing.assert_close(inv.double(), want_inv, rtol=1e-5, atol=1e-6)
        want = (kr * want_inv.unsqueeze(-1)).reshape(n, R)
        torch.testing.assert_close(key.double(), want, rtol=1e-2, atol=1e-2)


def test_fused_key_projection_rejects_fp32_and_odd_shapes():
    """fp32 (no tensor-core path at fp32 accuracy) and shapes outside the
    kernel return ATTNRES_ERR_UNSUPPORTED with nothing launched; the op then
    takes the library GEMM and the per-head norm kernel."""
    from attnres_b200 import _native as N
    import ctypes

    x = torch.randn(64, 384, device="cuda")
    w = torch.randn(64, 384, device="cuda")
    out = torch.empty(64, 64, device="cuda")
    inv = torch.empty(64, 1, device="cuda")
    vp = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    L = N.load()
    assert L.attnres_lrid_fused_key_projection(64, 384, 64, 0, 1, 0, vp(x), 384, vp(w), 384, 1, RMS_EPS, vp(out),
                                               vp(out), vp(inv), None) == 2
    xb, wb = x.bfloat16(), w.bfloat16()
    ob = torch.empty(64, 64, device="cuda", dtype=torch.bfloat16)
    # in_dim 352 is not a multiple of 64; head width 64 / 8 = 8 is not a multiple of 16
    assert L.attnres_lrid_fused_key_projection(64, 352, 64, 0, 1, 2, vp(xb), 384, vp(wb), 384, 1, RMS_EPS, vp(ob),
                                               vp(ob), vp(inv), None) == 2
    assert L.attnres_lrid_fused_key_projection(64, 384, 64, 0, 8, 2, vp(xb), 384, vp(wb), 384, 1, RMS_EPS, vp(ob),
                                               vp(ob), vp(inv), None) == 2
