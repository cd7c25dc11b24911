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
