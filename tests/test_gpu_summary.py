"""GPU parity of the block-summary op (running block sum + scaled block
source, model.py:990-1028 with the running sums of model.py:2377-2389) against
the reference's own PyTorch expressions on the same inputs: forward bit-exact
(the kernel rounds like the reference's dtype ops), gradients of partial, x and
a learned scale within the repository's tolerances."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(partial, x, scale):
    """model.py:2381-2383 / :990-1001: partial_block + layer_output, then * scale."""
    s = x if partial is None else partial + x
    return s, s * scale


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 128, 256), (3, 1000, 1024), (7, 33)])
@pytest.mark.parametrize("first", [False, True])
def test_block_summary_forward_matches_reference(dtype, shape, first):
    import attnres_b200 as A

    torch.manual_seed(sum(shape))
    x = torch.randn(shape, device="cuda", dtype=dtype)
    partial = None if first else torch.randn(shape, device="cuda", dtype=dtype)
    for count, alpha in [(1, 1.0), (3, 1.0), (4, 0.5)]:
        s, src = A.attention_residual_block_summary(partial, x, count=count, alpha=alpha)
        rs, rsrc = _ref(partial, x, float(count) ** (-alpha))
        assert torch.equal(s, rs)
        assert torch.equal(src, rsrc)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_block_summary_learned_scale_gradients(dtype):
    import attnres_b200 as A

    torch.manual_seed(5)
    shape = (4, 513, 768)  # ragged element count for the 16-byte packs
    x = torch.randn(shape, device="cuda", dtype=dtype, requires_grad=True)
    p = torch.randn(shape, device="cuda", dtype=dtype, requires_grad=True)
    scale = torch.tensor(0.37, device="cuda", requires_grad=True)
    g_src = torch.randn(shape, device="cuda", dtype=dtype)
    g_sum = torch.randn(shape, device="cuda", dtype=dtype)
    s, src = A.attention_residual_block_summary(p, x, scale=scale)
    torch.autograd.backward([src, s], [g_src, g_sum])

    x2 = x.detach().clone().requires_grad_(True)
    p2 = p.detach().clone().requires_grad_(True)
    scale2 = scale.detach().clone().requires_grad_(True)
    rs, rsrc = _ref(p2, x2, scale2.to(dtype))
    torch.autograd.backward([rsrc, rs], [g_src, g_sum])

    assert torch.equal(s, rs.detach()) and torch.equal(src, rsrc.detach())
    tol = dict(rtol=1e-5, atol=1e-6) if dtype == torch.float32 else dict(rtol=2e-2, atol=1e-2)
    torch.testing.assert_close(x.grad, x2.grad, **tol)
    torch.testing.assert_close(p.grad, p2.grad, **tol)
    # the scale gradient is a sum over all elements: compare against fp32 math
    want = (g_src.float() * rs.detach().float()).sum()
    torch.testing.assert_close(scale.grad, want, rtol=1e-4 if dtype == torch.float32 else 2e-2, atol=1e-3)


def test_block_summary_scale_gradient_is_deterministic():
    import attnres_b200 as A

    torch.manual_seed(9)
    x = torch.randn(8, 2048, 1024, device="cuda", dtype=torch.bfloat16)
    p = torch.randn_like(x)
    g = torch.randn_like(x)
    grads = []
    for _ in range(2):
        scale = torch.tensor(0.25, device="cuda", requires_grad=True)
        _, src = A.attention_residual_block_summary(p, x, scale=scale)
        src.backward(g)
        grads.append(scale.grad.clone())
    assert torch.equal(grads[0], grads[1])


def test_block_summary_tensor_alpha_gradient():
    """A learned alpha (tensor) keeps its gradient through count ** -alpha."""
    import attnres_b200 as A

    torch.manual_seed(2)
    x = torch.randn(2, 64, 256, device="cuda", dtype=torch.float32)
    p = torch.randn_like(x)
    alpha = torch.tensor(0.5, device="cuda", requires_grad=True)
    _, src = A.attention_residual_block_summary(p, x, count=4, alpha=alpha)
    src.sum().backward()
    alpha2 = alpha.detach().clone().requires_grad_(True)
    c = torch.exp(-alpha2 * torch.tensor(4.0, device="cuda").log())
    ((p + x) * c).sum().backward()
    torch.testing.assert_close(alpha.grad, alpha2.grad, rtol=1e-5, atol=1e-5)


def test_block_summary_cpu_tensors_fail_loudly():
    import attnres_b200 as A

    with pytest.raises(RuntimeError, match="CUDA"):
        A.attention_residual_block_summary(None, torch.randn(4, 8), count=2)


def _golden():
    import json
    import os

    import numpy as np

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "block_summary.npz")
    d = np.load(path)
    return d, json.loads(bytes(d["meta"]).decode())


_D, _META = _golden()


@pytest.mark.parametrize("case", sorted(_META))
def test_lrid_block_source_matches_the_reference_model(case):
    """attnres_b200.lrid_block_source against the reference model's own
    _lrid_block_source on the running sums (fixtures written by
    tests/golden/make_block_summary.py): count / sqrt / learned alpha / learned
    scale, the value norm, and key scaling when key norm is off."""
    import attnres_b200 as A
    from gpu_helpers import assert_close

    m = _META[case]
    dtype = getattr(torch, m["dtype"])
    get = lambda k: torch.tensor(_D[f"{case}/{k}"], device="cuda")  # noqa: E731
    t = {k: get(k).to(dtype).requires_grad_(not k.startswith("g")) for k in
         ("pv", "x", "pk", "k", "g_vsum", "g_vsrc", "g_ksum", "g_ksrc")}
    alpha = m["alpha"] if m["alpha"] is not None else 1.0
    scale = None
    if m["alpha_learned"]:
        alpha = torch.tensor(m["alpha"], device="cuda", requires_grad=True)
    if m["scale"] is not None:
        scale = torch.tensor(m["scale"], device="cuda", requires_grad=True)
    vsum, vsrc, ksum, ksrc = A.lrid_block_source(t["pv"], t["x"], t["pk"], t["k"], count=m["count"], alpha=alpha,
                                                 scale=scale, value_norm=m["value_norm"], key_norm=m["key_norm"])
    for name, got in (("vsum", vsum), ("vsrc", vsrc), ("ksum", ksum), ("ksrc", ksrc)):
        assert_close(name, got.detach().float().cpu().numpy(), _D[f"{case}/{name}"], dtype)
    loss = ((vsum * t["g_vsum"]).sum() + (vsrc * t["g_vsrc"]).sum() + (ksum * t["g_ksum"]).sum()
            + (ksrc * t["g_ksrc"]).sum())
    loss.float().backward()
    for name in ("pv", "x", "pk", "k"):
        assert_close(f"d_{name}", t[name].grad.float().cpu().numpy(), _D[f"{case}/d_{name}"], dtype)
    n = t["x"].numel()
    if m["alpha_learned"]:
        assert_close("d_alpha", alpha.grad.reshape(1).cpu().numpy(), _D[f"{case}/d_alpha"], torch.float32,
                     sum_terms=n)
    if scale is not None:
        assert_close("d_scale", scale.grad.reshape(1).cpu().numpy(), _D[f"{case}/d_scale"], torch.float32,
                     sum_terms=n)
