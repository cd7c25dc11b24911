"""The reference model's own calls, replayed through the drop-in on the GPU.

tests/golden/make_model_calls.py ran the reference's OBPM (model.py) on the
CPU with use_fused_attnres=True and recorded every call it made into the op API:
the arguments, the reference's result, and in training the upstream gradient
the model sent into the call and the gradients the call returned to its inputs.
Here each call goes through the drop-in `attnres_ops` (the B200 kernels) with
the same arguments; its outputs, and the input gradients for the same upstream
gradient, must match the reference within the stated tolerances:
  * fp32 calls: rtol 1e-5, with an absolute floor of 1e-5 of the tensor's
    largest magnitude (times sqrt(tokens) for gradients summed over tokens);
  * bf16 calls: rtol 2e-2 / atol 1e-2 against the reference's fp32 result on
    the same (bf16) inputs.
Because model.py is unchanged between the two runs, a match on every call is
a match of the whole model. Two configurations replay model.py with its call
sites patched to the entry points this package adds (in-kernel gated query,
in-op key projection); the generator checked on the CPU that the patch leaves
the model's output and gradients unchanged.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import assert_close
from model_calls import FILES, IDS, array, call_args, load

pytestmark = pytest.mark.gpu


def _tokens(leaves):
    n = 1
    for t in leaves:
        if t.dim() >= 3:
            n = max(n, t.shape[0] * t.shape[1])
    return n


@pytest.mark.parametrize("path", FILES, ids=IDS)
def test_reference_model_calls_through_the_drop_in(path):
    import attnres_ops

    d, meta = load(path)
    for i, call in enumerate(meta["calls"]):
        name = f"{meta['config']}[{i}] {call['fn']}"
        fn = getattr(attnres_ops, call["fn"])
        leaves, args, kwargs = call_args(d, call, device="cuda")
        low = "outs_f32" in call
        tol = torch.bfloat16 if low else torch.float32
        res = fn(*args, **kwargs)
        outs = res if call["tuple"] else (res,)
        refs = call["outs_f32"] if low else call["outs"]
        assert len(outs) == len(refs), name
        for j, (o, key) in enumerate(zip(outs, refs)):
            assert_close(f"{name} out{j}", o.detach().float().cpu().numpy(), array(d, key).float().numpy(), tol)
        if "grad_outs" not in call:
            continue
        pairs = [(o, array(d, key, o.dtype, "cuda")) for o, key in zip(outs, call["grad_outs"])
                 if key is not None and o.requires_grad]
        torch.autograd.backward([o for o, _ in pairs], [g for _, g in pairs])
        torch.cuda.synchronize()
        ntok = _tokens(leaves)
        grads = call["grad_in_f32"] if low else call["grad_in"]
        for idx, key in grads.items():
            leaf = leaves[int(idx)]
            assert leaf.grad is not None, f"{name}: no gradient for input {idx}"
            # parameters (query, gate, biases, key weight) sum over every token
            per_token = leaf.dim() >= 2 and leaf.shape[0] * leaf.shape[1] == ntok
            summed = leaf.dim() < 3 and not per_token
            assert_close(f"{name} grad{idx}", leaf.grad.float().cpu().numpy(), array(d, key).float().numpy(), tol,
                         sum_terms=ntok if summed else 1)
    torch.cuda.synchronize()
    from attnres_b200 import _native

    assert _native.device_status(reset=True) == 0
