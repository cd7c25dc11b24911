"""Shared helpers for the GPU parity tests: run the CUDA path through the public
API with autograd and compare against the CPU oracle."""
import numpy as np
import torch

from oracle import oracle

# Tolerances (north star): fp32 within rtol 1e-5; bf16/fp16 within rtol 2e-2 /
# atol 1e-2 against an fp32-or-better reference. Near-zero entries need an
# absolute floor relative to the tensor's scale: ATOL_REL * max|expected|.
# eps of the reference's RMS norms: F.rms_norm(eps=None) uses the eps of the
# type it computes in, fp32 for 16-bit inputs too
RMS_EPS = float(torch.finfo(torch.float32).eps)

TOL = {
    torch.float32: dict(rtol=1e-5, atol_rel=1e-5),
    torch.bfloat16: dict(rtol=2e-2, atol=1e-2),
    torch.float16: dict(rtol=2e-2, atol=1e-2),
}


def assert_close(name, actual, expected, dtype, sum_terms=1, scaled_atol=False):
    """|a - e| <= atol + rtol*|e| elementwise. For gradients summed over many
    tokens (`sum_terms` terms), fp32 rounding grows like sqrt(terms); the fp32
    absolute floor is scaled by that factor. For 16-bit dtypes the absolute
    floor is taken relative to the largest |expected| when the values are sums
    over tokens or when `scaled_atol` is set (gradients that pass through a
    16-bit saved output, whose rounding error scales with the gradient)."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert a.shape == e.shape, f"{name}: shape {a.shape} != {e.shape}"
    t = TOL[dtype]
    if dtype == torch.float32:
        atol = t["atol_rel"] * max(1.0, float(np.abs(e).max(initial=0.0))) * max(1.0, np.sqrt(sum_terms))
    else:
        atol = t["atol"] * max(1.0, float(np.abs(e).max(initial=0.0)) if (sum_terms > 1 or scaled_atol) else 1.0)
    err = np.abs(a - e)
    bound = atol + t["rtol"] * np.abs(e)
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{name}: {int(bad.sum())}/{bad.size} elements out of tolerance; worst at {i}: "
            f"actual {a[i]:.8g} expected {e[i]:.8g} (|err| {err[i]:.3e} > {bound[i]:.3e})"
        )


def to_np(t):
    return t.detach().float().cpu().numpy()


def dev_rows(x, B, T, dtype, requires_grad=True):
    t = torch.tensor(np.asarray(x, np.float32).reshape(B, T, -1), device="cuda", dtype=dtype)
    return t.requires_grad_(requires_grad)


def rounded(x, dtype):
    """The values the GPU actually sees (inputs rounded to dtype), as float32."""
    return torch.tensor(np.asarray(x, np.float32)).to(dtype).float().numpy()
