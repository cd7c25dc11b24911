"""Golden block summaries from the reference model's own functions.

Run (in a container where the reference checkout is available):
    ATTNRES_REFERENCE=/path/to/LR-AttnRes python tests/golden/make_block_summary.py

For each case the reference's OBPM (model.py) is built with the case's
block-average settings, and one LRID block step is computed the way the model
does it: the running sums value_sum = partial_value + x and key_sum =
partial_key + key (model.py:2377-2389), then the block source from the
model's `_lrid_block_source` (model.py:1003-1028) -- count^-alpha scaling
(count / sqrt modes, learned alpha), learned block scales, the value norm, and
key scaling when key norm is off. A seeded upstream gradient on the two sums
and the two sources is back-propagated with autograd. Inputs come from numpy
PCG64 seeds; the inputs, the alpha / scale the model used, the outputs and the
gradients are stored in block_summary.npz (one key prefix per case).
tests/test_gpu_summary.py compares attnres_b200.lrid_block_source with them.
"""
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

BASE = dict(n_layer=2, n_head=2, n_embd=256, mlp_hidden_dim=512, vocab_size=64, block_size=8,
            use_attnres=True, attnres_type="block", attnres_num_blocks=2, use_lrid=True, lrid_rank=64,
            lrid_num_heads=1)

# name -> (config overrides, count, summary_idx, dtype)
CASES = {
    "count_keynorm": (dict(attnres_block_average_mode="count"), 3, 2, torch.float32),
    "count_nokeynorm": (dict(attnres_block_average_mode="count", attnres_key_norm=False), 3, 2, torch.float32),
    "sqrt_nokeynorm_bf16": (dict(attnres_block_average_mode="sqrt", attnres_key_norm=False), 4, 3, torch.bfloat16),
    "learned_alpha_nokeynorm": (dict(attnres_block_alpha_learned=True, attnres_key_norm=False), 2, 1, torch.float32),
    # (the count prior needs alpha-formula summaries, model.py:160-168)
    "learned_scale_nokeynorm": (dict(attnres_block_learned_scale=True, attnres_key_norm=False,
                                     attnres_block_count_prior=False), 2, 2, torch.float32),
    "value_norm": (dict(attnres_block_value_norm=True, attnres_block_count_prior=False), 3, 2, torch.float32),
    "value_norm_nokeynorm": (dict(attnres_block_value_norm=True, attnres_key_norm=False,
                                  attnres_block_count_prior=False), 3, 2, torch.float32),
    "value_norm_bf16": (dict(attnres_block_value_norm=True, attnres_block_count_prior=False), 2, 1,
                        torch.bfloat16),
}


def _model_module():
    ref = os.environ.get("ATTNRES_REFERENCE", "/root/reference")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import model

    return model


def run_case(M, name, ov, count, idx, dtype, seed):
    torch.manual_seed(seed)
    m = M.OBPM(M.ModelConfig(**BASE, **ov)).to(dtype)
    rng = np.random.default_rng(seed)
    n, d, r = 2 * 8, BASE["n_embd"], BASE["lrid_rank"]
    f = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    arrays = {"pv": f(n, d), "x": f(n, d) * 0.5, "pk": f(n, r), "k": f(n, r) * 0.5,
              "g_vsum": f(n, d), "g_vsrc": f(n, d), "g_ksum": f(n, r), "g_ksrc": f(n, r)}
    t = {k: torch.tensor(v).to(dtype).requires_grad_(k[0] != "g") for k, v in arrays.items()}
    vsum = t["pv"] + t["x"]
    ksum = t["pk"] + t["k"]
    vsrc, ksrc = m._lrid_block_source(vsum, ksum, None, count, idx)[:2]
    alpha = None if ov.get("attnres_block_learned_scale") else m._attnres_block_alpha(summary_idx=idx)
    scale = m.transformer.attnres_block_scales[idx - 1] if ov.get("attnres_block_learned_scale") else None
    learned = [p for p in (alpha, scale) if torch.is_tensor(p)]
    # the scaled key path returns a new tensor; the unscaled one returns ksum itself
    loss = ((vsum * t["g_vsum"]).sum() + (vsrc * t["g_vsrc"]).sum() + (ksum * t["g_ksum"]).sum()
            + (ksrc * t["g_ksrc"]).sum())
    loss.float().backward()
    out = {k: v for k, v in arrays.items()}
    out.update(vsum=vsum.detach().float().numpy(), vsrc=vsrc.detach().float().numpy(),
               ksum=ksum.detach().float().numpy(), ksrc=ksrc.detach().float().numpy(),
               d_pv=t["pv"].grad.float().numpy(), d_x=t["x"].grad.float().numpy(),
               d_pk=t["pk"].grad.float().numpy(), d_k=t["k"].grad.float().numpy())
    meta = {"count": count, "dtype": str(dtype).replace("torch.", ""),
            "value_norm": bool(ov.get("attnres_block_value_norm", False)),
            "key_norm": bool(ov.get("attnres_key_norm", True)),
            "alpha": None if alpha is None else float(torch.as_tensor(alpha).detach()), "alpha_learned": torch.is_tensor(alpha),
            "scale": None if scale is None else float(scale.detach())}
    # learned alpha / scale are one entry of a parameter vector: its gradient
    for pname, key in (("attnres_block_alphas", "d_alpha"), ("attnres_block_scales", "d_scale")):
        par = getattr(m.transformer, pname, None) if learned else None
        if par is not None and par.grad is not None:
            out[key] = np.array([par.grad.float().sum().item()], np.float32)
    return out, meta


def main():
    M = _model_module()
    arrays, metas = {}, {}
    for i, (name, (ov, count, idx, dtype)) in enumerate(CASES.items()):
        out, meta = run_case(M, name, ov, count, idx, dtype, seed=500 + i)
        metas[name] = meta
        for k, v in out.items():
            arrays[f"{name}/{k}"] = v
        print(name, meta)
    arrays["meta"] = np.frombuffer(json.dumps(metas).encode(), dtype=np.uint8)
    np.savez_compressed(os.path.join(HERE, "block_summary.npz"), **arrays)


if __name__ == "__main__":
    main()
