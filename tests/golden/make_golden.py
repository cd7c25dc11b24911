"""Generate the golden fixtures in this directory from the reference itself.

Run (in a container where the reference checkout is available):
    ATTNRES_REFERENCE=/path/to/LR-AttnRes python tests/golden/make_golden.py [case-name-prefix ...]

It imports the reference's attnres_ops.py and runs its public read functions on
CPU fp32 tensors, which routes them through the reference's unfused PyTorch path
(attnres_ops.py:4969-4985 for LRID lists, :2193 for base lists,
:4259 / :2228 for the count-prior / logit-bias route), then back-propagates a
seeded upstream gradient with torch.autograd. Inputs are drawn from numpy's
PCG64 generator with fixed seeds (`case_inputs`, shared with the tests), so only
the reference's outputs and gradients are stored.

The fixtures pin the CPU oracle (tests/test_oracle_golden.py); the GPU parity
tests then compare the CUDA kernels against the oracle.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

from cases import CASES, case_inputs  # noqa: E402


def _ref_module():
    ref = os.environ.get("ATTNRES_REFERENCE", "/root/reference")
    sys.path.insert(0, ref)
    import attnres_ops  # the reference module

    return attnres_ops


def run_case(ref, case):
    import torch

    inp = case_inputs(case)
    kind = case["kind"]
    B, T = case["B"], case["T"]
    t = lambda x: torch.tensor(x, dtype=torch.float32, requires_grad=True)  # noqa: E731
    if kind == "phase2":
        res = {}
        D = case["D"]
        pv = torch.tensor(inp["partial_value"].reshape(B, T, D), requires_grad=True)
        io = torch.tensor(inp["interblock_output"].reshape(B, T, D), requires_grad=True)
        lse = torch.tensor(inp["interblock_lse"].reshape(B, T), requires_grad=True)
        bias = torch.tensor(inp["logit_bias"], requires_grad=True) if case.get("bias") else 0.0
        norm_out = case.get("normalize_output", False)
        if case["mode"] == "lrid":
            pk = torch.tensor(inp["partial_key"].reshape(B, T, -1), requires_grad=True)
            q = torch.tensor(inp["query"], requires_grad=True)
            out = ref.lrid_attention_residual_phase2(pv, pk, q, io, lse, case["scale"], case["key_norm"],
                                                     normalize_output=norm_out, logit_bias=bias)
        elif case["mode"] == "base":
            q = torch.tensor(inp["query"], requires_grad=True)
            out = ref.attention_residual_phase2(pv, q, io, lse, case["key_norm"], normalize_output=norm_out,
                                                logit_bias=bias)
        else:
            lg = torch.tensor(inp["partial_logit"].reshape(B, T), requires_grad=True)
            out = ref.attention_residual_phase2_from_logit(pv, lg, io, lse, normalize_output=norm_out)
        out.backward(torch.tensor(inp["grad_output"].reshape(B, T, D)))
        res["out"] = out.detach().numpy().reshape(B * T, D)
        res["d_partial_value"] = pv.grad.numpy().reshape(B * T, D)
        res["d_interblock_output"] = io.grad.numpy().reshape(B * T, D)
        res["d_interblock_lse"] = lse.grad.numpy().reshape(B * T)
        if case["mode"] == "lrid":
            res["d_partial_key"] = pk.grad.numpy().reshape(B * T, -1)
        if case["mode"] in ("lrid", "base"):
            res["dq"] = q.grad.numpy().reshape(-1)
        else:
            res["d_partial_logit"] = lg.grad.numpy().reshape(B * T)
        if case.get("bias"):
            res["dbias"] = np.array(bias.grad.item(), dtype=np.float32)
        return {k: np.asarray(v) for k, v in res.items()}
    values = [t(v.reshape(B, T, -1)) for v in inp["values"]]
    grad_out = (torch.tensor(inp["grad_output"].reshape(B, T, -1), dtype=torch.float32)
                if kind not in ("phase1", "phase2") else None)
    res = {}
    if kind == "phase1":
        Q = case["Q"]
        vs = torch.tensor(inp["values"].reshape(-1, B, T, inp["values"].shape[-1]), requires_grad=True)
        lg = torch.tensor(inp["logits"].reshape(Q, -1, B, T), requires_grad=True)
        out, lse = ref.attention_residual_phase1_from_logits(
            vs, lg, normalize_output=case.get("normalize_output", False))
        (out * torch.tensor(inp["grad_output"].reshape(Q, B, T, -1))).sum().add_(
            (lse * torch.tensor(inp["grad_lse"].reshape(Q, B, T))).sum()).backward()
        res["out"] = out.detach().numpy().reshape(Q, B * T, -1)
        res["lse"] = lse.detach().numpy().reshape(Q, B * T)
        res["dV"] = vs.grad.numpy().reshape(vs.shape[0], B * T, -1)
        res["dlogits"] = lg.grad.numpy().reshape(Q, -1, B * T)
        return res
    if kind == "lrid_kv":
        # keys from the values exactly as model.py:344-356 composes them
        import torch.nn.functional as F

        H = case["H"]
        weight = t(inp["key_weight"])
        query = t(inp["query"])
        vn = case.get("value_norm", True)
        keys = [F.linear(F.rms_norm(v, (v.size(-1),)) if vn else v, weight) for v in values]
        out = ref.lrid_attention_residual_read(values, keys, query, H, case["scale"], case["key_norm"])
        out.backward(grad_out)
        res["out"] = out.detach().numpy().reshape(B * T, -1)
        res["dV"] = np.stack([v.grad.numpy().reshape(B * T, -1) for v in values])
        res["dW"] = weight.grad.numpy()
        res["dq"] = query.grad.numpy().reshape(-1)
        return res
    if kind == "lrid":
        H = case["H"]
        keys = [t(k.reshape(B, T, -1)) for k in inp["keys"]]
        params = []
        if case["query"] == "static":
            query = t(inp["query"])
            q_used = query
            params.append(("dq", query))
        elif case["query"] == "dynamic":
            query = t(inp["query_dynamic"].reshape(B, T, H, -1))
            q_used = query
            params.append(("dq", query))
        else:  # gated hybrid, composed exactly as model.py:2104-2110
            qs = t(inp["query"])
            gate = t(inp["gate"])
            qd = t(inp["query_dynamic"].reshape(B, T, H, -1))
            q_used = qs.unsqueeze(0).unsqueeze(0) + gate.view(1, 1, H, 1) * qd
            params += [("dq", qs), ("dgate", gate), ("dq_dynamic", qd)]
        biases = None
        if case.get("bias"):
            biases = [t(np.float32(b)) for b in inp["logit_bias"]]
        out = ref.lrid_attention_residual_read(
            values, keys, q_used, H, case["scale"], case["key_norm"],
            normalize_output=case.get("normalize_output", False),
            source_logit_biases=biases,
        )
        out.backward(grad_out)
        res["out"] = out.detach().numpy().reshape(B * T, -1)
        res["dV"] = np.stack([v.grad.numpy().reshape(B * T, -1) for v in values])
        res["dK"] = np.stack([k.grad.numpy().reshape(B * T, -1) for k in keys])
        for name, p in params:
            g = p.grad.numpy()
            res[name] = g.reshape(B * T, -1) if name == "dq_dynamic" or case["query"] == "dynamic" else g.reshape(-1)
        if biases is not None:
            res["dbias"] = np.array([b.grad.item() for b in biases], dtype=np.float32)
    else:
        query = t(inp["query"])
        biases = None
        if case.get("bias"):
            biases = [t(np.float32(b)) for b in inp["logit_bias"]]
        out = ref.attention_residual_read(
            values, query, case["key_norm"],
            normalize_output=case.get("normalize_output", False),
            source_logit_biases=biases,
        )
        out.backward(grad_out)
        res["out"] = out.detach().numpy().reshape(B * T, -1)
        res["dV"] = np.stack([v.grad.numpy().reshape(B * T, -1) for v in values])
        res["dq"] = query.grad.numpy().reshape(-1)
        if biases is not None:
            res["dbias"] = np.array([b.grad.item() for b in biases], dtype=np.float32)
    keep = case.get("keep_tokens")
    if keep is not None:
        # large case: keep full out/dq, a token slice of the per-source grads,
        # and per-source sums of every grad as a checksum
        for name in ("dV", "dK"):
            if name in res:
                res[name + "_sum"] = res[name].astype(np.float64).sum(axis=(1, 2))
                res[name] = res[name][:, :keep]
    return {k: np.asarray(v) for k, v in res.items()}


def main():
    ref = _ref_module()
    import torch

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    only = sys.argv[1:]  # optional case-name prefixes: regenerate just those
    for case in CASES:
        if only and not any(case["name"].startswith(o) for o in only):
            continue
        res = run_case(ref, case)
        path = os.path.join(HERE, case["name"] + ".npz")
        np.savez_compressed(path, **res)
        print(f"wrote {path}: " + ", ".join(f"{k}{tuple(v.shape)}" for k, v in res.items()))


if __name__ == "__main__":
    main()
