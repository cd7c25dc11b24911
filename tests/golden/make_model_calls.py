"""Record the calls the reference model makes into the AttnRes op API.

Run (in a container where the reference checkout is available):
    ATTNRES_REFERENCE=/path/to/LR-AttnRes python tests/golden/make_model_calls.py

For each model configuration below, the reference's own `OBPM` (model.py) runs
on the CPU with `use_fused_attnres=True`. Every name that model.py imports from
attnres_ops (model.py:9-19) is wrapped, so each call the model makes is
recorded with:
  * its exact arguments (tensors, lists, scalars, keyword arguments),
  * the reference's result (its PyTorch path, which the CPU takes),
  * in training configurations, the upstream gradient that the model's
    backward sends into that call and the gradients the call returns to each
    of its tensor inputs, isolated per call.
Calls made with 16-bit tensors are also re-run in fp32 on the same
(upcast) inputs, which gives the fp32 reference that the bf16 tolerance is
stated against.

Two configurations are also recorded with model.py's call sites patched to the
entry points this package adds: the gated hybrid query formed inside the
kernel (`lrid_attention_residual_read_gated`) and, in shared key-from-value
mode, keys projected inside the op (`lrid_attention_residual_read_key_from_value`).
For those, the new entry points are composed here from the reference's own
functions, and the script first checks that the patched model's output and
parameter gradients equal the unpatched model's. PATCHES below is the patch;
INTEGRATION.md shows it as a diff.

Writes tests/golden/model_calls/<config>.npz: a JSON description of the calls
plus the arrays. tests/test_gpu_model_calls.py replays every call through the
drop-in `attnres_ops` on the GPU; tests/test_model_calls.py checks on the CPU
that each recorded call binds to the drop-in's signatures.
"""
import importlib.util
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "model_calls")

API = [
    "attention_residual_average_read",
    "attention_residual_phase1_from_logits",
    "attention_residual_phase2",
    "attention_residual_phase2_torch",
    "attention_residual_phase2_from_logit",
    "attention_residual_read",
    "lrid_attention_residual_phase2",
    "lrid_attention_residual_phase2_torch",
    "lrid_attention_residual_read",
]
NEW_API = ["lrid_attention_residual_read_gated", "lrid_attention_residual_read_key_from_value"]

# model.py call-site patch: (anchor text that must occur once, replacement)
PATCHES = [
    (
        "    lrid_attention_residual_read,\n)\n",
        "    lrid_attention_residual_read,\n"
        "    lrid_attention_residual_read_gated,\n"
        "    lrid_attention_residual_read_key_from_value,\n)\n",
    ),
    (
        "        if self.config.use_fused_attnres:\n"
        "            return lrid_attention_residual_read(\n",
        "        if (\n"
        "            self.config.use_fused_attnres\n"
        "            and self.config.lrid_input_dependent_query\n"
        "            and not self.config.attn_res_query_norm\n"
        "        ):\n"
        "            # static + gate * dynamic query formed inside the read kernel\n"
        "            return lrid_attention_residual_read_gated(\n"
        "                value_sources,\n"
        "                key_sources,\n"
        "                static_query,\n"
        "                self.transformer.lrid_query_gates[query_idx],\n"
        "                dynamic_query,\n"
        "                num_heads,\n"
        "                self.config.lrid_logit_scale,\n"
        "                self.config.attnres_key_norm,\n"
        "                normalize_output=normalize_output,\n"
        "                source_counts=source_counts,\n"
        "                source_logit_biases=source_logit_biases,\n"
        "            )\n"
        "        if (\n"
        "            self.config.use_fused_attnres\n"
        "            and self.config.lrid_key_from_value_shared\n"
        "            and not self.config.lrid_add_static_source_key\n"
        "            and not self.config.lrid_add_static_embedding_key\n"
        "            and not self.config.lrid_static_embedding_key\n"
        "        ):\n"
        "            # every source key is proj(norm(value)) with the shared projection:\n"
        "            # project inside the read instead of reading precomputed keys\n"
        "            return lrid_attention_residual_read_key_from_value(\n"
        "                value_sources,\n"
        "                self.transformer.lrid_embedding_key.proj.weight,\n"
        "                query,\n"
        "                num_heads,\n"
        "                self.config.lrid_logit_scale,\n"
        "                self.config.attnres_key_norm,\n"
        "                normalize_output=normalize_output,\n"
        "                value_norm=self.config.lrid_key_value_norm,\n"
        "                source_counts=source_counts,\n"
        "                source_logit_biases=source_logit_biases,\n"
        "            )\n"
        "        if self.config.use_fused_attnres:\n"
        "            return lrid_attention_residual_read(\n",
    ),
]

SMALL = dict(n_layer=3, n_head=4, n_embd=64, mlp_hidden_dim=128, vocab_size=128, block_size=12,
             flash_attention=False, norm_pos="before", use_attnres=True, attnres_num_blocks=2,
             attnres_block_average=True, attnres_key_norm=True, lrid_use_logit_scale=True)
# Training configurations: few tokens (one sequence of 8) but rows wide enough
# for the streaming kernels (d / H a multiple of 128 fp32 / 256 bf16 columns)
MID = dict(SMALL, n_layer=4, n_embd=256, mlp_hidden_dim=512, vocab_size=256, block_size=8,
           attn_res_query_init="normal", batch=1)
WIDE = dict(MID, n_embd=512, mlp_hidden_dim=1024)

# name -> (config overrides, train?, dtype, patched?)
CONFIGS = {
    # reference tests/test_attnres_ops.py:1150-1184 (eval, fp32)
    "eval_lrid_block_h2": (dict(SMALL, attnres_type="block", use_lrid=True, lrid_rank=32, lrid_num_heads=2),
                           False, torch.float32, False),
    "eval_lrid_full_tail": (dict(SMALL, attnres_type="full", use_lrid=True, lrid_rank=32, lrid_num_heads=2,
                                 lrid_key_from_output_tail=True), False, torch.float32, False),
    "eval_base_block": (dict(SMALL, attnres_type="block", use_lrid=False), False, torch.float32, False),
    # reference tests/test_attnres_ops.py:1187-1239 (cached block training, bf16)
    "train_cached_lrid_h1_bf16": (dict(MID, attnres_type="block", use_lrid=True, lrid_rank=32, lrid_num_heads=1),
                                  True, torch.bfloat16, False),
    "train_cached_base_bf16": (dict(MID, attnres_type="block", use_lrid=False), True, torch.bfloat16, False),
    # the same with phase 2 routed to the fused merge instead of its PyTorch form
    "train_cached_lrid_h1_fused_phase2_bf16": (dict(MID, attnres_type="block", use_lrid=True, lrid_rank=32,
                                                    lrid_num_heads=1, attnres_training_torch_phase2=False),
                                               True, torch.bfloat16, False),
    "train_cached_base_fused_phase2_bf16": (dict(MID, attnres_type="block", use_lrid=False,
                                                 attnres_training_torch_phase2=False), True, torch.bfloat16, False),
    # full AttnRes over every sublayer output: the base read
    "train_base_full": (dict(MID, attnres_type="full", use_lrid=False), True, torch.float32, False),
    # uncached block training: the fused read with its output norm and the count prior
    "train_lrid_h1_readnorm": (dict(MID, attnres_type="block", use_lrid=True, lrid_rank=32, lrid_num_heads=1,
                                    attnres_training_cache_phase1=False), True, torch.float32, False),
    "train_lrid_h2_count_prior": (dict(MID, attnres_type="block", use_lrid=True, lrid_rank=64, lrid_num_heads=2),
                                  True, torch.float32, False),
    "train_lrid_h2_bf16": (dict(WIDE, attnres_type="block", use_lrid=True, lrid_rank=64, lrid_num_heads=2),
                           True, torch.bfloat16, False),
    "train_gated_h2": (dict(MID, attnres_type="block", use_lrid=True, lrid_rank=32, lrid_num_heads=2,
                            lrid_input_dependent_query=True, attn_res_query_init="normal"), True, torch.float32,
                       False),
    "train_kv_shared_h2": (dict(MID, attnres_type="block", use_lrid=True, lrid_rank=32, lrid_num_heads=2,
                                lrid_key_from_value_shared=True, attn_res_query_init="normal"), True, torch.float32,
                           False),
    # model.py patched to the in-kernel gated query / in-op key projection
    "patched_gated_h2": (dict(MID, attnres_type="block", use_lrid=True, lrid_rank=32, lrid_num_heads=2,
                              lrid_input_dependent_query=True, attn_res_query_init="normal"), True, torch.float32,
                         True),
    "patched_kv_shared_h2": (dict(MID, attnres_type="block", use_lrid=True, lrid_rank=32, lrid_num_heads=2,
                                  lrid_key_from_value_shared=True, attn_res_query_init="normal"), True,
                             torch.float32, True),
}


def _reference_dir():
    return os.environ.get("ATTNRES_REFERENCE", "/root/reference")


def _ref_modules(patched):
    ref = _reference_dir()
    if ref not in sys.path:
        sys.path.insert(0, ref)
    import attnres_ops  # the reference module

    if not patched:
        import model

        return attnres_ops, model
    _install_new_entry_points(attnres_ops)
    src = open(os.path.join(ref, "model.py")).read()
    for anchor, repl in PATCHES:
        assert src.count(anchor) == 1, f"patch anchor not found once: {anchor[:60]!r}"
        src = src.replace(anchor, repl)
    spec = importlib.util.spec_from_loader("model_patched", loader=None)
    mod = importlib.util.module_from_spec(spec)
    exec(compile(src, "model.py (patched)", "exec"), mod.__dict__)
    return attnres_ops, mod


def _install_new_entry_points(ref_ops):
    """The two added entry points, composed from the reference's own read
    (their semantics by definition), for the patched model on the CPU."""

    def lrid_attention_residual_read_gated(values, keys, static_query, query_gate, dynamic_query, num_heads,
                                           logit_scale, key_norm, normalize_output=False, source_counts=None,
                                           source_logit_biases=None):
        H = int(num_heads)
        q = static_query.unsqueeze(0).unsqueeze(0) + query_gate.view(1, 1, H, 1) * dynamic_query
        return ref_ops.lrid_attention_residual_read(values, keys, q, H, logit_scale, key_norm,
                                                    normalize_output=normalize_output, source_counts=source_counts,
                                                    source_logit_biases=source_logit_biases)

    def lrid_attention_residual_read_key_from_value(values, key_weight, query, num_heads, logit_scale, key_norm,
                                                    normalize_output=False, value_norm=True, source_counts=None,
                                                    source_logit_biases=None, query_gate=None, dynamic_query=None):
        keys = [F.linear(F.rms_norm(v, (v.size(-1),)) if value_norm else v, key_weight) for v in values]
        return ref_ops.lrid_attention_residual_read(values, keys, query, num_heads, logit_scale, key_norm,
                                                    normalize_output=normalize_output, source_counts=source_counts,
                                                    source_logit_biases=source_logit_biases)

    ref_ops.lrid_attention_residual_read_gated = lrid_attention_residual_read_gated
    ref_ops.lrid_attention_residual_read_key_from_value = lrid_attention_residual_read_key_from_value


# ---------------------------------------------------------------------------
# recording
# ---------------------------------------------------------------------------
class Recorder:
    """Arrays are stored once per distinct content (the same source tensors
    reach many calls); bf16 tensors as their 16-bit patterns (key prefix b),
    everything else as fp32 (prefix f)."""

    def __init__(self):
        self.calls = []
        self.arrays = {}
        self.index = {}

    def save_tensor(self, t):
        t = t.detach().cpu().contiguous()
        if t.dtype == torch.bfloat16:
            arr, prefix = t.view(torch.int16).numpy(), "b"
        else:
            arr, prefix = t.float().numpy(), "f"
        sig = (prefix, arr.shape, arr.tobytes())
        key = self.index.get(sig)
        if key is None:
            key = f"{prefix}{len(self.arrays)}"
            self.arrays[key] = arr
            self.index[sig] = key
        return key


def _flatten(x, leaves):
    """Argument structure as JSON, tensors replaced by leaf indices."""
    if torch.is_tensor(x):
        leaves.append(x)
        return {"t": len(leaves) - 1}
    if isinstance(x, (list, tuple)):
        return {"l": [_flatten(e, leaves) for e in x]}
    if x is None or isinstance(x, (bool, int, float, str)):
        return {"v": x}
    raise TypeError(f"unsupported argument type {type(x)}")


def _rebuild(spec, leaves):
    if "t" in spec:
        return leaves[spec["t"]]
    if "l" in spec:
        return [_rebuild(e, leaves) for e in spec["l"]]
    return spec["v"]


class _Bridge(torch.autograd.Function):
    """Connects the call's isolated leaf graph to the model's graph; in the
    backward it records the upstream gradient and the call's input gradients."""

    @staticmethod
    def forward(ctx, state, *orig):
        ctx.state = state
        return tuple(o.detach().clone() for o in state["outs"])

    @staticmethod
    def backward(ctx, *gouts):
        st = ctx.state
        outs, leaves = st["outs"], st["grad_leaves"]
        pairs = [(o, g) for o, g in zip(outs, gouts) if g is not None and o.requires_grad]
        grads = [None] * len(leaves)
        if pairs and leaves:
            grads = torch.autograd.grad([o for o, _ in pairs], leaves, [g for _, g in pairs], allow_unused=True)
        st["on_backward"](gouts, grads)
        return (None, *grads)


def _wrap(name, fn, rec, train):
    def wrapper(*args, **kwargs):
        leaves = []
        spec = _flatten(list(args), leaves)
        kw_spec = {k: _flatten(v, leaves) for k, v in kwargs.items()}
        clones = [t.detach().clone().requires_grad_(t.requires_grad and t.is_floating_point()) for t in leaves]
        cargs = _rebuild(spec, clones)
        ckw = {k: _rebuild(s, clones) for k, s in kw_spec.items()}
        with torch.enable_grad():
            res = fn(*cargs, **ckw)
        outs = res if isinstance(res, tuple) else (res,)
        call = {
            "fn": name, "args": spec, "kwargs": kw_spec,
            "leaves": [{"a": rec.save_tensor(t), "dtype": str(t.dtype).replace("torch.", ""),
                        "requires_grad": bool(c.requires_grad)} for t, c in zip(leaves, clones)],
            "outs": [rec.save_tensor(o) for o in outs],
            "tuple": isinstance(res, tuple),
        }
        low = any(t.dtype in (torch.bfloat16, torch.float16) for t in leaves)
        if low:
            # the same call in fp32 on the upcast inputs: the fp32 reference
            c32 = [t.detach().float().requires_grad_(c.requires_grad) for t, c in zip(leaves, clones)]
            with torch.enable_grad():
                r32 = fn(*_rebuild(spec, c32), **{k: _rebuild(s, c32) for k, s in kw_spec.items()})
            o32 = r32 if isinstance(r32, tuple) else (r32,)
            call["outs_f32"] = [rec.save_tensor(o) for o in o32]
        rec.calls.append(call)
        grad_idx = [i for i, c in enumerate(clones) if c.requires_grad]
        if not train or not grad_idx or not any(o.requires_grad for o in outs):
            return res

        def on_backward(gouts, grads):
            call["grad_outs"] = [rec.save_tensor(g) if g is not None else None for g in gouts]
            call["grad_in"] = {str(i): rec.save_tensor(g) for i, g in zip(grad_idx, grads) if g is not None}
            if low:
                gl = [g.float() if g is not None else None for g in gouts]
                pairs = [(o, g) for o, g in zip(o32, gl) if g is not None and o.requires_grad]
                g32 = torch.autograd.grad([o for o, _ in pairs], [c32[i] for i in grad_idx], [g for _, g in pairs],
                                          allow_unused=True)
                call["grad_in_f32"] = {str(i): rec.save_tensor(g) for i, g in zip(grad_idx, g32) if g is not None}

        state = {"outs": outs, "grad_leaves": [clones[i] for i in grad_idx], "on_backward": on_backward}
        bridged = _Bridge.apply(state, *[leaves[i] for i in grad_idx])
        return bridged if isinstance(res, tuple) else bridged[0]

    return wrapper


def _build(mod, overrides, fused, dtype, train, seed):
    torch.manual_seed(seed)
    overrides = {k: v for k, v in overrides.items() if k != "batch"}
    cfg = mod.ModelConfig(**overrides, use_fused_attnres=fused)
    m = mod.OBPM(cfg)
    if cfg.use_lrid and cfg.lrid_input_dependent_query:
        with torch.no_grad():
            for gate in m.transformer.lrid_query_gates:
                gate.fill_(0.1)  # zero at init; BASELINE config 3 uses 0.1
    m = m.train() if train else m.eval()
    return m.to(dtype)


def _run(m, idx, train):
    if train:
        h = m(idx, return_hidden=True)
        h.float().square().mean().backward()
        return h.detach()
    with torch.no_grad():
        return m(idx, return_hidden=True)


def record(name, overrides, train, dtype, patched, seed=1234):
    ref_ops, mod = _ref_modules(patched)
    idx_gen = torch.Generator().manual_seed(seed)
    idx = torch.randint(0, overrides["vocab_size"], (overrides.get("batch", 2), overrides["block_size"]),
                        generator=idx_gen)
    if patched:
        # the patched call sites must not change the model
        base_ops, base_mod = _ref_modules(False)
        m0 = _build(base_mod, overrides, True, dtype, train, seed)
        m1 = _build(mod, overrides, True, dtype, train, seed)
        m1.load_state_dict(m0.state_dict())
        h0, h1 = _run(m0, idx, train), _run(m1, idx, train)
        torch.testing.assert_close(h1, h0, rtol=1e-5, atol=1e-6)
        if train:
            for (n0, p0), (_, p1) in zip(m0.named_parameters(), m1.named_parameters()):
                if p0.grad is not None or p1.grad is not None:
                    torch.testing.assert_close(p1.grad, p0.grad, rtol=1e-4, atol=1e-6, msg=lambda s: f"{n0}: {s}")
    rec = Recorder()
    saved = {}
    for n in API + (NEW_API if patched else []):
        if hasattr(mod, n):
            saved[n] = getattr(mod, n)
            setattr(mod, n, _wrap(n, saved[n], rec, train))
    try:
        m = _build(mod, overrides, True, dtype, train, seed)
        hidden = _run(m, idx, train)
    finally:
        for n, f in saved.items():
            setattr(mod, n, f)
    meta = {"config": name, "overrides": overrides, "train": train, "dtype": str(dtype).replace("torch.", ""),
            "patched": patched, "calls": rec.calls}
    arrays = dict(rec.arrays)
    arrays["hidden"] = hidden.float().numpy()
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    os.makedirs(OUT, exist_ok=True)
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **arrays)
    return len(rec.calls)


def main(names=None):
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, (ov, train, dtype, patched) in CONFIGS.items():
        if names and not any(name.startswith(p) for p in names):
            continue
        n = record(name, ov, train, dtype, patched)
        print(f"{name}: {n} calls")


if __name__ == "__main__":
    main(sys.argv[1:])
