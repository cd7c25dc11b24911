"""The config-5 GPT with the fused CUDA reads against its PyTorch read path
(which tests/test_gpt_model.py checks against the reference OBPM).

fp32: logits and every parameter gradient within the fp32 tolerance. bf16: a
multi-layer 16-bit network compounds rounding, so the fused model is held to
what the reference's own bf16 path achieves -- measured against the fp32
PyTorch path on the same (bf16-rounded) weights, its logit and gradient errors
may not exceed 1.5x those of the bf16 PyTorch path (plus 1e-3 of the scale)."""
import pytest
import torch

from gpu_helpers import assert_close

pytestmark = pytest.mark.gpu

KW = [dict(norm_pos="after", lrid_num_heads=2, attnres_num_blocks=3),
      dict(norm_pos="before", lrid_num_heads=1, attnres_num_blocks=4),
      dict(norm_pos="before", lrid_num_heads=2, attnres_num_blocks=2, lrid_key_from_output_tail=True)]
COMMON = dict(n_layer=4, n_head=4, n_embd=512, vocab_size=301, block_size=64, lrid_rank=64,
              attn_res_query_init="normal")


def _run(model, idx):
    out = model(idx)
    out.float().square().mean().backward()
    return out.detach().float(), {n: p.grad.float() for n, p in model.named_parameters()}


def _models(kw, dtype):
    from attnres_b200.gpt import GPT, GPTConfig

    torch.manual_seed(7)
    fused = GPT(GPTConfig(**COMMON, **kw, fused=True)).cuda().to(dtype).train()
    sd = fused.state_dict()
    torch_path = GPT(GPTConfig(**COMMON, **kw, fused=False)).cuda().to(dtype).train()
    torch_path.load_state_dict(sd)
    ref32 = GPT(GPTConfig(**COMMON, **kw, fused=False)).cuda().train()
    ref32.load_state_dict({k: v.float() for k, v in sd.items()})
    return fused, torch_path, ref32


@pytest.mark.parametrize("kw", KW)
def test_gpt_fused_path_matches_torch_path_fp32(kw):
    fused, torch_path, _ = _models(kw, torch.float32)
    idx = torch.randint(0, COMMON["vocab_size"], (2, COMMON["block_size"]), device="cuda")
    (a, ga), (b, gb) = _run(torch_path, idx), _run(fused, idx)
    assert_close("logits", b.cpu().numpy(), a.cpu().numpy(), torch.float32)
    for name in ga:
        assert_close(name, gb[name].cpu().numpy(), ga[name].cpu().numpy(), torch.float32, sum_terms=idx.numel())


@pytest.mark.parametrize("kw", KW)
def test_gpt_fused_bf16_is_as_accurate_as_the_torch_bf16_path(kw):
    fused, torch_path, ref32 = _models(kw, torch.bfloat16)
    idx = torch.randint(0, COMMON["vocab_size"], (2, COMMON["block_size"]), device="cuda")
    (r, gr), (t, gt), (f, gf) = _run(ref32, idx), _run(torch_path, idx), _run(fused, idx)

    def check(name, ours, theirs, exact):
        e_ours = float((ours - exact).abs().max())
        e_theirs = float((theirs - exact).abs().max())
        bound = 1.5 * e_theirs + 1e-3 * float(exact.abs().max())
        assert e_ours <= bound, f"{name}: fused bf16 error {e_ours:.3e} > {bound:.3e} (torch bf16 path {e_theirs:.3e})"

    check("logits", f, t, r)
    for name in gr:
        check(name, gf[name], gt[name], gr[name])
