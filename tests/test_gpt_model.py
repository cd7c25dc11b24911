"""The config-5 GPT (attnres_b200.gpt) against the reference model on the CPU.

The reference's OBPM (model.py) and attnres_b200.gpt.GPT are built with the
same block LR-AttnRes settings; the reference's state_dict loads into the GPT
(same module names), and with the GPT's PyTorch read path both must produce
the same logits and the same parameter gradients. Needs the reference checkout
(ATTNRES_REFERENCE, default the container's copy); skipped where it is absent,
as on the GPU box. tests/test_gpu_gpt.py then checks the GPT's fused (CUDA)
path against this PyTorch path.
"""
import os
import sys

import pytest
import torch

REF = os.environ.get("ATTNRES_REFERENCE", "/root/reference")

pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(REF, "model.py")),
                                reason="reference checkout not available")

SETTINGS = [
    dict(norm_pos="after", lrid_num_heads=2, attnres_num_blocks=2, attnres_block_average_mode="count"),
    dict(norm_pos="before", lrid_num_heads=2, attnres_num_blocks=3, attnres_block_average_mode="sqrt"),
    dict(norm_pos="after", lrid_num_heads=1, attnres_num_blocks=4, attnres_block_count_prior=False),
    dict(norm_pos="before", lrid_num_heads=2, attnres_num_blocks=2, lrid_key_from_output_tail=True),
]


def _reference_model(kw, common):
    if REF not in sys.path:
        sys.path.insert(0, REF)
    import model as M

    return M.OBPM(M.ModelConfig(**common, **kw, use_attnres=True, attnres_type="block", use_lrid=True,
                                attnres_block_average=True, flash_attention=False, use_fused_attnres=False,
                                attn_res_query_init="normal", lrid_use_logit_scale=True))


@pytest.mark.parametrize("kw", SETTINGS)
def test_gpt_torch_path_matches_reference_model(kw):
    from attnres_b200.gpt import GPT, GPTConfig

    common = dict(n_layer=3, n_head=4, n_embd=64, mlp_hidden_dim=128, vocab_size=97, block_size=16, lrid_rank=32)
    torch.manual_seed(3)
    ref = _reference_model(kw, common).train()
    gpt = GPT(GPTConfig(**common, **kw, fused=False, attn_res_query_init="normal")).train()
    missing, unexpected = gpt.load_state_dict(ref.state_dict(), strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    idx = torch.randint(0, common["vocab_size"], (2, common["block_size"]), generator=torch.Generator().manual_seed(4))
    if kw.get("lrid_key_from_output_tail"):
        # tests/test_attnres_ops.py:1306-1327: no key columns, key = value tail
        assert gpt.transformer.layers[0].attn.c_proj.proj.out_features == common["n_embd"]
        with torch.no_grad():
            value, key = gpt.transformer.layers[0].attn.c_proj(torch.randn(2, 8, common["n_embd"]))
        assert key.is_contiguous() and torch.equal(key, value[..., -common["lrid_rank"]:])
    a, b = ref(idx), gpt(idx)
    torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-6)
    a.float().square().mean().backward()
    b.float().square().mean().backward()
    gref = dict(ref.named_parameters())
    for name, p in gpt.named_parameters():
        torch.testing.assert_close(p.grad, gref[name].grad, rtol=1e-4, atol=1e-7, msg=lambda m: f"{name}: {m}")
