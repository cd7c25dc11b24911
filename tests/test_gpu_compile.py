"""The fused GPT under torch.compile, as the reference's train.py runs its model
(train.py compiles OBPM). The attnres:: custom ops carry fake implementations
and registered autograd, so dynamo traces the whole model into one graph
(fullgraph=True: no graph break at any read, block summary or projection), and
inductor's compiled forward and backward must give the eager fused model's
logits and parameter gradients."""
import pytest
import torch

from gpu_helpers import assert_close

pytestmark = pytest.mark.gpu

KW = [dict(norm_pos="after", lrid_num_heads=2, attnres_num_blocks=3),
      dict(norm_pos="before", lrid_num_heads=1, attnres_num_blocks=2, lrid_key_from_output_tail=True)]


@pytest.mark.parametrize("kw", KW)
def test_compiled_fused_gpt_matches_eager(kw):
    from attnres_b200.gpt import GPT, GPTConfig

    cfg = GPTConfig(n_layer=3, n_head=4, n_embd=256, vocab_size=301, block_size=32, lrid_rank=64,
                    attn_res_query_init="normal", fused=True, **kw)
    torch.manual_seed(5)
    eager = GPT(cfg).cuda().train()
    compiled_model = GPT(cfg).cuda().train()
    compiled_model.load_state_dict(eager.state_dict())
    compiled = torch.compile(compiled_model, fullgraph=True)
    idx = torch.randint(0, cfg.vocab_size, (2, cfg.block_size), device="cuda")
    outs = []
    for m in (eager, compiled):
        out = m(idx)
        out.float().square().mean().backward()
        outs.append(out.detach().float().cpu().numpy())
    assert_close("logits", outs[1], outs[0], torch.float32)
    ge = dict(eager.named_parameters())
    for name, p in compiled_model.named_parameters():
        assert_close(name, p.grad.cpu().numpy(), ge[name].grad.cpu().numpy(), torch.float32, sum_terms=idx.numel())
