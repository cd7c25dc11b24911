"""Block LR-AttnRes GPT for the whole-model measurement.

A compact restatement of the reference model's forward (OBPM, model.py:735 and
its generic block path, model.py:2225-2620) for one family of settings:
`use_attnres` with block AttnRes (`attnres_type="block"`), LRID keys from the
fused output projections (`LRIDFusedProjection`, model.py:316-388, fused-key
layout), static depth queries, the block-count logit prior (legacy beta),
count / sqrt block averaging (legacy alpha), per-head key norm, rotary
embeddings, q/k norm, SwiGLU MLPs and RMS norms before or after each sublayer;
or, with `lrid_key_from_output_tail` (model.py:101, :377-378, :418-419), keys
that are the last `lrid_rank` columns of each source's value.
Module and parameter names follow the reference, so a reference state_dict
loads into it (tests/test_gpt_model.py checks the forward against OBPM).

`fused=True` routes every depth read and block summary through this package's
kernels (`lrid_attention_residual_read`, `attention_residual_block_summary`,
`lrid_fused_projection_forward`); `fused=False` uses the reference's PyTorch
read (model.py:2130-2159) -- the model's unfused path. Everything else
(attention, GEMMs) is PyTorch.
"""
import math
from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch import Tensor


@dataclass
class GPTConfig:
    n_layer: int = 24
    n_head: int = 16
    n_embd: int = 1024
    mlp_hidden_dim: Optional[int] = None  # default n_embd * 4 (model.py:574)
    vocab_size: int = 100277
    block_size: int = 2048
    rope_theta: float = 500000.0
    norm_pos: str = "after"
    qk_norm: bool = True
    init_std: float = 0.02
    attnres_num_blocks: int = 12
    attnres_block_average_mode: str = "count"
    attnres_block_count_prior: bool = True
    attnres_key_norm: bool = True
    attnres_fuse_read_norm: bool = True
    lrid_rank: int = 64
    lrid_num_heads: int = 2
    lrid_key_from_output_tail: bool = False
    pad_vocab_to: int = 64
    attn_res_query_init: str = "zero"
    fused: bool = True

    @property
    def hidden_dim(self) -> int:
        return self.mlp_hidden_dim if self.mlp_hidden_dim is not None else int(self.n_embd * 4)

    @property
    def lrid_logit_scale(self) -> float:
        return 1.0 / math.sqrt(self.lrid_rank // self.lrid_num_heads)  # model.py:203-205


def norm(x: Tensor) -> Tensor:
    return F.rms_norm(x, (x.size(-1),))


def norm_heads(x: Tensor, heads: int) -> Tensor:
    """Per-head RMS norm of the last dim (model.py:34-37)."""
    s = x.shape
    return norm(x.reshape(*s[:-1], heads, s[-1] // heads)).reshape(s)


class RotaryEmbedding(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        dim = cfg.n_embd // cfg.n_head
        inv_freq = 1.0 / (cfg.rope_theta ** (torch.arange(0, dim, 2) / dim))
        freq = torch.outer(torch.arange(cfg.block_size), inv_freq)
        self.register_buffer("sin", freq.sin()[None, None])
        self.register_buffer("cos", freq.cos()[None, None])

    def rotate(self, x: Tensor) -> Tensor:
        T = x.size(-2)
        sin, cos = self.sin[:, :, :T], self.cos[:, :, :T]
        x1, x2 = x[..., 0::2], x[..., 1::2]
        return torch.stack([cos * x1 - sin * x2, sin * x1 + cos * x2], dim=-1).flatten(-2)


class LRIDFusedProjection(nn.Module):
    """Output projection emitting the sublayer output and its LRID key (the
    reference's fused-key layout: one weight [output + rank, input]; with the
    output-tail key, weight [output, input] and key = output[..., -rank:])."""

    def __init__(self, cfg: GPTConfig, input_dim: int, output_dim: int):
        super().__init__()
        self.cfg = cfg
        self.output_dim = output_dim
        extra = 0 if cfg.lrid_key_from_output_tail else cfg.lrid_rank
        self.proj = nn.Linear(input_dim, output_dim + extra, bias=False)

    def forward(self, x: Tensor):
        c = self.cfg
        if c.lrid_key_from_output_tail:
            out = self.proj(x)
            # the fused read takes the key as a strided view of the output rows;
            # the PyTorch path copies it like the reference (model.py:377-378)
            key = out[..., -c.lrid_rank:]
            return out, (key if c.fused else key.contiguous())
        if c.fused:
            from .ops import lrid_fused_projection_forward

            return lrid_fused_projection_forward(x, self.proj.weight, self.output_dim, c.lrid_rank, c.lrid_num_heads,
                                                 c.attnres_key_norm)
        y = self.proj(x)
        out = y[..., :self.output_dim].contiguous()
        key = y[..., self.output_dim:self.output_dim + c.lrid_rank]
        if c.attnres_key_norm:
            key = norm_heads(key, c.lrid_num_heads)
        return out, key


class LRIDSourceKeyProjection(nn.Module):
    """Key of the embedding source (model.py:391-423): proj(x), per-head normed,
    or the last `lrid_rank` columns of x with the output-tail key."""

    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.cfg = cfg
        self.proj = None if cfg.lrid_key_from_output_tail else nn.Linear(cfg.n_embd, cfg.lrid_rank, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        if self.proj is None:
            key = x[..., -self.cfg.lrid_rank:]
            return key if self.cfg.fused else key.contiguous()
        key = self.proj(x)
        return norm_heads(key, self.cfg.lrid_num_heads) if self.cfg.attnres_key_norm else key


class MultiHeadAttention(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.cfg = cfg
        self.head_dim = cfg.n_embd // cfg.n_head
        self.rope = RotaryEmbedding(cfg)
        self.c_attn = nn.Linear(cfg.n_embd, 3 * cfg.n_embd, bias=False)
        self.c_proj = LRIDFusedProjection(cfg, cfg.n_embd, cfg.n_embd)

    def forward(self, x: Tensor):
        B, T, C = x.shape
        q, k, v = self.c_attn(x).split(C, dim=2)
        q, k, v = (t.view(B, T, self.cfg.n_head, self.head_dim).transpose(1, 2) for t in (q, k, v))
        if self.cfg.qk_norm:
            q, k = norm(q), norm(k)
        q, k = self.rope.rotate(q), self.rope.rotate(k)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.c_proj(y.transpose(1, 2).contiguous().view(B, T, C))


class MLP(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.fc1 = nn.Linear(cfg.n_embd, cfg.hidden_dim * 2, bias=False)
        self.fc2 = LRIDFusedProjection(cfg, cfg.hidden_dim, cfg.n_embd)

    def forward(self, x: Tensor):
        x, gate = self.fc1(x).chunk(2, dim=-1)
        return self.fc2(F.silu(gate) * x)


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.cfg = cfg
        self.attn = MultiHeadAttention(cfg)
        self.mlp = MLP(cfg)

    def _sublayer(self, f, x: Tensor, x_is_normalized: bool):
        if self.cfg.norm_pos == "before" and not x_is_normalized:
            x = norm(x)
        out, key = f(x)
        if self.cfg.norm_pos == "after":
            out = norm(out)
        return out, key

    def forward_attention(self, x, x_is_normalized=False):
        return self._sublayer(self.attn, x, x_is_normalized)

    def forward_mlp(self, x, x_is_normalized=False):
        return self._sublayer(self.mlp, x, x_is_normalized)


class GPT(nn.Module):
    """OBPM with block LR-AttnRes (see the module docstring)."""

    def __init__(self, cfg: GPTConfig):
        super().__init__()
        self.cfg = cfg
        H, dk = cfg.lrid_num_heads, cfg.lrid_rank // cfg.lrid_num_heads
        self.transformer = nn.ModuleDict(dict(
            wte=nn.Embedding(cfg.vocab_size, cfg.n_embd),
            layers=nn.ModuleList([Block(cfg) for _ in range(cfg.n_layer)]),
            lrid_embedding_key=LRIDSourceKeyProjection(cfg),
            lrid_queries=nn.ParameterList([nn.Parameter(torch.empty(H, dk)) for _ in range(2 * cfg.n_layer)]),
        ))
        self.lm_head = nn.Linear(cfg.n_embd, cfg.vocab_size, bias=False)
        total = 2 * cfg.n_layer
        nb = min(cfg.attnres_num_blocks, total)
        self.block_ends = frozenset(math.ceil(total * i / nb) for i in range(1, nb + 1))  # model.py:828-836
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, mean=0.0, std=cfg.init_std)
        for q in self.transformer.lrid_queries:
            if cfg.attn_res_query_init == "zero":
                nn.init.zeros_(q)
            else:
                nn.init.normal_(q, mean=0.0, std=cfg.init_std)

    # ---- block bookkeeping (model.py:955-1069) --------------------------------
    def _scale(self, count: int) -> float:
        alpha = 0.5 if self.cfg.attnres_block_average_mode == "sqrt" else 1.0
        return float(count) ** (-alpha)

    def _bias(self, count: int) -> float:
        return math.log(float(count)) if (self.cfg.attnres_block_count_prior and count != 1) else 0.0

    def _biases(self, counts):
        b = [self._bias(c) for c in counts]
        return b if any(v != 0.0 for v in b) else None

    def _summary(self, partial: Optional[Tensor], out: Tensor, count: int):
        """New running block sum and its block source value (sum * count^-alpha)."""
        if self.cfg.fused:
            from .ops import attention_residual_block_summary

            alpha = 0.5 if self.cfg.attnres_block_average_mode == "sqrt" else 1.0
            return attention_residual_block_summary(partial, out, count=count, alpha=alpha)
        s = out if partial is None else partial + out
        return s, s * self._scale(count)

    def _read(self, idx: int, values, keys, biases, normalize_output: bool) -> Tensor:
        """The depth read at residual site `idx` (model.py:2081-2159)."""
        if len(values) == 1:
            return norm(values[0]) if normalize_output else values[0]
        c = self.cfg
        query = self.transformer.lrid_queries[idx - 1]
        if c.fused:
            from .ops import lrid_attention_residual_read

            return lrid_attention_residual_read(values, keys, query, c.lrid_num_heads, c.lrid_logit_scale,
                                                c.attnres_key_norm, normalize_output=normalize_output,
                                                source_logit_biases=biases)
        from .torch_ref import lrid_attention_residual_read_torch

        out = lrid_attention_residual_read_torch(values, keys, query, c.lrid_num_heads, c.lrid_logit_scale,
                                                 c.attnres_key_norm, source_logit_biases=biases)
        return norm(out) if normalize_output else out

    def forward(self, idx: Tensor, return_hidden: bool = False) -> Tensor:
        c = self.cfg
        x = self.transformer.wte(idx)
        fused_read_norm = (c.fused and c.norm_pos == "before" and c.attnres_fuse_read_norm
                           and c.lrid_num_heads == 1)  # model.py:2237-2243
        # completed block sources (value, key) and their counts; the live block
        done_v, done_k, done_n = [x], [self.transformer.lrid_embedding_key(x)], [1]
        part, part_src, part_key, part_n = None, None, None, 0

        def sources():
            if part is None:
                return done_v, done_k, done_n
            return done_v + [part_src], done_k + [part_key], done_n + [part_n]

        def read(site):
            v, k, n = sources()
            return self._read(site, v, k, self._biases(n), fused_read_norm)

        for li, block in enumerate(self.transformer.layers):
            for sub, f in ((0, block.forward_attention), (1, block.forward_mlp)):
                site = 2 * li + sub
                x = read(site) if site > 0 else (norm(x) if fused_read_norm else x)
                out, key = f(x, x_is_normalized=fused_read_norm)
                part_n += 1
                part, part_src = self._summary(part, out, part_n)
                part_key = key if part_n == 1 else part_key + key
                if site + 1 in self.block_ends:
                    done_v.append(part_src)
                    done_k.append(part_key)
                    done_n.append(part_n)
                    part, part_src, part_key, part_n = None, None, None, 0
        x = read(2 * c.n_layer)
        if not fused_read_norm:
            x = norm(x)
        return x if return_hidden else self.logits(x)

    def logits(self, x: Tensor) -> Tensor:
        """lm_head(x). With a vocabulary that is not a multiple of
        `pad_vocab_to` (the reference's 100 277 is odd) the logit rows are not
        16-byte aligned and the library GEMMs fall back to slow kernels, so
        the logits are computed against the weight padded with zero rows and
        returned as the [..., :vocab] view: the same values; the pad's backward
        drops the padding's gradient. Both read paths do this."""
        w = self.lm_head.weight
        pad = -w.size(0) % self.cfg.pad_vocab_to if self.cfg.pad_vocab_to > 1 else 0
        if pad == 0:
            return self.lm_head(x)
        return F.linear(x, F.pad(w, (0, 0, 0, pad)))[..., :w.size(0)]
