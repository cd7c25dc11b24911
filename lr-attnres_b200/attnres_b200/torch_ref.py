"""PyTorch functions of the reference's attnres_ops API that are PyTorch by
definition there: the `*_torch` reference reads and the phase-2 merges.

They restate attnres_ops.py's own PyTorch code paths (cited per function) so
that `model.py` finds every name it imports. They run on whatever device their
inputs live on; they are separate public functions, never a fallback of the
fused CUDA reads in attnres_b200.ops.
"""
from typing import Optional

import torch
from torch import Tensor
from torch.nn import functional as F

from .ops import phase1_from_logits, source_logit_bias


def _norm(x: Tensor) -> Tensor:
    return F.rms_norm(x, (x.size(-1),))


def _stack(values):
    return values if isinstance(values, Tensor) else torch.stack(list(values), dim=0)


def attention_residual_read_torch(values, query: Tensor, key_norm: bool, source_counts=None,
                                  source_logit_biases=None) -> Tensor:
    """attnres_ops.py:2176-2225: keys = rms_norm(values), logits = <q, k>,
    softmax over sources in fp32, weighted sum in the value dtype."""
    values = _stack(values)
    keys = _norm(values) if key_norm else values
    query = query.to(keys.dtype)
    logits = torch.einsum("d,sbtd->sbt", query, keys)
    bias = source_logit_bias(source_counts, source_logit_biases, values.size(0), logits.device)
    if bias is not None:
        logits = logits + bias.view(-1, 1, 1)
    weights = F.softmax(logits.float(), dim=0).to(values.dtype)
    return torch.einsum("sbt,sbtd->btd", weights, values)


def lrid_attention_residual_read_torch(values, keys, query: Tensor, num_heads: int, logit_scale: float,
                                       key_norm: bool, source_counts=None, source_logit_biases=None) -> Tensor:
    """attnres_ops.py:4163-4256: per-head key rms-norm in fp32, scaled logits,
    softmax over sources in fp32, weighted sum per head."""
    values, keys = _stack(values), _stack(keys)
    H = int(num_heads)
    dk, dv = keys.size(-1) // H, values.size(-1) // H
    keys = keys.reshape(*keys.shape[:-1], H, dk)
    vals = values.reshape(*values.shape[:-1], H, dv)
    if key_norm:
        keys = _norm(keys.float()).to(values.dtype)
    query = query.to(keys.dtype)
    if query.dim() == 4:
        logits = torch.einsum("sbthr,bthr->sbth", keys, query) * logit_scale
    else:
        logits = torch.einsum("sbthr,hr->sbth", keys, query) * logit_scale
    bias = source_logit_bias(source_counts, source_logit_biases, values.size(0), logits.device)
    if bias is not None:
        logits = logits + bias.view(-1, 1, 1, 1)
    weights = F.softmax(logits.float(), dim=0).to(values.dtype)
    out = torch.einsum("sbth,sbthd->bthd", weights, vals)
    return out.reshape(out.size(0), out.size(1), H * dv)


def _add_bias(logit: Tensor, logit_bias) -> Tensor:
    if logit_bias is None:
        return logit
    if isinstance(logit_bias, Tensor):
        return logit + logit_bias.to(device=logit.device, dtype=torch.float32)
    return logit + float(logit_bias) if float(logit_bias) != 0.0 else logit


def attention_residual_phase2_from_logit(partial_value: Tensor, partial_logit: Tensor, interblock_output: Tensor,
                                         interblock_lse: Tensor, force_triton: bool = False,
                                         normalize_output: bool = False) -> Tensor:
    """attnres_ops.py:4043-4072: merge the live partial block into the phase-1
    result, p = sigmoid(logit - lse), out = prev + p * (partial - prev)."""
    prob = torch.sigmoid(partial_logit.float() - interblock_lse.float()).to(partial_value.dtype)
    out = torch.addcmul(interblock_output, partial_value - interblock_output, prob.unsqueeze(-1))
    return _norm(out) if normalize_output else out


def attention_residual_phase2_torch(partial_value: Tensor, query: Tensor, interblock_output: Tensor,
                                    interblock_lse: Tensor, key_norm: bool, normalize_output: bool = False,
                                    logit_bias=0.0) -> Tensor:
    """attnres_ops.py:4022-4040 with the merge of :2630-2642."""
    query = query.to(partial_value.dtype)
    key = _norm(partial_value) if key_norm else partial_value
    logit = _add_bias(torch.sum(key * query.to(key.dtype), dim=-1).float(), logit_bias)
    return attention_residual_phase2_from_logit(partial_value, logit, interblock_output, interblock_lse,
                                                normalize_output=normalize_output)


def attention_residual_phase2(partial_value: Tensor, query: Tensor, interblock_output: Tensor,
                              interblock_lse: Tensor, key_norm: bool, force_triton: bool = False,
                              normalize_output: bool = False, logit_bias=0.0) -> Tensor:
    """attnres_ops.py:3964-4019 (same result as the PyTorch merge)."""
    return attention_residual_phase2_torch(partial_value, query, interblock_output, interblock_lse, key_norm,
                                           normalize_output, logit_bias)


def lrid_attention_residual_phase2_torch(partial_value: Tensor, partial_key: Tensor, query: Tensor,
                                         interblock_output: Tensor, interblock_lse: Tensor, logit_scale: float,
                                         key_norm: bool, normalize_output: bool = False,
                                         logit_bias=0.0) -> Tensor:
    """attnres_ops.py:4142-4160. Unlike the base and given-logit merges (addcmul,
    :2642 and :4071), the LRID merge is a torch.lerp (:4159), which rounds
    differently in 16-bit dtypes."""
    query = query.reshape(-1).to(partial_key.dtype)
    partial_key = partial_key.reshape(partial_key.size(0), partial_key.size(1), -1)
    key = _norm(partial_key.float()).to(partial_value.dtype) if key_norm else partial_key
    logit = torch.sum(key * query.to(key.dtype).view(1, 1, -1), dim=-1) * float(logit_scale)
    logit = _add_bias(logit.float(), logit_bias)
    prob = torch.sigmoid(logit.float() - interblock_lse.float()).to(partial_value.dtype)
    out = torch.lerp(interblock_output, partial_value, prob.unsqueeze(-1))
    return _norm(out) if normalize_output else out


def lrid_attention_residual_phase2(partial_value: Tensor, partial_key: Tensor, query: Tensor,
                                   interblock_output: Tensor, interblock_lse: Tensor, logit_scale: float,
                                   key_norm: bool, force_triton: bool = False, normalize_output: bool = False,
                                   logit_bias=0.0) -> Tensor:
    """attnres_ops.py:4075-4139 (same result as the PyTorch merge)."""
    return lrid_attention_residual_phase2_torch(partial_value, partial_key, query, interblock_output,
                                                interblock_lse, logit_scale, key_norm, normalize_output,
                                                logit_bias)


def attention_residual_phase1(values, queries: Tensor, key_norm: bool, force_triton: bool = False):
    """attnres_ops.py:3862-3907: Q base-AttnRes reads of the same sources;
    logits = <q, rms_norm(v)> per query, then the fused cached-logit read."""
    values = _stack(values)
    queries = queries.to(values.dtype)
    keys = _norm(values) if key_norm else values
    logits = torch.einsum("qd,sbtd->qsbt", queries, keys)
    out, lse, _ = phase1_from_logits(list(values.unbind(0)), logits, False)
    return out, lse
