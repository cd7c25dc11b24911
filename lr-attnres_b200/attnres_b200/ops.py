"""torch.library operators and public read functions over libattnres_b200.

Mirrors the reference's op layer (attnres_ops.py of jon123boss/LR-AttnRes):

  attnres::lrid_read_list / attnres::lrid_read_list_backward
      same names, schemas and outputs as attnres_ops.py:4636-4802, including
      register_autograd (attnres_ops.py:4805-4847).
  attnres::lrid_read / attnres::lrid_read_backward
      the general LRID read used by the public function: static, dynamic or
      gated-hybrid query (model.py:2102-2115), per-source logit biases
      (attnres_ops.py:84-105), and output RMS norm per head or per row.
  attnres::base_read / attnres::base_read_backward
      the base AttnRes read (attnres_ops.py:2301-2421).
  lrid_attention_residual_read(...)   signature of attnres_ops.py:4852
  attention_residual_read(...)        signature of attnres_ops.py:2503

Every tensor argument must live on a CUDA device; the work is enqueued on the
current stream through the C ABI. There is no CPU fallback: a CPU tensor is a
RuntimeError.
"""
import ctypes
import os
from typing import List, Optional, Sequence

import torch
from torch import Tensor
from torch.nn import functional as F

from . import _native as N

F32_EPS = float(torch.finfo(torch.float32).eps)

_DTYPES = {torch.float32: N.DTYPE_F32, torch.float16: N.DTYPE_F16, torch.bfloat16: N.DTYPE_BF16}


def _dtype_code(dt):
    try:
        return _DTYPES[dt]
    except KeyError:
        raise RuntimeError(f"attnres_b200: unsupported dtype {dt}; use float32, float16 or bfloat16") from None


def _require_cuda(tensors, what):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                f"attnres_b200: {what} must be CUDA tensors (the fused read has no CPU path)"
            )


def _stream_ptr(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _row_view(t: Tensor, width: int):
    """A token-row view of a [B, T, width] / [N, width] source: returns the
    tensor (made dense in its last dim if needed) and its row stride."""
    if t.size(-1) != width:
        raise RuntimeError(f"attnres_b200: source last dim {t.size(-1)} != {width}")
    if t.dim() == 3:
        if t.stride(-1) != 1 or t.stride(0) != t.size(1) * t.stride(1):
            t = t.contiguous()
        return t, (t.stride(1) if t.size(1) > 1 or t.size(0) > 1 else width)
    if t.dim() == 2:
        if t.stride(-1) != 1:
            t = t.contiguous()
        return t, (t.stride(0) if t.size(0) > 1 else width)
    raise RuntimeError("attnres_b200: sources must be [B, T, C] or [N, C]")


def _sources(tensors: Sequence[Tensor], width: int, dtype):
    rows, strides = [], []
    for t in tensors:
        if t.dtype != dtype:
            raise RuntimeError("attnres_b200: all sources of a read must share one dtype")
        t, st = _row_view(t, width)
        rows.append(t)
        strides.append(max(int(st), width))
    return rows, strides


def _ntok(t: Tensor):
    return t.numel() // t.size(-1)


def _lead_shape(t: Tensor):
    return tuple(t.shape[:-1])


def _output_norm_mode(normalize_output: bool, num_heads: int) -> int:
    """The reference fuses the output norm per head when H == 1 and otherwise
    RMS-normalises the whole output row (attnres_ops.py:4871, :4985)."""
    if not normalize_output:
        return N.NORM_NONE
    return N.NORM_PER_HEAD if int(num_heads) == 1 else N.NORM_ROW


# ---------------------------------------------------------------------------
# raw launchers (no autograd)
# ---------------------------------------------------------------------------
def _lrid_forward_impl(values, keys, query, query_gate, query_dynamic, logit_bias, num_heads,
                       logit_scale, key_norm, output_norm, save_aux):
    S = len(values)
    if S < 1 or len(keys) != S:
        raise RuntimeError("attnres_b200: need one key tensor per value source (S >= 1)")
    if S > N.MAX_SOURCES:
        raise RuntimeError(f"attnres_b200: at most {N.MAX_SOURCES} sources per read")
    _require_cuda([*values, *keys, query, query_gate, query_dynamic, logit_bias], "LRID read inputs")
    H = int(num_heads)
    d = values[0].size(-1)
    R = keys[0].size(-1)
    if H < 1 or d % H or R % H:
        raise RuntimeError(f"attnres_b200: value dim {d} and key dim {R} must divide by num_heads {H}")
    dtype = values[0].dtype
    code = _dtype_code(dtype)
    vrows, vstr = _sources(values, d, dtype)
    krows, kstr = _sources(keys, R, dtype)
    n = _ntok(values[0])
    device = values[0].device
    qmode, q, g, qd = _query_pack(query, query_gate, query_dynamic, H, R, n, dtype)
    bias = None if logit_bias is None else logit_bias.to(torch.float32).reshape(-1).contiguous()
    if bias is not None and bias.numel() != S:
        raise RuntimeError("source_logit_biases length must match the number of sources")
    out = torch.empty((*_lead_shape(values[0]), d), device=device, dtype=dtype)
    if output_norm == N.NORM_PER_HEAD:
        out_inv = torch.empty((n, H), device=device, dtype=torch.float32)
    elif output_norm == N.NORM_ROW:
        out_inv = torch.empty((n,), device=device, dtype=torch.float32)
    else:
        out_inv = torch.empty((1,), device=device, dtype=torch.float32)
    if save_aux:
        alpha = torch.empty((n, H, S), device=device, dtype=torch.float32)
        kinv = torch.empty((n, H, S), device=device, dtype=torch.float32)
    else:
        alpha = torch.empty((1,), device=device, dtype=torch.float32)
        kinv = torch.empty((1,), device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        rc = N.load().attnres_lrid_forward(
            S, n, d, R, H, code,
            N.ptr_array([t.data_ptr() for t in vrows]), N.i64_array(vstr),
            N.ptr_array([t.data_ptr() for t in krows]), N.i64_array(kstr),
            qmode, _ptr(q), _ptr(g), _ptr(qd),
            float(logit_scale), int(bool(key_norm)), F32_EPS, _ptr(bias),
            int(output_norm), _rms_eps(),
            _ptr(out), _ptr(out_inv) if output_norm != N.NORM_NONE else None,
            _ptr(alpha) if save_aux else None, _ptr(kinv) if save_aux else None,
            _stream_ptr(device),
        )
    N.check(rc, "attnres_lrid_forward")
    return out, out_inv, alpha, kinv


def _query_pack(query, gate, query_dynamic, H, R, n, dtype):
    dk = R // H
    if query_dynamic is not None:
        qd = query_dynamic.to(dtype).reshape(n, H, dk).contiguous()
        if query is None:
            return N.QUERY_DYNAMIC, None, None, qd
        if gate is None:
            raise RuntimeError("attnres_b200: a gated query needs query_gate")
        q = query.to(dtype).reshape(H, dk).contiguous()
        g = gate.to(dtype).reshape(H).contiguous()
        return N.QUERY_GATED, q, g, qd
    if query is None:
        raise RuntimeError("attnres_b200: query is required")
    if query.dim() == 4:
        return N.QUERY_DYNAMIC, None, None, query.to(dtype).reshape(n, H, dk).contiguous()
    if query.numel() != R:
        raise RuntimeError(f"attnres_b200: static query must have {R} elements ([H, R/H])")
    return N.QUERY_STATIC, query.to(dtype).reshape(H, dk).contiguous(), None, None


def _lrid_backward_impl(values, keys, query, query_gate, query_dynamic, logit_bias, grad_output,
                        normed_output, output_inv_rms, num_heads, logit_scale, key_norm,
                        output_norm, need_bias_grad=True, write_dv=True):
    S = len(values)
    H = int(num_heads)
    d = values[0].size(-1)
    R = keys[0].size(-1)
    dtype = values[0].dtype
    code = _dtype_code(dtype)
    _require_cuda([*values, *keys, query, query_gate, query_dynamic, logit_bias, grad_output],
                  "LRID read backward inputs")
    vrows, vstr = _sources(values, d, dtype)
    krows, kstr = _sources(keys, R, dtype)
    n = _ntok(values[0])
    device = values[0].device
    qmode, q, g, qd = _query_pack(query, query_gate, query_dynamic, H, R, n, dtype)
    bias = None if logit_bias is None else logit_bias.to(torch.float32).reshape(-1).contiguous()
    grad_output = grad_output.to(dtype).reshape(n, d).contiguous()
    y = None
    if output_norm != N.NORM_NONE:
        y = normed_output.to(dtype).reshape(n, d).contiguous()
        output_inv_rms = output_inv_rms.to(torch.float32).contiguous()
    grad_values = [torch.empty((*_lead_shape(v), d), device=device, dtype=dtype) for v in values]
    grad_keys = [torch.empty((*_lead_shape(k), R), device=device, dtype=dtype) for k in keys]
    if qmode == N.QUERY_DYNAMIC:
        dq = torch.empty((n, H, R // H), device=device, dtype=dtype)
    else:
        dq = torch.empty((H, R // H), device=device, dtype=torch.float32)
    dgate = torch.empty((H,), device=device, dtype=torch.float32) if qmode == N.QUERY_GATED else None
    dqd = torch.empty((n, H, R // H), device=device, dtype=dtype) if qmode == N.QUERY_GATED else None
    dbias = torch.empty((S,), device=device, dtype=torch.float32) if (bias is not None and need_bias_grad) else None
    with torch.cuda.device(device):
        L = N.load()
        ws_bytes = L.attnres_lrid_backward_workspace_bytes(S, n, d, R, H, code)
        ws = torch.empty((max(16, ws_bytes),), device=device, dtype=torch.uint8)
        rc = L.attnres_lrid_backward(
            S, n, d, R, H, code,
            N.ptr_array([t.data_ptr() for t in vrows]), N.i64_array(vstr),
            N.ptr_array([t.data_ptr() for t in krows]), N.i64_array(kstr),
            qmode, _ptr(q), _ptr(g), _ptr(qd),
            float(logit_scale), int(bool(key_norm)), F32_EPS, _ptr(bias),
            int(output_norm), _rms_eps(),
            _ptr(grad_output), _ptr(y), _ptr(output_inv_rms) if y is not None else None,
            N.ptr_array([t.data_ptr() for t in grad_values]) if write_dv else None,
            N.ptr_array([t.data_ptr() for t in grad_keys]),
            _ptr(dq), _ptr(dgate), _ptr(dqd), _ptr(dbias),
            _ptr(ws), ws.numel(), _stream_ptr(device),
        )
    N.check(rc, "attnres_lrid_backward")
    return grad_values, grad_keys, dq, dgate, dqd, dbias


# ---------------------------------------------------------------------------
# attnres::lrid_read_list — reference-compatible library op
# ---------------------------------------------------------------------------
@torch.library.custom_op("attnres::lrid_read_list", mutates_args=())
def lrid_read_list(
    values: List[Tensor],
    keys: List[Tensor],
    query: Tensor,
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    normalize_output: bool,
    save_aux: bool,
) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """Reference attnres_ops.py:4636. normalize_output normalises each head."""
    norm = N.NORM_PER_HEAD if normalize_output else N.NORM_NONE
    out, inv, alpha, kinv = _lrid_forward_impl(
        list(values), list(keys), query, None, None, None, num_heads, logit_scale, key_norm,
        norm, save_aux,
    )
    return out, inv, alpha, kinv


@lrid_read_list.register_fake
def _(values, keys, query, num_heads, logit_scale, key_norm, normalize_output, save_aux):
    v0 = values[0]
    n = v0.numel() // v0.size(-1)
    H, S = int(num_heads), len(values)
    out = v0.new_empty(v0.shape)
    inv = v0.new_empty((n, H) if normalize_output else (1,), dtype=torch.float32)
    aux = (n, H, S) if save_aux else (1,)
    return out, inv, v0.new_empty(aux, dtype=torch.float32), v0.new_empty(aux, dtype=torch.float32)


@torch.library.custom_op("attnres::lrid_read_list_backward", mutates_args=())
def lrid_read_list_backward(
    values: List[Tensor],
    keys: List[Tensor],
    query: Tensor,
    grad_output: Tensor,
    normed_output: Tensor,
    output_inv_rms: Tensor,
    alpha_saved: Tensor,
    key_inv_rms_saved: Tensor,
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    normalize_output: bool,
    use_aux: bool,
) -> tuple[List[Tensor], List[Tensor], Tensor]:
    """Reference attnres_ops.py:4725. The softmax weights are recomputed from the
    keys with the forward's arithmetic, so `alpha_saved` / `key_inv_rms_saved`
    (use_aux) are accepted for interface parity and give identical results."""
    norm = N.NORM_PER_HEAD if normalize_output else N.NORM_NONE
    gv, gk, dq, _, _, _ = _lrid_backward_impl(
        list(values), list(keys), query, None, None, None, grad_output, normed_output,
        output_inv_rms, num_heads, logit_scale, key_norm, norm,
    )
    return gv, gk, dq.reshape(query.shape).to(query.dtype)


@lrid_read_list_backward.register_fake
def _(values, keys, query, grad_output, normed_output, output_inv_rms, alpha_saved,
      key_inv_rms_saved, num_heads, logit_scale, key_norm, normalize_output, use_aux):
    return ([v.new_empty(v.shape) for v in values], [k.new_empty(k.shape) for k in keys],
            query.new_empty(query.shape))


def _lrid_read_list_setup(ctx, inputs, output):
    values, keys, query, num_heads, logit_scale, key_norm, normalize_output, save_aux = inputs
    out, inv, alpha, kinv = output
    ctx.save_for_backward(query, out, inv, alpha, kinv, *values, *keys)
    ctx.num_sources = len(values)
    ctx.num_heads = int(num_heads)
    ctx.logit_scale = float(logit_scale)
    ctx.key_norm = bool(key_norm)
    ctx.normalize_output = bool(normalize_output)
    ctx.use_aux = bool(save_aux)


def _lrid_read_list_bwd(ctx, grad_out, grad_inv, grad_alpha, grad_kinv):
    saved = ctx.saved_tensors
    query, out, inv, alpha, kinv = saved[:5]
    values = list(saved[5:5 + ctx.num_sources])
    keys = list(saved[5 + ctx.num_sources:])
    gv, gk, dq = lrid_read_list_backward(
        values, keys, query, grad_out, out, inv, alpha, kinv, ctx.num_heads, ctx.logit_scale,
        ctx.key_norm, ctx.normalize_output, ctx.use_aux,
    )
    return gv, gk, dq, None, None, None, None, None


lrid_read_list.register_autograd(_lrid_read_list_bwd, setup_context=_lrid_read_list_setup)


# ---------------------------------------------------------------------------
# attnres::lrid_read — general LRID read (gated query, logit bias, row norm)
# ---------------------------------------------------------------------------
@torch.library.custom_op("attnres::lrid_read", mutates_args=())
def lrid_read(
    values: List[Tensor],
    keys: List[Tensor],
    query: Optional[Tensor],
    query_gate: Optional[Tensor],
    query_dynamic: Optional[Tensor],
    logit_bias: Optional[Tensor],
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    output_norm: int,
) -> tuple[Tensor, Tensor]:
    out, inv, _, _ = _lrid_forward_impl(
        list(values), list(keys), query, query_gate, query_dynamic, logit_bias, num_heads,
        logit_scale, key_norm, int(output_norm), False,
    )
    return out, inv


@lrid_read.register_fake
def _(values, keys, query, query_gate, query_dynamic, logit_bias, num_heads, logit_scale,
      key_norm, output_norm):
    v0 = values[0]
    n = v0.numel() // v0.size(-1)
    shape = {N.NORM_PER_HEAD: (n, int(num_heads)), N.NORM_ROW: (n,)}.get(int(output_norm), (1,))
    return v0.new_empty(v0.shape), v0.new_empty(shape, dtype=torch.float32)


@torch.library.custom_op("attnres::lrid_read_backward", mutates_args=())
def lrid_read_backward(
    values: List[Tensor],
    keys: List[Tensor],
    query: Optional[Tensor],
    query_gate: Optional[Tensor],
    query_dynamic: Optional[Tensor],
    logit_bias: Optional[Tensor],
    grad_output: Tensor,
    normed_output: Tensor,
    output_inv_rms: Tensor,
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    output_norm: int,
) -> tuple[List[Tensor], List[Tensor], Tensor, Tensor, Tensor, Tensor]:
    """Returns (dV list, dK list, dq, dgate, dq_dynamic, dbias); dq is fp32 [H, dk]
    for a static/gated query and [N, H, dk] in the value dtype for a dynamic one;
    absent gradients are returned as empty tensors."""
    gv, gk, dq, dgate, dqd, dbias = _lrid_backward_impl(
        list(values), list(keys), query, query_gate, query_dynamic, logit_bias, grad_output,
        normed_output, output_inv_rms, num_heads, logit_scale, key_norm, int(output_norm),
    )
    e = values[0].new_empty((0,), dtype=torch.float32)
    return (gv, gk, dq, dgate if dgate is not None else e, dqd if dqd is not None else e.clone(),
            dbias if dbias is not None else e.clone())


@lrid_read_backward.register_fake
def _(values, keys, query, query_gate, query_dynamic, logit_bias, grad_output, normed_output,
      output_inv_rms, num_heads, logit_scale, key_norm, output_norm):
    v0 = values[0]
    n = v0.numel() // v0.size(-1)
    H, R = int(num_heads), keys[0].size(-1)
    e = v0.new_empty((0,), dtype=torch.float32)
    if query_dynamic is not None and query is None:
        dq = v0.new_empty((n, H, R // H))
    else:
        dq = v0.new_empty((H, R // H), dtype=torch.float32)
    gated = query_dynamic is not None and query is not None
    return ([v.new_empty(v.shape) for v in values], [k.new_empty(k.shape) for k in keys], dq,
            v0.new_empty((H,), dtype=torch.float32) if gated else e,
            v0.new_empty((n, H, R // H)) if gated else e.clone(),
            v0.new_empty((len(values),), dtype=torch.float32) if logit_bias is not None else e.clone())


def _lrid_read_setup(ctx, inputs, output):
    values, keys, query, gate, qdyn, bias, num_heads, logit_scale, key_norm, output_norm = inputs
    out, inv = output
    ctx.has = (query is not None, gate is not None, qdyn is not None, bias is not None)
    opt = [x for x in (query, gate, qdyn, bias) if x is not None]
    ctx.save_for_backward(out, inv, *opt, *values, *keys)
    ctx.num_sources = len(values)
    ctx.n_opt = len(opt)
    ctx.args = (int(num_heads), float(logit_scale), bool(key_norm), int(output_norm))


def _lrid_read_bwd(ctx, grad_out, grad_inv):
    saved = list(ctx.saved_tensors)
    out, inv = saved[0], saved[1]
    opt = iter(saved[2:2 + ctx.n_opt])
    query, gate, qdyn, bias = (next(opt) if h else None for h in ctx.has)
    rest = saved[2 + ctx.n_opt:]
    values, keys = list(rest[:ctx.num_sources]), list(rest[ctx.num_sources:])
    H, scale, key_norm, output_norm = ctx.args
    gv, gk, dq, dgate, dqd, dbias = lrid_read_backward(
        values, keys, query, gate, qdyn, bias, grad_out, out, inv, H, scale, key_norm, output_norm,
    )
    g_query = g_gate = g_qdyn = g_bias = None
    if qdyn is not None and query is None:
        g_qdyn = dq.reshape(qdyn.shape).to(qdyn.dtype)
    else:
        g_query = dq.reshape(query.shape).to(query.dtype)
        if qdyn is not None:
            g_gate = dgate.reshape(gate.shape).to(gate.dtype)
            g_qdyn = dqd.reshape(qdyn.shape).to(qdyn.dtype)
    if bias is not None:
        g_bias = dbias.reshape(bias.shape).to(bias.dtype)
    return gv, gk, g_query, g_gate, g_qdyn, g_bias, None, None, None, None


lrid_read.register_autograd(_lrid_read_bwd, setup_context=_lrid_read_setup)


# ---------------------------------------------------------------------------
# attnres::base_read — base AttnRes read (keys are rms-normed values)
# ---------------------------------------------------------------------------
def _base_forward_impl(values, query, logit_bias, key_norm, normalize_output):
    S = len(values)
    if S < 1 or S > N.MAX_SOURCES:
        raise RuntimeError(f"attnres_b200: base read needs 1..{N.MAX_SOURCES} sources")
    _require_cuda([*values, query, logit_bias], "base read inputs")
    d = values[0].size(-1)
    dtype = values[0].dtype
    code = _dtype_code(dtype)
    rows, strides = _sources(values, d, dtype)
    n = _ntok(values[0])
    device = values[0].device
    q = query.to(dtype).reshape(d).contiguous()
    bias = None if logit_bias is None else logit_bias.to(torch.float32).reshape(-1).contiguous()
    eps = _rms_eps()
    out = torch.empty((*_lead_shape(values[0]), d), device=device, dtype=dtype)
    inv = torch.empty((n,) if normalize_output else (1,), device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        rc = N.load().attnres_base_forward(
            S, n, d, code, N.ptr_array([t.data_ptr() for t in rows]), N.i64_array(strides),
            _ptr(q), int(bool(key_norm)), eps, _ptr(bias),
            N.NORM_ROW if normalize_output else N.NORM_NONE, eps,
            _ptr(out), _ptr(inv) if normalize_output else None, _stream_ptr(device),
        )
    N.check(rc, "attnres_base_forward")
    return out, inv


@torch.library.custom_op("attnres::base_read", mutates_args=())
def base_read(
    values: List[Tensor],
    query: Tensor,
    logit_bias: Optional[Tensor],
    key_norm: bool,
    normalize_output: bool,
) -> tuple[Tensor, Tensor]:
    return _base_forward_impl(list(values), query, logit_bias, key_norm, normalize_output)


@base_read.register_fake
def _(values, query, logit_bias, key_norm, normalize_output):
    v0 = values[0]
    n = v0.numel() // v0.size(-1)
    return v0.new_empty(v0.shape), v0.new_empty((n,) if normalize_output else (1,), dtype=torch.float32)


@torch.library.custom_op("attnres::base_read_backward", mutates_args=())
def base_read_backward(
    values: List[Tensor],
    query: Tensor,
    logit_bias: Optional[Tensor],
    grad_output: Tensor,
    normed_output: Tensor,
    output_inv_rms: Tensor,
    key_norm: bool,
    normalize_output: bool,
) -> tuple[List[Tensor], Tensor, Tensor]:
    values = list(values)
    S = len(values)
    d = values[0].size(-1)
    dtype = values[0].dtype
    code = _dtype_code(dtype)
    _require_cuda([*values, query, grad_output], "base read backward inputs")
    rows, strides = _sources(values, d, dtype)
    n = _ntok(values[0])
    device = values[0].device
    q = query.to(dtype).reshape(d).contiguous()
    bias = None if logit_bias is None else logit_bias.to(torch.float32).reshape(-1).contiguous()
    eps = _rms_eps()
    g = grad_output.to(dtype).reshape(n, d).contiguous()
    y = normed_output.to(dtype).reshape(n, d).contiguous() if normalize_output else None
    inv = output_inv_rms.to(torch.float32).contiguous() if normalize_output else None
    gv = [torch.empty((*_lead_shape(v), d), device=device, dtype=dtype) for v in values]
    dq = torch.empty((d,), device=device, dtype=torch.float32)
    dbias = torch.empty((S,), device=device, dtype=torch.float32) if bias is not None else None
    with torch.cuda.device(device):
        L = N.load()
        ws_bytes = L.attnres_base_backward_workspace_bytes(S, n, d, code)
        ws = torch.empty((max(16, ws_bytes),), device=device, dtype=torch.uint8)
        rc = L.attnres_base_backward(
            S, n, d, code, N.ptr_array([t.data_ptr() for t in rows]), N.i64_array(strides),
            _ptr(q), int(bool(key_norm)), eps, _ptr(bias),
            N.NORM_ROW if normalize_output else N.NORM_NONE, eps,
            _ptr(g), _ptr(y), _ptr(inv), N.ptr_array([t.data_ptr() for t in gv]),
            _ptr(dq), _ptr(dbias), _ptr(ws), ws.numel(), _stream_ptr(device),
        )
    N.check(rc, "attnres_base_backward")
    e = values[0].new_empty((0,), dtype=torch.float32)
    return gv, dq.reshape(query.shape).to(query.dtype), dbias if dbias is not None else e


@base_read_backward.register_fake
def _(values, query, logit_bias, grad_output, normed_output, output_inv_rms, key_norm,
      normalize_output):
    e = values[0].new_empty((0,), dtype=torch.float32)
    db = values[0].new_empty((len(values),), dtype=torch.float32) if logit_bias is not None else e
    return [v.new_empty(v.shape) for v in values], query.new_empty(query.shape), db


def _base_read_setup(ctx, inputs, output):
    values, query, bias, key_norm, normalize_output = inputs
    out, inv = output
    ctx.has_bias = bias is not None
    ctx.save_for_backward(out, inv, query, *([bias] if bias is not None else []), *values)
    ctx.args = (bool(key_norm), bool(normalize_output))


def _base_read_bwd(ctx, grad_out, grad_inv):
    saved = list(ctx.saved_tensors)
    out, inv, query = saved[:3]
    bias = saved[3] if ctx.has_bias else None
    values = saved[4 if ctx.has_bias else 3:]
    key_norm, normalize_output = ctx.args
    gv, dq, dbias = base_read_backward(values, query, bias, grad_out, out, inv, key_norm, normalize_output)
    g_bias = dbias.reshape(bias.shape).to(bias.dtype) if bias is not None else None
    return gv, dq, g_bias, None, None


base_read.register_autograd(_base_read_bwd, setup_context=_base_read_setup)


# ---------------------------------------------------------------------------
# public functions (signatures of the reference's attnres_ops.py)
# ---------------------------------------------------------------------------
def _norm(x: Tensor) -> Tensor:
    return F.rms_norm(x, (x.size(-1),))


def _rms_eps() -> float:
    """The eps of the reference's RMS norms, F.rms_norm(x, eps=None)
    (attnres_ops.py:49-52, model.py:28-31): PyTorch takes the eps of the type it
    computes in, fp32 for fp32, fp16 and bf16 inputs alike -- not the eps of the
    16-bit input dtype (7.8e-3 for bf16, which would change rows of small RMS)."""
    return F32_EPS


def source_logit_bias(source_counts, source_logit_biases, n_sources: int, device) -> Optional[Tensor]:
    """Per-source fp32 logit bias: log(count) for `source_counts`, or the given
    (possibly learned) biases. Same rules and errors as attnres_ops.py:61-105."""
    if source_counts is not None and source_logit_biases is not None:
        raise RuntimeError("source_counts and source_logit_biases are mutually exclusive")
    if source_logit_biases is None:
        if source_counts is None:
            return None
        if isinstance(source_counts, Tensor):
            counts = source_counts.reshape(-1).to(device=device, dtype=torch.float32)
        elif isinstance(source_counts, (int, float)):
            counts = torch.full((n_sources,), float(source_counts), device=device, dtype=torch.float32)
        else:
            if len(source_counts) != n_sources:
                raise RuntimeError("source_counts length must match the number of sources")
            vals = [float(c) for c in source_counts]
            if any(c <= 0.0 for c in vals):
                raise RuntimeError("source_counts must be positive")
            counts = torch.tensor(vals, device=device, dtype=torch.float32)
        if counts.numel() != n_sources:
            raise RuntimeError("source_counts length must match the number of sources")
        return counts.log()
    if isinstance(source_logit_biases, Tensor):
        biases = source_logit_biases.reshape(-1).to(device=device, dtype=torch.float32)
    elif isinstance(source_logit_biases, (int, float)):
        biases = torch.full((n_sources,), float(source_logit_biases), device=device, dtype=torch.float32)
    else:
        if len(source_logit_biases) != n_sources:
            raise RuntimeError("source_logit_biases length must match the number of sources")
        biases = torch.stack([
            b.to(device=device, dtype=torch.float32).reshape(())
            if isinstance(b, Tensor) else torch.tensor(float(b), device=device, dtype=torch.float32)
            for b in source_logit_biases
        ])
    if biases.numel() != n_sources:
        raise RuntimeError("source_logit_biases length must match the number of sources")
    return biases


def _as_list(x):
    return list(x.unbind(0)) if isinstance(x, Tensor) else list(x)


def lrid_attention_residual_read(
    values,
    keys,
    query: Tensor,
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    force_triton: bool = False,
    normalize_output: bool = False,
    source_counts=None,
    source_logit_biases=None,
) -> Tensor:
    """LR-AttnRes read (reference attnres_ops.py:4852). `values`/`keys` are lists
    (or stacked [S, ...] tensors) of [B, T, d] / [B, T, R]; `query` is static
    [H, R/H] or dynamic [B, T, H, R/H]. `force_triton` is accepted for signature
    compatibility; the fused CUDA path is the only path."""
    values, keys = _as_list(values), _as_list(keys)
    query = query.to(keys[0].dtype)
    if len(values) == 1:
        return _norm(values[0]) if normalize_output else values[0]
    if keys[0].dtype != values[0].dtype:
        keys = [k.to(values[0].dtype) for k in keys]
    bias = source_logit_bias(source_counts, source_logit_biases, len(values), values[0].device)
    norm = _output_norm_mode(normalize_output, num_heads)
    if query.dim() == 4:
        out, _ = lrid_read(values, keys, None, None, query, bias, int(num_heads), float(logit_scale),
                           bool(key_norm), norm)
    else:
        out, _ = lrid_read(values, keys, query, None, None, bias, int(num_heads), float(logit_scale),
                           bool(key_norm), norm)
    return out


def lrid_attention_residual_read_gated(
    values,
    keys,
    static_query: Tensor,
    query_gate: Tensor,
    dynamic_query: Tensor,
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    normalize_output: bool = False,
    source_counts=None,
    source_logit_biases=None,
) -> Tensor:
    """LR-AttnRes read with the input-dependent gated hybrid query
    q_t = static_query + query_gate * dynamic_query_t (model.py:2104-2110), formed
    inside the kernel. Gradients flow to all three query tensors."""
    values, keys = _as_list(values), _as_list(keys)
    dtype = keys[0].dtype
    if len(values) == 1:
        return _norm(values[0]) if normalize_output else values[0]
    if keys[0].dtype != values[0].dtype:
        keys = [k.to(values[0].dtype) for k in keys]
    bias = source_logit_bias(source_counts, source_logit_biases, len(values), values[0].device)
    norm = _output_norm_mode(normalize_output, num_heads)
    out, _ = lrid_read(values, keys, static_query.to(dtype), query_gate.to(dtype), dynamic_query.to(dtype),
                       bias, int(num_heads), float(logit_scale), bool(key_norm), norm)
    return out


def attention_residual_read(
    values,
    query: Tensor,
    key_norm: bool,
    force_triton: bool = False,
    normalize_output: bool = False,
    source_counts=None,
    source_logit_biases=None,
) -> Tensor:
    """Base AttnRes read (reference attnres_ops.py:2503): keys are the rms-normed
    values, logits <key, query> (+ per-source bias), softmax over sources."""
    values = _as_list(values)
    if len(values) == 1:
        return _norm(values[0]) if normalize_output else values[0]
    query = query.to(values[0].dtype)
    bias = source_logit_bias(source_counts, source_logit_biases, len(values), values[0].device)
    out, _ = base_read(values, query, bias, bool(key_norm), bool(normalize_output))
    return out


def is_fused_attnres_available() -> bool:
    """True when the CUDA library loads and a CUDA device is present."""
    try:
        N.load()
    except N.AttnResError:
        return False
    return torch.cuda.is_available()


# ---------------------------------------------------------------------------
# attnres::lrid_kv_read — LRID read with keys projected from the values
# (lrid_key_from_value: keys_s = rms_norm(V_s) @ W^T, model.py:344-356)
# ---------------------------------------------------------------------------
def _kv_project(values, weight, value_norm):
    S = len(values)
    d = values[0].size(-1)
    R = weight.size(0)
    if weight.dim() != 2 or weight.size(1) != d:
        raise RuntimeError(f"attnres_b200: key weight must be [R, {d}] (nn.Linear weight)")
    dtype = values[0].dtype
    _require_cuda([*values, weight], "key projection inputs")
    rows, strides = _sources(values, d, dtype)
    n = _ntok(values[0])
    device = values[0].device
    w = weight.to(dtype)
    if w.stride(-1) != 1:
        w = w.contiguous()
    keys = torch.empty((S, *_lead_shape(values[0]), R), device=device, dtype=dtype)
    inv = torch.empty((S, n), device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        rc = N.load().attnres_lrid_key_projection(
            S, n, d, R, _dtype_code(dtype), N.ptr_array([t.data_ptr() for t in rows]), N.i64_array(strides),
            _ptr(w), int(w.stride(0)), int(bool(value_norm)), _rms_eps(),
            _ptr(keys), _ptr(inv), _stream_ptr(device))
    N.check(rc, "attnres_lrid_key_projection")
    return keys, inv


def _kv_fused_forward(values, weight, query, bias, H, scale, key_norm, value_norm):
    """The one-kernel key-from-value forward (projection, softmax and weighted
    sum with V read from HBM once: clusters of value_dim / 512 CTAs, W held in
    tensor memory, partial keys reduce-scattered through distributed shared
    memory); returns (out, keys [S, *lead, R], value_inv_rms [S, N],
    alpha [N, H, S]), or None when it is not selected or the shapes are outside
    the kernel. It is selected with ATTNRES_KV_FWD=one: at config 4 it measures
    4.6 ms against 3.4 ms for the projection kernel followed by the read kernel
    (a ring stage waits ~10 us for its logits to return through the cluster),
    so the two-kernel path is the default."""
    if os.environ.get("ATTNRES_KV_FWD", "") != "one":
        return None
    S, d, R = len(values), values[0].size(-1), weight.size(0)
    dtype = values[0].dtype
    if dtype not in (torch.float16, torch.bfloat16):
        return None
    rows, strides = _sources(values, d, dtype)
    n = _ntok(values[0])
    device = values[0].device
    w = weight.to(dtype)
    if w.stride(-1) != 1:
        w = w.contiguous()
    q = query.to(dtype).reshape(-1).contiguous()
    b = None if bias is None else bias.to(torch.float32).reshape(-1).contiguous()
    out = torch.empty((*_lead_shape(values[0]), d), device=device, dtype=dtype)
    keys = torch.empty((S, *_lead_shape(values[0]), R), device=device, dtype=dtype)
    inv = torch.empty((S, n), device=device, dtype=torch.float32)
    alpha = torch.empty((n, H, S), device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        rc = N.load().attnres_lrid_key_from_value_forward(
            S, n, d, R, int(H), _dtype_code(dtype), N.ptr_array([t.data_ptr() for t in rows]), N.i64_array(strides),
            _ptr(w), int(w.stride(0)), int(bool(value_norm)), _rms_eps(), _ptr(q), float(scale), int(bool(key_norm)),
            F32_EPS, _ptr(b), _ptr(out), _ptr(keys), _ptr(inv), _ptr(alpha), _stream_ptr(device))
    if rc == 2:  # ATTNRES_ERR_UNSUPPORTED: outside the one-kernel shapes
        return None
    N.check(rc, "attnres_lrid_key_from_value_forward")
    return out, keys, inv, alpha


@torch.library.custom_op("attnres::lrid_kv_read", mutates_args=())
def lrid_kv_read(
    values: List[Tensor],
    key_weight: Tensor,
    query: Optional[Tensor],
    query_gate: Optional[Tensor],
    query_dynamic: Optional[Tensor],
    logit_bias: Optional[Tensor],
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    output_norm: int,
    value_norm: bool,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns (out, output_inv_rms, keys [S, *lead, R], value_inv_rms [S, N],
    alpha [N, H, S] -- the softmax weights, kept so the backward forms dV in
    one pass; [1] when the output is normalised)."""
    values = list(values)
    if int(output_norm) == N.NORM_NONE and query is not None and query_dynamic is None and len(values) > 1:
        _require_cuda([*values, key_weight, query, logit_bias], "key-from-value read inputs")
        fused = _kv_fused_forward(values, key_weight, query, logit_bias, int(num_heads), logit_scale, key_norm,
                                  value_norm)
        if fused is not None:
            out, keys, inv, alpha = fused
            return out, out.new_empty((1,), dtype=torch.float32), keys, inv, alpha
    keys, inv = _kv_project(values, key_weight, value_norm)
    save = int(output_norm) == N.NORM_NONE
    out, oinv, alpha, _ = _lrid_forward_impl(values, list(keys.unbind(0)), query, query_gate, query_dynamic,
                                             logit_bias, num_heads, logit_scale, key_norm, int(output_norm), save)
    return out, oinv, keys, inv, alpha


@lrid_kv_read.register_fake
def _(values, key_weight, query, query_gate, query_dynamic, logit_bias, num_heads, logit_scale, key_norm,
      output_norm, value_norm):
    v0 = values[0]
    n = v0.numel() // v0.size(-1)
    S, R = len(values), key_weight.size(0)
    shape = {N.NORM_PER_HEAD: (n, int(num_heads)), N.NORM_ROW: (n,)}.get(int(output_norm), (1,))
    aux = (n, int(num_heads), S) if int(output_norm) == N.NORM_NONE else (1,)
    return (v0.new_empty(v0.shape), v0.new_empty(shape, dtype=torch.float32),
            v0.new_empty((S, *v0.shape[:-1], R)), v0.new_empty((S, n), dtype=torch.float32),
            v0.new_empty(aux, dtype=torch.float32))


def _kv_backward_one_pass(values, key_weight, keys, value_inv_rms, alpha, query, logit_bias, grad_output, output,
                          H, scale, key_norm, value_norm):
    """Key-from-value read backward with a static query in one kernel that
    reads each value row once (the read backward, the key-norm backward and
    the key-projection backward fused; partial dots exchanged between the
    column slices of a token tile through cluster shared memory). Selected
    with ATTNRES_KV_BWD=one: at config 4 it measures 12-16 ms against 5.4 ms
    for the read backward followed by the tensor-core projection backward (a
    ring stage stays resident through the exchange round trip), so the
    two-kernel path is the default. Returns the lrid_kv_read_backward tuple,
    or None when the shapes are outside the kernel."""
    S, d, R = len(values), values[0].size(-1), key_weight.size(0)
    dtype = values[0].dtype
    n = _ntok(values[0])
    device = values[0].device
    with torch.cuda.device(device):
        L = N.load()
        ws_bytes = L.attnres_lrid_key_from_value_backward_workspace_bytes(S, n, d, R, int(H), _dtype_code(dtype))
        if ws_bytes == 0:
            return None
        rows, strides = _sources(values, d, dtype)
        w = key_weight.to(dtype)
        if w.stride(-1) != 1:
            w = w.contiguous()
        q = query.to(dtype).reshape(-1).contiguous()
        g = grad_output.to(dtype).reshape(n, d).contiguous()
        out = output.to(dtype).reshape(n, d).contiguous()
        gv = [torch.empty(v.shape, device=device, dtype=dtype) for v in values]
        dw = torch.empty((R, d), device=device, dtype=torch.float32)
        dq = torch.empty((int(H), R // int(H)), device=device, dtype=torch.float32)
        e = values[0].new_empty((0,), dtype=torch.float32)
        dbias = torch.empty((S,), device=device, dtype=torch.float32) if logit_bias is not None else None
        ws = torch.empty(ws_bytes, device=device, dtype=torch.uint8)
        kd = keys.reshape(S, n, R).contiguous()
        vinv = value_inv_rms.contiguous()
        al = alpha.contiguous()
        rc = L.attnres_lrid_key_from_value_backward(
            S, n, d, R, int(H), _dtype_code(dtype), N.ptr_array([t.data_ptr() for t in rows]), N.i64_array(strides),
            _ptr(w), int(w.stride(0)), _ptr(kd), int(bool(value_norm)), _ptr(vinv), _ptr(al), _ptr(q), float(scale), int(bool(key_norm)),
            F32_EPS, _ptr(g), _ptr(out), N.ptr_array([t.data_ptr() for t in gv]), _ptr(dw), _ptr(dq),
            _ptr(dbias), _ptr(ws), ws_bytes, _stream_ptr(device))
    N.check(rc, "attnres_lrid_key_from_value_backward")
    return gv, dw, dq, e, e.clone(), dbias if dbias is not None else e.clone()


@torch.library.custom_op("attnres::lrid_kv_read_backward", mutates_args=())
def lrid_kv_read_backward(
    values: List[Tensor],
    key_weight: Tensor,
    keys: Tensor,
    value_inv_rms: Tensor,
    alpha: Tensor,
    query: Optional[Tensor],
    query_gate: Optional[Tensor],
    query_dynamic: Optional[Tensor],
    logit_bias: Optional[Tensor],
    grad_output: Tensor,
    normed_output: Tensor,
    output_inv_rms: Tensor,
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    output_norm: int,
    value_norm: bool,
) -> tuple[List[Tensor], Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns (dV list, d key_weight [R, d] fp32, dq, dgate, dq_dynamic, dbias)."""
    values = list(values)
    S, d = len(values), values[0].size(-1)
    R = key_weight.size(0)
    dtype = values[0].dtype
    one_pass = int(output_norm) == N.NORM_NONE and alpha.numel() > 1
    if (one_pass and query is not None and query_gate is None and query_dynamic is None
            and os.environ.get("ATTNRES_KV_BWD", "tc") == "one"):
        fused = _kv_backward_one_pass(values, key_weight, keys, value_inv_rms, alpha, query, logit_bias, grad_output,
                                      normed_output, int(num_heads), logit_scale, key_norm, value_norm)
        if fused is not None:
            return fused
    gv, gk, dq, dgate, dqd, dbias = _lrid_backward_impl(
        values, list(keys.unbind(0)), query, query_gate, query_dynamic, logit_bias, grad_output, normed_output,
        output_inv_rms, num_heads, logit_scale, key_norm, int(output_norm), write_dv=not one_pass)
    n = _ntok(values[0])
    g_rows = grad_output.to(dtype).reshape(n, d).contiguous() if one_pass else None
    device = values[0].device
    if one_pass and os.environ.get("ATTNRES_KV_BWD", "tc") != "gemm":
        # fused tensor-core projection backward: dV written once, dW in the same pass
        with torch.cuda.device(device):
            L = N.load()
            ws_bytes = L.attnres_lrid_key_projection_backward_tc_workspace_bytes(
                S, n, d, R, int(num_heads), _dtype_code(dtype))
            if ws_bytes > 0:
                rows, strides = _sources(values, d, dtype)
                w = key_weight.to(dtype)
                ws = torch.empty(ws_bytes, device=device, dtype=torch.uint8)
                dw = torch.empty((R, d), device=device, dtype=torch.float32)
                gks = [g.reshape(n, R).contiguous() for g in gk]
                rc = L.attnres_lrid_key_projection_backward_tc(
                    S, n, d, R, int(num_heads), _dtype_code(dtype), N.ptr_array([t.data_ptr() for t in rows]),
                    N.i64_array(strides), _ptr(w), w.stride(0), N.ptr_array([g.data_ptr() for g in gks]),
                    _ptr(keys.reshape(S, n, R)), _ptr(value_inv_rms), _ptr(g_rows), _ptr(alpha.contiguous()),
                    int(bool(value_norm)), N.ptr_array([g.data_ptr() for g in gv]), _ptr(dw), _ptr(ws), ws_bytes,
                    _stream_ptr(device))
                N.check(rc, "attnres_lrid_key_projection_backward_tc")
                e = values[0].new_empty((0,), dtype=torch.float32)
                return (gv, dw, dq, dgate if dgate is not None else e, dqd if dqd is not None else e.clone(),
                        dbias if dbias is not None else e.clone())
    dk = torch.stack([g.reshape(n, R) for g in gk])  # [S, n, R]
    w = key_weight.to(dtype)
    dn = torch.matmul(dk, w)  # [S, n, d]: plain GEMM (cuBLAS)
    rows, strides = _sources(values, d, dtype)
    with torch.cuda.device(device):
        rc = N.load().attnres_lrid_key_projection_backward(
            S, n, d, R, int(num_heads), _dtype_code(dtype), N.ptr_array([t.data_ptr() for t in rows]),
            N.i64_array(strides), N.ptr_array([g.data_ptr() for g in gv]), _ptr(dn), _ptr(dk),
            _ptr(keys.reshape(S, n, R)), _ptr(value_inv_rms), _ptr(g_rows),
            _ptr(alpha.contiguous()) if one_pass else None, int(bool(value_norm)), _stream_ptr(device))
    N.check(rc, "attnres_lrid_key_projection_backward")
    # d W = sum_s (inv_s * dK_s)^T @ V_s  (plain GEMMs, fp32 accumulation over sources)
    dw = torch.zeros((R, d), device=device, dtype=torch.float32)
    scale = value_inv_rms if value_norm else torch.ones_like(value_inv_rms)
    for s in range(S):
        a = (dk[s].float() * scale[s].unsqueeze(-1)).to(dtype)
        dw += torch.matmul(a.t(), rows[s].reshape(n, d)).float()
    e = values[0].new_empty((0,), dtype=torch.float32)
    return (gv, dw, dq, dgate if dgate is not None else e, dqd if dqd is not None else e.clone(),
            dbias if dbias is not None else e.clone())


@lrid_kv_read_backward.register_fake
def _(values, key_weight, keys, value_inv_rms, alpha, query, query_gate, query_dynamic, logit_bias, grad_output,
      normed_output, output_inv_rms, num_heads, logit_scale, key_norm, output_norm, value_norm):
    v0 = values[0]
    n = v0.numel() // v0.size(-1)
    H, R = int(num_heads), key_weight.size(0)
    e = v0.new_empty((0,), dtype=torch.float32)
    if query_dynamic is not None and query is None:
        dq = v0.new_empty((n, H, R // H))
    else:
        dq = v0.new_empty((H, R // H), dtype=torch.float32)
    gated = query_dynamic is not None and query is not None
    return ([v.new_empty(v.shape) for v in values], key_weight.new_empty(key_weight.shape, dtype=torch.float32), dq,
            v0.new_empty((H,), dtype=torch.float32) if gated else e,
            v0.new_empty((n, H, R // H)) if gated else e.clone(),
            v0.new_empty((len(values),), dtype=torch.float32) if logit_bias is not None else e.clone())


def _lrid_kv_setup(ctx, inputs, output):
    (values, key_weight, query, gate, qdyn, bias, num_heads, logit_scale, key_norm, output_norm,
     value_norm) = inputs
    out, oinv, keys, inv, alpha = output
    ctx.has = (query is not None, gate is not None, qdyn is not None, bias is not None)
    opt = [x for x in (query, gate, qdyn, bias) if x is not None]
    ctx.save_for_backward(out, oinv, keys, inv, alpha, key_weight, *opt, *values)
    ctx.n_opt = len(opt)
    ctx.args = (int(num_heads), float(logit_scale), bool(key_norm), int(output_norm), bool(value_norm))


def _lrid_kv_bwd(ctx, grad_out, grad_oinv, grad_keys, grad_inv, grad_alpha):
    saved = list(ctx.saved_tensors)
    out, oinv, keys, inv, alpha, key_weight = saved[:6]
    opt = iter(saved[6:6 + ctx.n_opt])
    query, gate, qdyn, bias = (next(opt) if h else None for h in ctx.has)
    values = saved[6 + ctx.n_opt:]
    H, scale, key_norm, output_norm, value_norm = ctx.args
    gv, dw, dq, dgate, dqd, dbias = lrid_kv_read_backward(
        values, key_weight, keys, inv, alpha, query, gate, qdyn, bias, grad_out, out, oinv, H, scale, key_norm,
        output_norm, value_norm)
    g_query = g_gate = g_qdyn = g_bias = None
    if qdyn is not None and query is None:
        g_qdyn = dq.reshape(qdyn.shape).to(qdyn.dtype)
    else:
        g_query = dq.reshape(query.shape).to(query.dtype)
        if qdyn is not None:
            g_gate = dgate.reshape(gate.shape).to(gate.dtype)
            g_qdyn = dqd.reshape(qdyn.shape).to(qdyn.dtype)
    if bias is not None:
        g_bias = dbias.reshape(bias.shape).to(bias.dtype)
    return gv, dw.to(key_weight.dtype), g_query, g_gate, g_qdyn, g_bias, None, None, None, None, None


lrid_kv_read.register_autograd(_lrid_kv_bwd, setup_context=_lrid_kv_setup)


def lrid_attention_residual_read_key_from_value(
    values,
    key_weight: Tensor,
    query: Tensor,
    num_heads: int,
    logit_scale: float,
    key_norm: bool,
    normalize_output: bool = False,
    value_norm: bool = True,
    source_counts=None,
    source_logit_biases=None,
    query_gate: Optional[Tensor] = None,
    dynamic_query: Optional[Tensor] = None,
) -> Tensor:
    """LR-AttnRes read whose keys are projected from the values inside the op:
    keys_s = rms_norm(V_s) @ key_weight^T (lrid_key_from_value, unshared;
    model.py:344-356 with `value_key_proj.weight` as key_weight and
    `lrid_key_value_norm` as value_norm). The projection runs on tcgen05
    tensor cores for bf16/fp16 rows that allow it. Gradients flow to the values
    (through both the read and the projection), key_weight and the query."""
    values = _as_list(values)
    if len(values) == 1:
        return _norm(values[0]) if normalize_output else values[0]
    dtype = values[0].dtype
    bias = source_logit_bias(source_counts, source_logit_biases, len(values), values[0].device)
    norm = _output_norm_mode(normalize_output, num_heads)
    if dynamic_query is not None and query_gate is not None:
        q, g, qd = query.to(dtype), query_gate.to(dtype), dynamic_query.to(dtype)
    elif query.dim() == 4:
        q, g, qd = None, None, query.to(dtype)
    else:
        q, g, qd = query.to(dtype), None, None
    out, _, _, _, _ = lrid_kv_read(values, key_weight, q, g, qd, bias, int(num_heads), float(logit_scale),
                                   bool(key_norm), norm, bool(value_norm))
    return out


# ---------------------------------------------------------------------------
# attnres::phase1_from_logits — cached-logit block read (attnres_ops.py:3910)
# ---------------------------------------------------------------------------
@torch.library.custom_op("attnres::phase1_from_logits", mutates_args=())
def phase1_from_logits(values: List[Tensor], logits: Tensor, normalize_output: bool) -> tuple[Tensor, Tensor, Tensor]:
    """values: S sources [*lead, D]; logits [Q, S, *lead]. Returns
    (out [Q, *lead, D], lse [Q, *lead] fp32, output_inv_rms [Q, N] or [1])."""
    values = list(values)
    S, d = len(values), values[0].size(-1)
    if S < 1 or S > N.MAX_SOURCES:
        raise RuntimeError(f"attnres_b200: phase1 needs 1..{N.MAX_SOURCES} sources")
    Q = logits.size(0)
    if logits.size(1) != S:
        raise RuntimeError("attnres_b200: logits must be [Q, S, ...] with S = number of sources")
    _require_cuda([*values, logits], "phase1 inputs")
    dtype = values[0].dtype
    rows, strides = _sources(values, d, dtype)
    n = _ntok(values[0])
    lead = _lead_shape(values[0])
    lg = logits.reshape(Q, S, n).contiguous()
    device = values[0].device
    out = torch.empty((Q, *lead, d), device=device, dtype=dtype)
    lse = torch.empty((Q, *lead), device=device, dtype=torch.float32)
    inv = torch.empty((Q, n) if normalize_output else (1,), device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        rc = N.load().attnres_phase1_forward(
            S, Q, n, d, _dtype_code(dtype), N.ptr_array([t.data_ptr() for t in rows]), N.i64_array(strides),
            _ptr(lg), _dtype_code(lg.dtype), N.NORM_ROW if normalize_output else N.NORM_NONE,
            _rms_eps(), _ptr(out), _ptr(lse), _ptr(inv) if normalize_output else None,
            _stream_ptr(device))
    N.check(rc, "attnres_phase1_forward")
    return out, lse, inv


@phase1_from_logits.register_fake
def _(values, logits, normalize_output):
    v0 = values[0]
    n = v0.numel() // v0.size(-1)
    Q = logits.size(0)
    return (v0.new_empty((Q, *v0.shape)), v0.new_empty((Q, *v0.shape[:-1]), dtype=torch.float32),
            v0.new_empty((Q, n) if normalize_output else (1,), dtype=torch.float32))


@torch.library.custom_op("attnres::phase1_from_logits_backward", mutates_args=())
def phase1_from_logits_backward(values: List[Tensor], logits: Tensor, grad_output: Tensor,
                                grad_lse: Optional[Tensor], normed_output: Tensor, output_inv_rms: Tensor,
                                normalize_output: bool) -> tuple[List[Tensor], Tensor]:
    values = list(values)
    S, d = len(values), values[0].size(-1)
    Q = logits.size(0)
    dtype = values[0].dtype
    rows, strides = _sources(values, d, dtype)
    n = _ntok(values[0])
    lg = logits.reshape(Q, S, n).contiguous()
    device = values[0].device
    g = grad_output.to(dtype).reshape(Q, n, d).contiguous()
    gl = None if grad_lse is None else grad_lse.to(torch.float32).reshape(Q, n).contiguous()
    y = normed_output.to(dtype).reshape(Q, n, d).contiguous() if normalize_output else None
    yi = output_inv_rms.contiguous() if normalize_output else None
    gv = [torch.empty((*_lead_shape(v), d), device=device, dtype=dtype) for v in values]
    dlg = torch.empty_like(lg)
    with torch.cuda.device(device):
        rc = N.load().attnres_phase1_backward(
            S, Q, n, d, _dtype_code(dtype), N.ptr_array([t.data_ptr() for t in rows]), N.i64_array(strides),
            _ptr(lg), _dtype_code(lg.dtype), N.NORM_ROW if normalize_output else N.NORM_NONE,
            _rms_eps(), _ptr(g), _ptr(gl), _ptr(y), _ptr(yi),
            N.ptr_array([t.data_ptr() for t in gv]), _ptr(dlg), _stream_ptr(device))
    N.check(rc, "attnres_phase1_backward")
    return gv, dlg.reshape(logits.shape)


@phase1_from_logits_backward.register_fake
def _(values, logits, grad_output, grad_lse, normed_output, output_inv_rms, normalize_output):
    return [v.new_empty(v.shape) for v in values], logits.new_empty(logits.shape)


def _phase1_setup(ctx, inputs, output):
    values, logits, normalize_output = inputs
    out, lse, inv = output
    ctx.save_for_backward(logits, out, inv, *values)
    ctx.normalize_output = bool(normalize_output)


def _phase1_bwd(ctx, grad_out, grad_lse, grad_inv):
    logits, out, inv, *values = ctx.saved_tensors
    gv, dlg = phase1_from_logits_backward(list(values), logits, grad_out, grad_lse, out, inv, ctx.normalize_output)
    return gv, dlg, None


phase1_from_logits.register_autograd(_phase1_bwd, setup_context=_phase1_setup)


def attention_residual_phase1_from_logits(values, logits: Tensor, force_triton: bool = False,
                                          normalize_output: bool = False):
    """Cached-logit block read (reference attnres_ops.py:3910): values are S
    sources (list or stacked [S, ...]), logits [Q, S, ...]. Returns
    (out [Q, ..., D], lse [Q, ...] fp32)."""
    values = _as_list(values)
    if len(values) == 0:
        raise RuntimeError("Cached-logit AttnRes phase1 requires at least one source")
    out, lse, _ = phase1_from_logits(values, logits, bool(normalize_output))
    return out, lse


def attention_residual_average_read(values, normalize_output: bool = False, force_triton: bool = False) -> Tensor:
    """Mean over the sources (reference attnres_ops.py:2568): the base read with
    a zero query and no key norm gives every source the weight 1/S."""
    values = _as_list(values)
    if len(values) == 1:
        return _norm(values[0]) if normalize_output else values[0]
    q = torch.zeros(values[0].size(-1), device=values[0].device, dtype=values[0].dtype)
    out, _ = base_read(values, q, None, False, bool(normalize_output))
    return out


# ---------------------------------------------------------------------------
# attnres::block_summary — running block sum and scaled block source (one pass)
# ---------------------------------------------------------------------------
@torch.library.custom_op("attnres::block_summary", mutates_args=())
def block_summary(partial: Optional[Tensor], x: Tensor, scale: Optional[Tensor],
                  scale_value: float) -> tuple[Tensor, Tensor]:
    """sum = partial + x (partial None: sum = x), source = sum * c with c the
    device scalar `scale` (fp32, one element) when given, else `scale_value`."""
    _require_cuda([partial, x, scale], "block summary inputs")
    dtype = x.dtype
    xc = x.contiguous()
    pc = None if partial is None else partial.to(dtype).contiguous()
    if pc is not None and pc.shape != xc.shape:
        raise RuntimeError("attnres_b200: block summary partial and x must have one shape")
    sc = None if scale is None else scale.to(torch.float32).reshape(1).contiguous()
    out_sum = torch.empty_like(xc)
    src = torch.empty_like(xc)
    with torch.cuda.device(x.device):
        rc = N.load().attnres_block_summary_forward(
            xc.numel(), _dtype_code(dtype), _ptr(pc), _ptr(xc), _ptr(sc), float(scale_value), _ptr(out_sum),
            _ptr(src), _stream_ptr(x.device))
    N.check(rc, "attnres_block_summary_forward")
    return out_sum, src


@block_summary.register_fake
def _(partial, x, scale, scale_value):
    return x.new_empty(x.shape), x.new_empty(x.shape)


@torch.library.custom_op("attnres::block_summary_backward", mutates_args=())
def block_summary_backward(grad_source: Optional[Tensor], grad_sum: Optional[Tensor], out_sum: Tensor,
                           scale: Optional[Tensor], scale_value: float, want_scale_grad: bool) -> tuple[Tensor, Tensor]:
    """Returns (gradient of partial and of x, scale gradient [1] fp32 or empty)."""
    dtype = out_sum.dtype
    gs = None if grad_source is None else grad_source.to(dtype).contiguous()
    gm = None if grad_sum is None else grad_sum.to(dtype).contiguous()
    sc = None if scale is None else scale.to(torch.float32).reshape(1).contiguous()
    n = out_sum.numel()
    g = torch.empty_like(out_sum)
    dsc = torch.empty((1,) if want_scale_grad else (0,), device=out_sum.device, dtype=torch.float32)
    L = N.load()
    ws_bytes = L.attnres_block_summary_backward_workspace_bytes(n) if want_scale_grad else 0
    ws = torch.empty((max(ws_bytes, 1),), device=out_sum.device, dtype=torch.uint8)
    with torch.cuda.device(out_sum.device):
        rc = L.attnres_block_summary_backward(
            n, _dtype_code(dtype), _ptr(gs), _ptr(gm), _ptr(out_sum), _ptr(sc), float(scale_value), _ptr(g),
            _ptr(dsc) if want_scale_grad else None, _ptr(ws), ws_bytes, _stream_ptr(out_sum.device))
    N.check(rc, "attnres_block_summary_backward")
    return g, dsc


@block_summary_backward.register_fake
def _(grad_source, grad_sum, out_sum, scale, scale_value, want_scale_grad):
    return out_sum.new_empty(out_sum.shape), out_sum.new_empty((1,) if want_scale_grad else (0,),
                                                               dtype=torch.float32)


def _block_summary_setup(ctx, inputs, output):
    partial, x, scale, scale_value = inputs
    out_sum, _ = output
    ctx.has_partial = partial is not None
    ctx.scale_value = float(scale_value)
    ctx.scale_shape = None if scale is None else scale.shape
    ctx.scale_dtype = None if scale is None else scale.dtype
    ctx.save_for_backward(out_sum, scale)


def _block_summary_bwd(ctx, grad_sum, grad_source):
    out_sum, scale = ctx.saved_tensors
    want = scale is not None and ctx.needs_input_grad[2]
    g, dsc = block_summary_backward(grad_source, grad_sum, out_sum, scale, ctx.scale_value, want)
    dscale = dsc.reshape(ctx.scale_shape).to(ctx.scale_dtype) if want else None
    return (g if ctx.has_partial else None, g, dscale, None)


block_summary.register_autograd(_block_summary_bwd, setup_context=_block_summary_setup)


@torch.library.custom_op("attnres::block_summary_norm", mutates_args=())
def block_summary_norm(partial: Optional[Tensor], x: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """sum = partial + x, source = rms_norm(sum) over the last dim (fp32 eps);
    returns (sum, source, inverse rms [rows] fp32)."""
    _require_cuda([partial, x], "block summary inputs")
    dtype = x.dtype
    d = x.size(-1)
    xc = x.contiguous()
    pc = None if partial is None else partial.to(dtype).contiguous()
    if pc is not None and pc.shape != xc.shape:
        raise RuntimeError("attnres_b200: block summary partial and x must have one shape")
    rows = xc.numel() // d
    out_sum, src = torch.empty_like(xc), torch.empty_like(xc)
    inv = torch.empty((rows,), device=x.device, dtype=torch.float32)
    with torch.cuda.device(x.device):
        rc = N.load().attnres_block_summary_norm_forward(
            rows, d, _dtype_code(dtype), _ptr(pc), _ptr(xc), _rms_eps(), _ptr(out_sum), _ptr(src), _ptr(inv),
            _stream_ptr(x.device))
    N.check(rc, "attnres_block_summary_norm_forward")
    return out_sum, src, inv


@block_summary_norm.register_fake
def _(partial, x):
    return x.new_empty(x.shape), x.new_empty(x.shape), x.new_empty((x.numel() // x.size(-1),), dtype=torch.float32)


@torch.library.custom_op("attnres::block_summary_norm_backward", mutates_args=())
def block_summary_norm_backward(grad_source: Tensor, grad_sum: Optional[Tensor], out_sum: Tensor,
                                inv_rms: Tensor) -> Tensor:
    """The gradient of partial and of x."""
    dtype = out_sum.dtype
    d = out_sum.size(-1)
    rows = out_sum.numel() // d
    gs = grad_source.to(dtype).contiguous()
    gm = None if grad_sum is None else grad_sum.to(dtype).contiguous()
    g = torch.empty_like(out_sum)
    with torch.cuda.device(out_sum.device):
        rc = N.load().attnres_block_summary_norm_backward(
            rows, d, _dtype_code(dtype), _ptr(gs), _ptr(gm), _ptr(out_sum), _ptr(inv_rms), _ptr(g),
            _stream_ptr(out_sum.device))
    N.check(rc, "attnres_block_summary_norm_backward")
    return g


@block_summary_norm_backward.register_fake
def _(grad_source, grad_sum, out_sum, inv_rms):
    return out_sum.new_empty(out_sum.shape)


def _block_summary_norm_setup(ctx, inputs, output):
    partial, _ = inputs
    out_sum, _, inv = output
    ctx.has_partial = partial is not None
    ctx.save_for_backward(out_sum, inv)


def _block_summary_norm_bwd(ctx, grad_sum, grad_source, grad_inv):
    out_sum, inv = ctx.saved_tensors
    if grad_source is None:
        g = grad_sum
    else:
        g = block_summary_norm_backward(grad_source, grad_sum, out_sum, inv)
    return (g if ctx.has_partial else None, g)


block_summary_norm.register_autograd(_block_summary_norm_bwd, setup_context=_block_summary_norm_setup)


def attention_residual_block_summary(partial_block: Optional[Tensor], layer_output: Tensor, count: int = 1,
                                     alpha=1.0, scale: Optional[Tensor] = None, value_norm: bool = False):
    """The running block sum and the scaled block source of block Attention
    Residuals in one pass: returns (partial_block + layer_output,
    (partial_block + layer_output) * c). c is the learned `scale` (cast to the
    value dtype, as model.py:978-983 does), else count ** -alpha with alpha a
    float or a tensor (model.py:955-959; a tensor alpha keeps its gradient).
    Replaces the add and the multiply of model.py:2377-2389 / :990-1001; the
    same call scales key sums (model.py:1011-1016). value_norm=True
    (attnres_block_value_norm) returns rms_norm(sum) as the source instead
    (model.py:991-992, :1004-1005)."""
    dtype = layer_output.dtype
    if value_norm:
        # attnres_block_value_norm: the source is rms_norm(sum) (model.py:991-992)
        out_sum, src, _ = block_summary_norm(partial_block, layer_output)
        return out_sum, src
    if scale is not None:
        return block_summary(partial_block, layer_output, scale.to(dtype), 1.0)
    if torch.is_tensor(alpha):
        c = torch.exp(-alpha * alpha.new_tensor(float(count)).log())
        return block_summary(partial_block, layer_output, c.to(dtype), 1.0)
    return block_summary(partial_block, layer_output, None, float(count) ** (-float(alpha)))


def lrid_block_source(partial_value: Optional[Tensor], value: Tensor, partial_key: Optional[Tensor],
                      key: Optional[Tensor], count: int = 1, alpha=1.0, scale: Optional[Tensor] = None,
                      value_norm: bool = False, key_norm: bool = True, key_from_value: bool = False):
    """One LRID block step: the running value and key sums (model.py:2377-2389)
    and the block source the read consumes (_lrid_block_source,
    model.py:1003-1018). Returns (value_sum, value_source, key_sum, key_source):
      * value_source = rms_norm(value_sum) with value_norm, else value_sum * c
        (c = the learned `scale`, else count ** -alpha);
      * key_source = key_sum * c only when neither the value norm, key_norm nor
        key_from_value is on (model.py:1015-1018), else key_sum.
    Key arguments may be None (key-from-value sources have no running key)."""
    value_sum, value_source = attention_residual_block_summary(partial_value, value, count, alpha, scale,
                                                               value_norm)
    if key is None:
        return value_sum, value_source, None, None
    if value_norm or key_norm or key_from_value:
        key_sum = key if partial_key is None else block_summary(partial_key, key, None, 1.0)[1]
        return value_sum, value_source, key_sum, key_sum
    key_sum, key_source = attention_residual_block_summary(partial_key, key, count, alpha, scale)
    return value_sum, value_source, key_sum, key_source


# ---------------------------------------------------------------------------
# attnres::phase2 — cached-logit phase 2 (merge of the live partial block)
# ---------------------------------------------------------------------------
PHASE2_LRID, PHASE2_BASE, PHASE2_LOGIT = 0, 1, 2


def _phase2_key_eps(mode, dtype):
    # LRID keys are normed as _norm(partial_key.float()) (attnres_ops.py:4127);
    # the base key as _norm(partial_value) in the value dtype (:2638)
    return _rms_eps()


@torch.library.custom_op("attnres::phase2", mutates_args=())
def phase2(mode: int, partial_value: Tensor, partial_key: Optional[Tensor], partial_logit: Optional[Tensor],
           query: Optional[Tensor], interblock_output: Tensor, interblock_lse: Tensor, logit_scale: float,
           key_norm: bool, logit_bias: Optional[Tensor], logit_bias_value: float,
           normalize_output: bool) -> tuple[Tensor, Tensor]:
    """Returns (output [*, d] value dtype, output inverse rms [N] fp32 or [1])."""
    _require_cuda([partial_value, partial_key, partial_logit, query, interblock_output, interblock_lse, logit_bias],
                  "phase-2 inputs")
    dtype = partial_value.dtype
    d = partial_value.size(-1)
    n = _ntok(partial_value)
    pv = partial_value.reshape(n, d).contiguous()
    io = interblock_output.to(dtype).reshape(n, d).contiguous()
    lse = interblock_lse.to(torch.float32).reshape(n).contiguous()
    pk = None if partial_key is None else partial_key.to(dtype).reshape(n, -1).contiguous()
    lg = None if partial_logit is None else partial_logit.to(torch.float32).reshape(n).contiguous()
    q = None if query is None else query.reshape(-1).to(dtype).contiguous()
    R = pk.size(1) if pk is not None else 0
    b = None if logit_bias is None else logit_bias.to(torch.float32).reshape(1).contiguous()
    out = torch.empty((n, d), device=pv.device, dtype=dtype)
    inv = torch.empty((n,) if normalize_output else (1,), device=pv.device, dtype=torch.float32)
    with torch.cuda.device(pv.device):
        rc = N.load().attnres_phase2_forward(
            int(mode), n, d, R, _dtype_code(dtype), _ptr(pv), _ptr(pk), _ptr(lg), _ptr(q), float(logit_scale),
            int(bool(key_norm)), _phase2_key_eps(mode, dtype), float(logit_bias_value), _ptr(b), _ptr(io), _ptr(lse),
            int(bool(normalize_output)), _rms_eps(), _ptr(out), _ptr(inv),
            _stream_ptr(pv.device))
    N.check(rc, "attnres_phase2_forward")
    return out.reshape(partial_value.shape), inv


@phase2.register_fake
def _(mode, partial_value, partial_key, partial_logit, query, interblock_output, interblock_lse, logit_scale,
      key_norm, logit_bias, logit_bias_value, normalize_output):
    n = partial_value.numel() // partial_value.size(-1)
    return partial_value.new_empty(partial_value.shape), partial_value.new_empty(
        (n,) if normalize_output else (1,), dtype=torch.float32)


@torch.library.custom_op("attnres::phase2_backward", mutates_args=())
def phase2_backward(mode: int, partial_value: Tensor, partial_key: Optional[Tensor], partial_logit: Optional[Tensor],
                    query: Optional[Tensor], interblock_output: Tensor, interblock_lse: Tensor, logit_scale: float,
                    key_norm: bool, logit_bias: Optional[Tensor], logit_bias_value: float, normalize_output: bool,
                    output: Tensor, output_inv_rms: Tensor, grad_output: Tensor, want_query_grad: bool,
                    want_bias_grad: bool) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Returns (d partial_value, d partial_key, d partial_logit, d interblock_output,
    d interblock_lse, d query, d bias); the unused ones are empty."""
    dtype = partial_value.dtype
    d = partial_value.size(-1)
    n = _ntok(partial_value)
    dev = partial_value.device
    pv = partial_value.reshape(n, d).contiguous()
    io = interblock_output.to(dtype).reshape(n, d).contiguous()
    lse = interblock_lse.to(torch.float32).reshape(n).contiguous()
    pk = None if partial_key is None else partial_key.to(dtype).reshape(n, -1).contiguous()
    lg = None if partial_logit is None else partial_logit.to(torch.float32).reshape(n).contiguous()
    q = None if query is None else query.reshape(-1).to(dtype).contiguous()
    R = pk.size(1) if pk is not None else 0
    b = None if logit_bias is None else logit_bias.to(torch.float32).reshape(1).contiguous()
    g = grad_output.to(dtype).reshape(n, d).contiguous()
    y = output.to(dtype).reshape(n, d).contiguous() if normalize_output else None
    yi = output_inv_rms.contiguous() if normalize_output else None
    e = lambda: torch.empty((0,), device=dev, dtype=torch.float32)  # noqa: E731  (distinct, non-aliased)
    dpv = torch.empty((n, d), device=dev, dtype=dtype)
    dio = torch.empty((n, d), device=dev, dtype=dtype)
    dlse = torch.empty((n,), device=dev, dtype=torch.float32)
    dpk = torch.empty((n, R), device=dev, dtype=dtype) if pk is not None else e()
    dlg = torch.empty((n,), device=dev, dtype=torch.float32) if lg is not None else e()
    qn = (R if mode == PHASE2_LRID else d)
    dq = torch.empty((qn,), device=dev, dtype=torch.float32) if (want_query_grad and q is not None) else e()
    db = torch.empty((1,), device=dev, dtype=torch.float32) if want_bias_grad else e()
    L = N.load()
    ws_bytes = L.attnres_phase2_backward_workspace_bytes(int(mode), n, d, R)
    ws = torch.empty((max(ws_bytes, 1),), device=dev, dtype=torch.uint8)
    with torch.cuda.device(dev):
        rc = L.attnres_phase2_backward(
            int(mode), n, d, R, _dtype_code(dtype), _ptr(pv), _ptr(pk), _ptr(lg), _ptr(q), float(logit_scale),
            int(bool(key_norm)), _phase2_key_eps(mode, dtype), float(logit_bias_value), _ptr(b), _ptr(io), _ptr(lse),
            int(bool(normalize_output)), _ptr(y), _ptr(yi), _ptr(g), _ptr(dpv),
            _ptr(dpk) if pk is not None else None, _ptr(dlg) if lg is not None else None, _ptr(dio), _ptr(dlse),
            _ptr(dq) if dq.numel() else None, _ptr(db) if want_bias_grad else None, _ptr(ws), ws_bytes,
            _stream_ptr(dev))
    N.check(rc, "attnres_phase2_backward")
    return dpv, dpk, dlg, dio, dlse, dq, db


@phase2_backward.register_fake
def _(mode, partial_value, partial_key, partial_logit, query, interblock_output, interblock_lse, logit_scale,
      key_norm, logit_bias, logit_bias_value, normalize_output, output, output_inv_rms, grad_output,
      want_query_grad, want_bias_grad):
    n = partial_value.numel() // partial_value.size(-1)
    d = partial_value.size(-1)
    f = partial_value.new_empty
    R = 0 if partial_key is None else partial_key.numel() // n
    return (f((n, d)), f((n, R)) if partial_key is not None else f((0,), dtype=torch.float32),
            f((n,), dtype=torch.float32) if partial_logit is not None else f((0,), dtype=torch.float32), f((n, d)),
            f((n,), dtype=torch.float32),
            f((R if mode == PHASE2_LRID else d,), dtype=torch.float32) if (want_query_grad and query is not None)
            else f((0,), dtype=torch.float32),
            f((1,), dtype=torch.float32) if want_bias_grad else f((0,), dtype=torch.float32))


def _phase2_setup(ctx, inputs, output):
    (mode, pv, pk, lg, q, io, lse, scale, key_norm, bias, bias_value, normalize_output) = inputs
    out, inv = output
    ctx.args = (int(mode), float(scale), bool(key_norm), float(bias_value), bool(normalize_output))
    ctx.has = (pk is not None, lg is not None, q is not None, bias is not None)
    ctx.meta = dict(pv=(pv.shape, pv.dtype), io=(io.shape, io.dtype), lse=(lse.shape, lse.dtype),
                    pk=None if pk is None else (pk.shape, pk.dtype), lg=None if lg is None else (lg.shape, lg.dtype),
                    q=None if q is None else (q.shape, q.dtype), b=None if bias is None else (bias.shape, bias.dtype))
    opt = [t for t in (pk, lg, q, bias) if t is not None]
    ctx.save_for_backward(pv, io, lse, out, inv, *opt)


def _phase2_bwd(ctx, grad_out, grad_inv):
    pv, io, lse, out, inv, *opt = ctx.saved_tensors
    it = iter(opt)
    pk, lg, q, bias = (next(it) if h else None for h in ctx.has)
    mode, scale, key_norm, bias_value, normalize_output = ctx.args
    want_q = q is not None and ctx.needs_input_grad[4]
    want_b = bias is not None and ctx.needs_input_grad[9]
    dpv, dpk, dlg, dio, dlse, dq, db = phase2_backward(mode, pv, pk, lg, q, io, lse, scale, key_norm, bias,
                                                       bias_value, normalize_output, out, inv, grad_out, want_q,
                                                       want_b)
    m = ctx.meta

    def cast(t, key):
        shape, dtype = m[key]
        return t.reshape(shape).to(dtype)

    return (None, cast(dpv, "pv"), cast(dpk, "pk") if pk is not None else None,
            cast(dlg, "lg") if lg is not None else None, cast(dq, "q") if want_q else None, cast(dio, "io"),
            cast(dlse, "lse"), None, None, cast(db, "b") if want_b else None, None, None)


phase2.register_autograd(_phase2_bwd, setup_context=_phase2_setup)


def _phase2_bias(logit_bias):
    """(tensor, value) for a logit bias given as None, a float or a tensor
    (attnres_ops.py:108-120)."""
    if logit_bias is None:
        return None, 0.0
    if isinstance(logit_bias, Tensor):
        return logit_bias, 0.0
    return None, float(logit_bias)


def lrid_attention_residual_phase2(partial_value: Tensor, partial_key: Tensor, query: Tensor,
                                   interblock_output: Tensor, interblock_lse: Tensor, logit_scale: float,
                                   key_norm: bool, force_triton: bool = False, normalize_output: bool = False,
                                   logit_bias=0.0) -> Tensor:
    """attnres_ops.py:4075-4139 on the B200 kernel: merge of the live partial
    block (LRID key, one query) into the phase-1 result."""
    bt, bv = _phase2_bias(logit_bias)
    out, _ = phase2(PHASE2_LRID, partial_value, partial_key, None, query, interblock_output, interblock_lse,
                    float(logit_scale), bool(key_norm), bt, bv, bool(normalize_output))
    return out


def attention_residual_phase2(partial_value: Tensor, query: Tensor, interblock_output: Tensor,
                              interblock_lse: Tensor, key_norm: bool, force_triton: bool = False,
                              normalize_output: bool = False, logit_bias=0.0) -> Tensor:
    """attnres_ops.py:3964-4019 on the B200 kernel: base key rms_norm(partial)."""
    bt, bv = _phase2_bias(logit_bias)
    out, _ = phase2(PHASE2_BASE, partial_value, None, None, query, interblock_output, interblock_lse, 1.0,
                    bool(key_norm), bt, bv, bool(normalize_output))
    return out


def attention_residual_phase2_from_logit(partial_value: Tensor, partial_logit: Tensor, interblock_output: Tensor,
                                         interblock_lse: Tensor, force_triton: bool = False,
                                         normalize_output: bool = False) -> Tensor:
    """attnres_ops.py:4043-4072 on the B200 kernel: the partial logit is given."""
    out, _ = phase2(PHASE2_LOGIT, partial_value, None, partial_logit, None, interblock_output, interblock_lse, 1.0,
                    False, None, 0.0, bool(normalize_output))
    return out


# ---------------------------------------------------------------------------
# attnres::lrid_fused_projection — LRIDFusedProjection.forward (model.py:363-388)
# ---------------------------------------------------------------------------
@torch.library.custom_op("attnres::lrid_fused_projection", mutates_args=())
def lrid_fused_projection(x: Tensor, weight: Tensor, output_dim: int, rank: int, num_heads: int, key_norm: bool,
                          query_rank: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """The projection x @ weight^T with weight [output_dim + rank + query_rank, in],
    returned as (output [*, output_dim] contiguous, key [*, rank] (per-head rms
    normalised when key_norm), query [*, query_rank] or empty, key inverse rms
    [N, num_heads] fp32 or empty). The output columns are a plain library GEMM
    straight into their own buffer (the reference's single GEMM is followed by a
    .contiguous() copy of them). The key/query columns, for 16-bit data, come
    from the tcgen05 projection kernel with the per-head key norm in its
    epilogue (attnres_lrid_fused_key_projection); for fp32 (no tensor-core
    path at fp32 accuracy) or shapes outside that kernel, from a second library
    GEMM and the per-head norm kernel reading the key columns in place."""
    _require_cuda([x, weight], "fused projection inputs")
    dt = x.dtype
    n = x.numel() // x.size(-1)
    x2 = x.reshape(n, x.size(-1))
    w = weight.to(dt)
    lead = x.shape[:-1]
    out = torch.matmul(x2, w[:output_dim].t())
    e = lambda: x.new_empty((0,), dtype=torch.float32)  # noqa: E731
    tc = _fused_key_projection_tc(x2, w, output_dim, rank, num_heads, key_norm, query_rank)
    if tc is not None:
        kq, key, inv = tc
        query = kq[:, rank:].contiguous() if query_rank else x.new_empty((0,))
        if not key_norm:
            key, inv = kq[:, :rank].contiguous(), e()
        return (out.reshape(*lead, output_dim), key.reshape(*lead, rank),
                query.reshape(*lead, query_rank) if query_rank else query, inv)
    kq = torch.matmul(x2, w[output_dim:output_dim + rank + query_rank].t())  # [n, rank + query_rank]
    if key_norm:
        key = torch.empty((n, rank), device=x.device, dtype=dt)
        inv = torch.empty((n, num_heads), device=x.device, dtype=torch.float32)
        with torch.cuda.device(x.device):
            rc = N.load().attnres_head_rms_norm_forward(n, rank, num_heads, _dtype_code(dt), _ptr(kq), kq.stride(0),
                                                         _rms_eps(), _ptr(key), _ptr(inv),
                                                         _stream_ptr(x.device))
        N.check(rc, "attnres_head_rms_norm_forward")
    else:
        key = kq[:, :rank].contiguous()
        inv = e()
    query = kq[:, rank:].contiguous() if query_rank else x.new_empty((0,))
    return (out.reshape(*lead, output_dim), key.reshape(*lead, rank),
            query.reshape(*lead, query_rank) if query_rank else query, inv)


def _fused_key_projection_tc(x2, w, output_dim, rank, num_heads, key_norm, query_rank, normed=True):
    """(kq [n, rank + query_rank] pre-norm, key [n, rank] normed or None, inv
    [n, H] or None) from the tcgen05 projection kernel, or None for fp32 and
    for shapes outside it (ATTNRES_ERR_UNSUPPORTED, nothing launched)."""
    if x2.dtype not in (torch.float16, torch.bfloat16) or x2.stride(-1) != 1:
        return None
    n = x2.size(0)
    wk = w[output_dim:output_dim + rank + query_rank]
    if wk.stride(-1) != 1:
        return None
    norm = bool(key_norm) and normed
    kq = torch.empty((n, rank + query_rank), device=x2.device, dtype=x2.dtype)
    key = torch.empty((n, rank), device=x2.device, dtype=x2.dtype) if norm else None
    inv = torch.empty((n, num_heads), device=x2.device, dtype=torch.float32) if norm else None
    with torch.cuda.device(x2.device):
        rc = N.load().attnres_lrid_fused_key_projection(
            n, x2.size(1), rank, query_rank, num_heads, _dtype_code(x2.dtype), _ptr(x2), x2.stride(0), _ptr(wk),
            wk.stride(0), int(norm), _rms_eps(), _ptr(kq), _ptr(key), _ptr(inv), _stream_ptr(x2.device))
    if rc == 2:  # ATTNRES_ERR_UNSUPPORTED
        return None
    N.check(rc, "attnres_lrid_fused_key_projection")
    return kq, key, inv


@lrid_fused_projection.register_fake
def _(x, weight, output_dim, rank, num_heads, key_norm, query_rank):
    lead = x.shape[:-1]
    n = x.numel() // x.size(-1)
    return (x.new_empty((*lead, output_dim)), x.new_empty((*lead, rank)),
            x.new_empty((*lead, query_rank)) if query_rank else x.new_empty((0,)),
            x.new_empty((n, num_heads) if key_norm else (0,), dtype=torch.float32))


@torch.library.custom_op("attnres::lrid_fused_projection_backward", mutates_args=())
def lrid_fused_projection_backward(x: Tensor, weight: Tensor, key: Tensor, key_inv: Tensor,
                                   grad_output: Optional[Tensor], grad_key: Optional[Tensor],
                                   grad_query: Optional[Tensor], output_dim: int, rank: int, num_heads: int,
                                   key_norm: bool, query_rank: int) -> tuple[Tensor, Tensor]:
    """(d x, d weight [output_dim + rank + query_rank, in] in weight's dtype)."""
    dt = x.dtype
    n = x.numel() // x.size(-1)
    x2 = x.reshape(n, x.size(-1))
    w = weight.to(dt)
    kq_rows = slice(output_dim, output_dim + rank + query_rank)
    dw = torch.zeros_like(weight)
    dx = None
    # the gradient of each column block goes through its own GEMMs, accumulated
    # in place (no [n, output + rank] gradient buffer)
    blocks = []
    if grad_output is not None:
        blocks.append((slice(0, output_dim), grad_output.to(dt).reshape(n, output_dim)))
    if grad_key is not None:
        gk = grad_key.to(dt).reshape(n, rank).contiguous()
        if key_norm:
            # the pre-norm key columns, recomputed with the forward's own
            # projection (the tcgen05 kernel, or the [n, rank + query_rank]
            # library GEMM: bitwise the values the saved inverse rms belongs
            # to), so the norm backward works from them in fp32
            tc = _fused_key_projection_tc(x2, w, output_dim, rank, num_heads, key_norm, query_rank, normed=False)
            kraw = tc[0] if tc is not None else torch.matmul(x2, w[kq_rows].t())
            gkn = torch.empty((n, rank), device=x.device, dtype=dt)
            with torch.cuda.device(x.device):
                rc = N.load().attnres_head_rms_norm_backward(n, rank, num_heads, _dtype_code(dt), _ptr(gk),
                                                             _ptr(kraw), kraw.stride(0), _ptr(key_inv), _ptr(gkn),
                                                             rank, _stream_ptr(x.device))
            N.check(rc, "attnres_head_rms_norm_backward")
            gk = gkn
        blocks.append((slice(output_dim, output_dim + rank), gk))
    if grad_query is not None and query_rank:
        blocks.append((slice(output_dim + rank, output_dim + rank + query_rank),
                       grad_query.to(dt).reshape(n, query_rank)))
    for rows, g in blocks:
        dx = torch.matmul(g, w[rows]) if dx is None else torch.addmm(dx, g, w[rows])
        dw[rows] = torch.matmul(g.t(), x2).to(weight.dtype)
    if dx is None:
        dx = torch.zeros_like(x2)
    return dx.reshape(x.shape), dw


@lrid_fused_projection_backward.register_fake
def _(x, weight, key, key_inv, grad_output, grad_key, grad_query, output_dim, rank, num_heads, key_norm, query_rank):
    return x.new_empty(x.shape), weight.new_empty(weight.shape)


def _lfp_setup(ctx, inputs, output):
    x, weight, output_dim, rank, num_heads, key_norm, query_rank = inputs
    out, key, query, inv = output
    ctx.args = (int(output_dim), int(rank), int(num_heads), bool(key_norm), int(query_rank))
    ctx.save_for_backward(x, weight, key, inv)


def _lfp_bwd(ctx, g_out, g_key, g_query, g_inv):
    x, weight, key, inv = ctx.saved_tensors
    output_dim, rank, num_heads, key_norm, query_rank = ctx.args
    dx, dw = lrid_fused_projection_backward(x, weight, key, inv, g_out, g_key, g_query if query_rank else None,
                                            output_dim, rank, num_heads, key_norm, query_rank)
    return dx, dw, None, None, None, None, None


lrid_fused_projection.register_autograd(_lfp_bwd, setup_context=_lfp_setup)


def lrid_fused_projection_forward(x: Tensor, weight: Tensor, output_dim: int, rank: int, num_heads: int,
                                  key_norm: bool, query_rank: int = 0):
    """LRIDFusedProjection.forward (model.py:363-388) for the fused-key layout
    (use_key, optionally use_fused_query): returns (output, key) or
    (output, key, query) like the reference module."""
    out, key, query, _ = lrid_fused_projection(x, weight, int(output_dim), int(rank), int(num_heads),
                                               bool(key_norm), int(query_rank))
    return (out, key, query) if query_rank else (out, key)
