"""TEST INFRASTRUCTURE ONLY — ctypes wrapper of the C oracle (attnres_oracle.c).

The oracle restates the reference's unfused PyTorch semantics of the block
Attention-Residual read in double precision (see the citations in
attnres_oracle.c). Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline / reference arm use it, always as the checker or the timed CPU
baseline, never as part of the product path.

Arrays are numpy; sources are passed stacked and dense: values [S, N, d],
keys [S, N, R]; query [H, dk] (static / gated), query_dynamic [N, H, dk].
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libattnres_oracle.so")

Q_STATIC, Q_DYNAMIC, Q_GATED = 0, 1, 2
NORM_NONE, NORM_PER_HEAD, NORM_ROW = 0, 1, 2

_lib = None


def build(force=False):
    src = os.path.join(HERE, "attnres_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(src) > os.path.getmtime(LIB_PATH):
        subprocess.run(["make", "-s", "-C", HERE, "-B" if force else "-s"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.c_void_p
        I, LL, D = ctypes.c_int, ctypes.c_longlong, ctypes.c_double
        L.oracle_lrid_forward.argtypes = [I, LL, I, I, I, P, P, I, P, P, P, D, I, D, P, I, D, P, P, P, P]
        L.oracle_lrid_backward.argtypes = [I, LL, I, I, I, P, P, I, P, P, P, D, I, D, P, I, D, P, P, P, P, P, P, P]
        L.oracle_base_forward.argtypes = [I, LL, I, P, P, I, D, P, I, D, P, P]
        L.oracle_base_backward.argtypes = [I, LL, I, P, P, I, D, P, I, D, P, P, P, P]
        L.oracle_num_threads.restype = I
        L.oracle_set_num_threads.argtypes = [I]
        _lib = L
    return _lib


def set_num_threads(n):
    lib().oracle_set_num_threads(int(n))


def num_threads():
    return lib().oracle_num_threads()


def _f32(x):
    if x is None:
        return None
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _p(x):
    return None if x is None else x.ctypes.data_as(ctypes.c_void_p)


def _query_args(query, gate, query_dynamic):
    if query_dynamic is None:
        return Q_STATIC, _f32(query), None, None
    if query is None:
        return Q_DYNAMIC, None, None, _f32(query_dynamic)
    return Q_GATED, _f32(query), _f32(gate), _f32(query_dynamic)


def lrid_forward(values, keys, num_heads, logit_scale, key_norm, query=None, gate=None,
                 query_dynamic=None, logit_bias=None, output_norm=NORM_NONE,
                 key_eps=float(np.finfo(np.float32).eps), output_eps=float(np.finfo(np.float32).eps)):
    """Returns (out [N,d], out_inv, alpha [N,H,S], key_inv_rms [N,H,S]) in float64."""
    values, keys = _f32(values), _f32(keys)
    S, N, d = values.shape
    R = keys.shape[2]
    H = int(num_heads)
    qmode, q, g, qd = _query_args(query, gate, query_dynamic)
    bias = _f32(logit_bias)
    out = np.zeros((N, d), np.float64)
    inv = np.zeros((N, H) if output_norm == NORM_PER_HEAD else (N,), np.float64)
    alpha = np.zeros((N, H, S), np.float64)
    kinv = np.zeros((N, H, S), np.float64)
    lib().oracle_lrid_forward(S, N, d, R, H, _p(values), _p(keys), qmode, _p(q), _p(g), _p(qd),
                              float(logit_scale), int(bool(key_norm)), float(key_eps), _p(bias),
                              int(output_norm), float(output_eps), _p(out), _p(inv), _p(alpha), _p(kinv))
    return out, inv, alpha, kinv


def lrid_backward(values, keys, num_heads, logit_scale, key_norm, grad_output, query=None, gate=None,
                  query_dynamic=None, logit_bias=None, output_norm=NORM_NONE,
                  key_eps=float(np.finfo(np.float32).eps), output_eps=float(np.finfo(np.float32).eps)):
    """Returns dict with dV [S,N,d], dK [S,N,R], dq, and dgate/dq_dynamic/dbias when relevant."""
    values, keys, grad_output = _f32(values), _f32(keys), _f32(grad_output)
    S, N, d = values.shape
    R = keys.shape[2]
    H = int(num_heads)
    qmode, q, g, qd = _query_args(query, gate, query_dynamic)
    bias = _f32(logit_bias)
    dV = np.zeros((S, N, d), np.float64)
    dK = np.zeros((S, N, R), np.float64)
    dq = np.zeros((N, R) if qmode == Q_DYNAMIC else (R,), np.float64)
    dgate = np.zeros((H,), np.float64) if qmode == Q_GATED else None
    dqdyn = np.zeros((N, R), np.float64) if qmode == Q_GATED else None
    dbias = np.zeros((S,), np.float64) if bias is not None else None
    lib().oracle_lrid_backward(S, N, d, R, H, _p(values), _p(keys), qmode, _p(q), _p(g), _p(qd),
                               float(logit_scale), int(bool(key_norm)), float(key_eps), _p(bias),
                               int(output_norm), float(output_eps), _p(grad_output), _p(dV), _p(dK),
                               _p(dq), _p(dgate), _p(dqdyn), _p(dbias))
    res = {"dV": dV, "dK": dK, "dq": dq}
    if qmode == Q_GATED:
        res["dgate"] = dgate
        res["dq_dynamic"] = dqdyn
    if bias is not None:
        res["dbias"] = dbias
    return res


def base_forward(values, query, key_norm, logit_bias=None, output_norm=NORM_NONE,
                 key_eps=float(np.finfo(np.float32).eps), output_eps=float(np.finfo(np.float32).eps)):
    values, q, bias = _f32(values), _f32(query), _f32(logit_bias)
    S, N, d = values.shape
    out = np.zeros((N, d), np.float64)
    inv = np.zeros((N,), np.float64)
    lib().oracle_base_forward(S, N, d, _p(values), _p(q), int(bool(key_norm)), float(key_eps), _p(bias),
                              int(output_norm), float(output_eps), _p(out), _p(inv))
    return out, inv


def base_backward(values, query, key_norm, grad_output, logit_bias=None, output_norm=NORM_NONE,
                  key_eps=float(np.finfo(np.float32).eps), output_eps=float(np.finfo(np.float32).eps)):
    values, q, bias, g = _f32(values), _f32(query), _f32(logit_bias), _f32(grad_output)
    S, N, d = values.shape
    dV = np.zeros((S, N, d), np.float64)
    dq = np.zeros((d,), np.float64)
    dbias = np.zeros((S,), np.float64) if bias is not None else None
    lib().oracle_base_backward(S, N, d, _p(values), _p(q), int(bool(key_norm)), float(key_eps), _p(bias),
                               int(output_norm), float(output_eps), _p(g), _p(dV), _p(dq), _p(dbias))
    res = {"dV": dV, "dq": dq}
    if bias is not None:
        res["dbias"] = dbias
    return res


def _kv_keys(values, weight, value_norm, value_eps):
    """Key-from-value projection, double precision: keys_s = rms_norm(V_s) @ W^T
    (reference model.py:344-356; norm = F.rms_norm over the last dim)."""
    v = np.asarray(values, np.float64)
    w = np.asarray(weight, np.float64)
    inv = 1.0 / np.sqrt((v * v).mean(-1, keepdims=True) + value_eps) if value_norm else np.ones(v.shape[:-1] + (1,))
    nhat = v * inv
    return nhat @ w.T, inv, nhat


def lrid_kv_forward(values, weight, num_heads, logit_scale, key_norm, value_norm=True,
                    value_eps=float(np.finfo(np.float32).eps), **kw):
    keys, _, _ = _kv_keys(values, weight, value_norm, value_eps)
    return lrid_forward(values, keys.astype(np.float32), num_heads, logit_scale, key_norm, **kw)[0], keys


def lrid_kv_backward(values, weight, num_heads, logit_scale, key_norm, grad_output, value_norm=True,
                     value_eps=float(np.finfo(np.float32).eps), **kw):
    """Read backward plus the projection backward:
    dV += inv * (dK W - nhat * <dK, key>/d), dW = sum_s dK_s^T nhat_s."""
    keys, inv, nhat = _kv_keys(values, weight, value_norm, value_eps)
    res = lrid_backward(values, keys.astype(np.float32), num_heads, logit_scale, key_norm, grad_output, **kw)
    dk = res["dK"]
    w = np.asarray(weight, np.float64)
    d = nhat.shape[-1]
    dn = dk @ w
    if value_norm:
        c = (dk * keys).sum(-1, keepdims=True) / d
        res["dV"] = res["dV"] + inv * (dn - nhat * c)
    else:
        res["dV"] = res["dV"] + dn
    res["dW"] = np.einsum("snr,snd->rd", dk, nhat)
    res["keys"] = keys
    return res


def phase1_forward(values, logits, normalize_output=False, output_eps=float(np.finfo(np.float32).eps)):
    """Cached-logit read, double precision (attnres_ops.py:3955-3961):
    values [S, N, d], logits [Q, S, N] -> out [Q, N, d], lse [Q, N]."""
    v = np.asarray(values, np.float64)
    lg = np.asarray(logits, np.float64)
    m = lg.max(axis=1, keepdims=True)
    e = np.exp(lg - m)
    alpha = e / e.sum(axis=1, keepdims=True)  # [Q, S, N]
    acc = np.einsum("qsn,snd->qnd", alpha, v)
    lse = (m[:, 0] + np.log(e.sum(axis=1)))
    inv = None
    if normalize_output:
        inv = 1.0 / np.sqrt((acc * acc).mean(-1, keepdims=True) + output_eps)
        out = acc * inv
    else:
        out = acc
    return out, lse, alpha, acc, inv


def phase1_backward(values, logits, grad_output, grad_lse=None, normalize_output=False,
                    output_eps=float(np.finfo(np.float32).eps)):
    """Analytic gradients of phase1_forward (as the reference's backward
    kernels compute them, attnres_ops.py:1069-1140)."""
    v = np.asarray(values, np.float64)
    out, lse, alpha, acc, inv = phase1_forward(values, logits, normalize_output, output_eps)
    g = np.asarray(grad_output, np.float64)
    if normalize_output:
        y = acc * inv
        g = inv * (g - y * (g * y).mean(-1, keepdims=True))
    dV = np.einsum("qsn,qnd->snd", alpha, g)
    dw = np.einsum("qnd,snd->qsn", g, v)
    dl = alpha * (dw - (alpha * dw).sum(axis=1, keepdims=True))
    if grad_lse is not None:
        dl = dl + np.asarray(grad_lse, np.float64)[:, None, :] * alpha
    return {"dV": dV, "dlogits": dl}


PHASE2_LRID, PHASE2_BASE, PHASE2_LOGIT = 0, 1, 2


def phase2_forward(mode, partial_value, interblock_output, interblock_lse, partial_key=None, query=None,
                   partial_logit=None, logit_scale=1.0, key_norm=False, key_eps=float(np.finfo(np.float32).eps),
                   logit_bias=0.0, normalize_output=False, output_eps=float(np.finfo(np.float32).eps)):
    """Cached-logit phase 2, double precision: the live partial block merged into
    the phase-1 result (attnres_ops.py:4142-4160 for LRID keys, :2630-2642 for
    the base key rms_norm(partial_value), :4043-4072 given the logit):
      logit = scale <k_hat, q> + bias (or the given logit), p = sigmoid(logit - lse)
      merged = prev + p (v - prev),   out = merged (* rms inv when normalized).
    partial_value / interblock_output [N, d], interblock_lse [N], partial_key
    [N, R], query [R] (LRID) or [d] (base), partial_logit [N]."""
    v = np.asarray(partial_value, np.float64)
    prev = np.asarray(interblock_output, np.float64)
    lse = np.asarray(interblock_lse, np.float64)
    kinv = None
    khat = None
    if mode == PHASE2_LOGIT:
        logit = np.asarray(partial_logit, np.float64).copy()
    else:
        k = np.asarray(partial_key if mode == PHASE2_LRID else partial_value, np.float64)
        q = np.asarray(query, np.float64).reshape(-1)
        kinv = 1.0 / np.sqrt((k * k).mean(-1) + key_eps) if key_norm else np.ones(k.shape[0])
        khat = k * kinv[:, None]
        logit = (khat @ q) * (logit_scale if mode == PHASE2_LRID else 1.0)
    logit = logit + float(logit_bias)
    p = 1.0 / (1.0 + np.exp(-(logit - lse)))
    merged = prev + p[:, None] * (v - prev)
    inv = None
    out = merged
    if normalize_output:
        inv = 1.0 / np.sqrt((merged * merged).mean(-1) + output_eps)
        out = merged * inv[:, None]
    return out, {"p": p, "merged": merged, "inv": inv, "kinv": kinv, "khat": khat}


def phase2_backward(mode, partial_value, interblock_output, interblock_lse, grad_output, partial_key=None,
                    query=None, partial_logit=None, logit_scale=1.0, key_norm=False,
                    key_eps=float(np.finfo(np.float32).eps), logit_bias=0.0, normalize_output=False,
                    output_eps=float(np.finfo(np.float32).eps), saved_output=None):
    """Analytic gradients of phase2_forward (the reference's backward kernel
    attnres_ops.py:2058-2121 and the autograd of its PyTorch path). With
    normalize_output the output-norm backward uses `saved_output` when given:
    the reference's backward kernel loads the saved, value-dtype output
    (attnres_ops.py:2090-2093)."""
    v = np.asarray(partial_value, np.float64)
    prev = np.asarray(interblock_output, np.float64)
    out, st = phase2_forward(mode, partial_value, interblock_output, interblock_lse, partial_key, query,
                             partial_logit, logit_scale, key_norm, key_eps, logit_bias, normalize_output,
                             output_eps)
    g = np.asarray(grad_output, np.float64)
    if normalize_output:
        y = out if saved_output is None else np.asarray(saved_output, np.float64)
        g = st["inv"][:, None] * (g - y * (g * y).mean(-1, keepdims=True))
    p = st["p"]
    dl = p * (1.0 - p) * (g * (v - prev)).sum(-1)
    res = {"d_partial_value": p[:, None] * g, "d_interblock_output": (1.0 - p)[:, None] * g,
           "d_interblock_lse": -dl, "dbias": dl.sum()}
    if mode == PHASE2_LOGIT:
        res["d_partial_logit"] = dl
        return res
    q = np.asarray(query, np.float64).reshape(-1)
    sc = logit_scale if mode == PHASE2_LRID else 1.0
    khat, kinv = st["khat"], st["kinv"]
    dkhat = (dl * sc)[:, None] * q[None, :]
    if key_norm:
        dk = kinv[:, None] * (dkhat - khat * (dkhat * khat).mean(-1, keepdims=True))
    else:
        dk = dkhat
    res["dq"] = ((dl * sc)[:, None] * khat).sum(0)
    if mode == PHASE2_LRID:
        res["d_partial_key"] = dk
    else:
        res["d_partial_value"] = res["d_partial_value"] + dk
    return res
