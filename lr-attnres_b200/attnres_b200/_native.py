"""ctypes binding of libattnres_b200.so (declared in include/attnres_b200.h).

The library is built in-tree by lr-attnres_b200/build.py. Loading fails loudly
when it is missing: there is no CPU or Python fallback for the fused read.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libattnres_b200.so")

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
QUERY_STATIC, QUERY_DYNAMIC, QUERY_GATED = 0, 1, 2
NORM_NONE, NORM_PER_HEAD, NORM_ROW = 0, 1, 2
MAX_SOURCES = 64

STATUS_NAMES = {
    0: "ok",
    1: "invalid argument",
    2: "unsupported",
    3: "CUDA error",
    4: "workspace too small",
}

EXPORTED_SYMBOLS = (
    "attnres_abi_version",
    "attnres_last_error",
    "attnres_device_status",
    "attnres_lrid_forward",
    "attnres_lrid_backward_workspace_bytes",
    "attnres_lrid_backward",
    "attnres_base_forward",
    "attnres_base_backward_workspace_bytes",
    "attnres_base_backward",
    "attnres_lrid_backward_noalloc",
    "attnres_lrid_key_projection",
    "attnres_lrid_key_projection_backward",
    "attnres_lrid_key_from_value_forward",
    "attnres_lrid_key_projection_backward_tc_workspace_bytes",
    "attnres_lrid_key_projection_backward_tc",
    "attnres_lrid_key_from_value_backward_workspace_bytes",
    "attnres_lrid_key_from_value_backward",
    "attnres_block_summary_forward",
    "attnres_block_summary_backward_workspace_bytes",
    "attnres_block_summary_backward",
    "attnres_block_summary_norm_forward",
    "attnres_block_summary_norm_backward",
    "attnres_head_rms_norm_forward",
    "attnres_head_rms_norm_backward",
    "attnres_lrid_fused_key_projection",
    "attnres_phase2_forward",
    "attnres_phase2_backward_workspace_bytes",
    "attnres_phase2_backward",
    "attnres_phase1_forward",
    "attnres_phase1_backward",
    "attnres_noalloc_scratch_bytes",
)

_lib = None


class AttnResError(RuntimeError):
    """Raised when a libattnres_b200 call returns a non-zero status."""


def load(path=None):
    """Load the shared library (once) and declare every entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise AttnResError(
            f"libattnres_b200.so not found at {path}; build it with "
            "`python lr-attnres_b200/build.py` (nvcc, sm_100a)"
        )
    L = ctypes.CDLL(path)
    P, I, I64, F, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
    PP = ctypes.POINTER(ctypes.c_void_p)
    PI64 = ctypes.POINTER(ctypes.c_int64)
    L.attnres_abi_version.restype = I
    L.attnres_abi_version.argtypes = []
    L.attnres_last_error.restype = ctypes.c_char_p
    L.attnres_last_error.argtypes = []
    L.attnres_device_status.restype = I
    L.attnres_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint), I]
    L.attnres_lrid_forward.restype = I
    L.attnres_lrid_forward.argtypes = [
        I, I64, I, I, I, I,          # S, N, d, R, H, dtype
        PP, PI64, PP, PI64,          # values, strides, keys, strides
        I, P, P, P,                  # query mode, query, gate, query_dynamic
        F, I, F, P,                  # scale, key_norm, key_eps, logit_bias
        I, F,                        # output_norm, output_eps
        P, P, P, P,                  # output, output_inv_rms, alpha, key_inv_rms
        P,                           # stream
    ]
    L.attnres_lrid_backward_workspace_bytes.restype = SZ
    L.attnres_lrid_backward_workspace_bytes.argtypes = [I, I64, I, I, I, I]
    L.attnres_lrid_backward.restype = I
    L.attnres_lrid_backward.argtypes = [
        I, I64, I, I, I, I,
        PP, PI64, PP, PI64,
        I, P, P, P,
        F, I, F, P,
        I, F,
        P, P, P,                     # grad_output, normed_output, output_inv_rms
        PP, PP,                      # grad_values, grad_keys
        P, P, P, P,                  # grad_query, grad_gate, grad_query_dynamic, grad_bias
        P, SZ,                       # workspace, bytes
        P,                           # stream
    ]
    L.attnres_lrid_backward_noalloc.restype = I
    L.attnres_lrid_backward_noalloc.argtypes = L.attnres_lrid_backward.argtypes[:-3] + [P]
    L.attnres_noalloc_scratch_bytes.restype = SZ
    L.attnres_noalloc_scratch_bytes.argtypes = []
    L.attnres_lrid_key_projection.restype = I
    L.attnres_lrid_key_projection.argtypes = [I, I64, I, I, I, PP, PI64, P, I64, I, F, P, P, P]
    L.attnres_lrid_key_projection_backward.restype = I
    L.attnres_lrid_key_projection_backward.argtypes = [I, I64, I, I, I, I, PP, PI64, PP, P, P, P, P, P, P, I, P]
    L.attnres_lrid_key_from_value_forward.restype = I
    L.attnres_lrid_key_from_value_forward.argtypes = [
        I, I64, I, I, I, I,          # S, N, d, R, H, dtype
        PP, PI64, P, I64,            # values, strides, weight, weight row stride
        I, F, P, F, I, F, P,         # value_norm, value_eps, query, scale, key_norm, key_eps, logit_bias
        P, P, P, P, P,               # output, keys, value_inv_rms, alpha, stream
    ]
    L.attnres_lrid_key_projection_backward_tc_workspace_bytes.restype = SZ
    L.attnres_lrid_key_projection_backward_tc_workspace_bytes.argtypes = [I, I64, I, I, I, I]
    L.attnres_lrid_key_projection_backward_tc.restype = I
    L.attnres_lrid_key_projection_backward_tc.argtypes = [
        I, I64, I, I, I, I,          # S, N, d, R, H, dtype
        PP, PI64, P, I64,            # values, strides, weight, weight row stride
        PP, P, P, P, P, I,           # grad_keys, keys, inv_rms, grad_output, alpha, value_norm
        PP, P, P, SZ,                # grad_values, grad_weight, workspace, workspace bytes
        P,                           # stream
    ]
    L.attnres_lrid_key_from_value_backward_workspace_bytes.restype = SZ
    L.attnres_lrid_key_from_value_backward_workspace_bytes.argtypes = [I, I64, I, I, I, I]
    L.attnres_lrid_key_from_value_backward.restype = I
    L.attnres_lrid_key_from_value_backward.argtypes = [
        I, I64, I, I, I, I,          # S, N, d, R, H, dtype
        PP, PI64, P, I64,            # values, strides, weight, weight row stride
        P, I, P, P, P,               # keys, value_norm, value_inv_rms, alpha, query
        F, I, F, P, P,               # scale, key_norm, key_eps, grad_output, output
        PP, P, P, P,                 # grad_values, grad_weight, grad_query, grad_logit_bias
        P, SZ, P,                    # workspace, workspace bytes, stream
    ]
    L.attnres_block_summary_forward.restype = I
    L.attnres_block_summary_forward.argtypes = [I64, I, P, P, P, F, P, P, P]
    L.attnres_block_summary_backward_workspace_bytes.restype = SZ
    L.attnres_block_summary_backward_workspace_bytes.argtypes = [I64]
    L.attnres_block_summary_backward.restype = I
    L.attnres_block_summary_backward.argtypes = [I64, I, P, P, P, P, F, P, P, P, SZ, P]
    L.attnres_block_summary_norm_forward.restype = I
    L.attnres_block_summary_norm_forward.argtypes = [I64, I, I, P, P, F, P, P, P, P]
    L.attnres_block_summary_norm_backward.restype = I
    L.attnres_block_summary_norm_backward.argtypes = [I64, I, I, P, P, P, P, P, P]
    L.attnres_head_rms_norm_forward.restype = I
    L.attnres_head_rms_norm_forward.argtypes = [I64, I, I, I, P, I64, F, P, P, P]
    L.attnres_lrid_fused_key_projection.restype = I
    L.attnres_lrid_fused_key_projection.argtypes = [I64, I, I, I, I, I, P, I64, P, I64, I, F, P, P, P, P]
    L.attnres_head_rms_norm_backward.restype = I
    L.attnres_head_rms_norm_backward.argtypes = [I64, I, I, I, P, P, I64, P, P, I64, P]
    L.attnres_phase2_forward.restype = I
    L.attnres_phase2_forward.argtypes = [
        I, I64, I, I, I,             # mode, N, value_dim, key_dim, dtype
        P, P, P, P,                  # partial value, partial key, partial logit, query
        F, I, F, F, P,               # logit scale, key norm, key eps, bias, bias (device)
        P, P, I, F, P, P, P,         # interblock output, lse, normalize, output eps, output, inv, stream
    ]
    L.attnres_phase2_backward_workspace_bytes.restype = SZ
    L.attnres_phase2_backward_workspace_bytes.argtypes = [I, I64, I, I]
    L.attnres_phase2_backward.restype = I
    L.attnres_phase2_backward.argtypes = [
        I, I64, I, I, I,             # mode, N, value_dim, key_dim, dtype
        P, P, P, P,                  # partial value, partial key, partial logit, query
        F, I, F, F, P,               # logit scale, key norm, key eps, bias, bias (device)
        P, P, I, P, P, P,            # interblock output, lse, normalize, output, output inv, grad output
        P, P, P, P, P, P, P,         # grads: partial value, key, logit, interblock output, lse, query, bias
        P, SZ, P,                    # workspace, bytes, stream
    ]
    L.attnres_phase1_forward.restype = I
    L.attnres_phase1_forward.argtypes = [I, I, I64, I, I, PP, PI64, P, I, I, F, P, P, P, P]
    L.attnres_phase1_backward.restype = I
    L.attnres_phase1_backward.argtypes = [I, I, I64, I, I, PP, PI64, P, I, I, F, P, P, P, P, PP, P, P]
    L.attnres_base_forward.restype = I
    L.attnres_base_forward.argtypes = [
        I, I64, I, I, PP, PI64, P, I, F, P, I, F, P, P, P,
    ]
    L.attnres_base_backward_workspace_bytes.restype = SZ
    L.attnres_base_backward_workspace_bytes.argtypes = [I, I64, I, I]
    L.attnres_base_backward.restype = I
    L.attnres_base_backward.argtypes = [
        I, I64, I, I, PP, PI64, P, I, F, P, I, F, P, P, P, PP, P, P, P, SZ, P,
    ]
    if path == LIB_PATH:
        _lib = L
    return L


def check(status, what):
    if status != 0:
        msg = load().attnres_last_error().decode(errors="replace")
        raise AttnResError(f"{what} failed ({STATUS_NAMES.get(status, status)}): {msg}")


def device_status(reset=False):
    """Bits set by a bulk-copy kernel that abandoned a bounded wait (0 = healthy)."""
    st = ctypes.c_uint(0)
    check(load().attnres_device_status(ctypes.byref(st), int(bool(reset))), "attnres_device_status")
    return st.value


def ptr_array(ptrs):
    arr = (ctypes.c_void_p * max(1, len(ptrs)))()
    for i, p in enumerate(ptrs):
        arr[i] = p
    return arr


def i64_array(vals):
    arr = (ctypes.c_int64 * max(1, len(vals)))()
    for i, v in enumerate(vals):
        arr[i] = int(v)
    return arr
