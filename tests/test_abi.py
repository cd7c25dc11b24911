"""CPU-side checks of the C ABI: the shared library loads without a GPU, exports
every entry point that include/*.h declares, and rejects bad arguments with
the documented status codes before touching the device."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

from attnres_b200 import _native as N

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for hdr in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(hdr).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"^\s*(?:const\s+)?\w[\w\s\*]*?\b(attnres_\w+)\s*\(", text, flags=re.M))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("attnres_lrid_forward", "attnres_lrid_backward", "attnres_base_forward",
                     "attnres_base_backward", "attnres_last_error", "attnres_device_status"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = N.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    nm = subprocess.run(["nm", "-D", "--defined-only", N.LIB_PATH], capture_output=True, text=True).stdout
    for name in declared_symbols():
        assert re.search(rf"\bT {name}\b", nm), name


def test_python_binding_covers_the_header():
    assert set(N.EXPORTED_SYMBOLS) | {"attnres_device_status"} >= set(declared_symbols())


def test_abi_version():
    assert N.load().attnres_abi_version() == 1


def _fwd(S=2, n=4, d=8, R=4, H=1, dtype=N.DTYPE_F32, qmode=N.QUERY_STATIC, q=1, norm=N.NORM_NONE,
         values=True, keys=True, strides=None, out=1):
    L = N.load()
    vals = N.ptr_array([16] * S) if values else None
    ks = N.ptr_array([16] * S) if keys else None
    vstr = N.i64_array(strides or [d] * S)
    kstr = N.i64_array([R] * S)
    return L.attnres_lrid_forward(S, n, d, R, H, dtype, vals, vstr, ks, kstr, qmode,
                                  q, None, None, 1.0, 1, 1e-6, None, norm, 1e-6, out, None, None,
                                  None, None)


@pytest.mark.parametrize("kwargs,code,msg", [
    (dict(S=0), 2, "num_sources"),
    (dict(S=65), 2, "num_sources"),
    (dict(n=-1), 1, "negative"),
    (dict(d=10, H=3), 1, "divide"),
    (dict(dtype=7), 1, "dtype"),
    (dict(qmode=9), 1, "query_mode"),
    (dict(q=None), 1, "static query"),
    (dict(norm=5), 1, "output_norm"),
    (dict(values=False), 1, "values"),
    (dict(strides=[4, 8]), 1, "stride"),
    (dict(out=None), 1, "output"),
])
def test_forward_argument_validation(kwargs, code, msg):
    assert _fwd(**kwargs) == code
    assert msg in N.load().attnres_last_error().decode()


def test_zero_tokens_is_a_no_op_without_a_device():
    assert _fwd(n=0, out=None) == 0


def test_workspace_query_rejects_invalid_geometry():
    L = N.load()
    assert L.attnres_lrid_backward_workspace_bytes(0, 16, 64, 16, 1, 2) == 0
    assert L.attnres_lrid_backward_workspace_bytes(4, 16, 64, 15, 2, 2) == 0
    assert L.attnres_base_backward_workspace_bytes(4, -1, 64, 2) == 0


def test_check_raises_with_library_message():
    _fwd(S=0)
    with pytest.raises(N.AttnResError, match="num_sources"):
        N.check(2, "attnres_lrid_forward")


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(N.AttnResError, match="not found"):
        N.load(str(tmp_path / "nope.so"))


ERR_INVALID_ARGUMENT = 1  # include/attnres_b200.h


@pytest.mark.parametrize("args,msg", [
    ((64, 384, 64, 0, 0), "bad geometry"),    # no heads
    ((64, 384, 64, 0, 3), "bad geometry"),    # rank not a multiple of the heads
    ((-1, 384, 64, 0, 1), "bad geometry"),    # negative token count
    ((64, 384, 64, -2, 1), "bad geometry"),   # negative query rank
])
def test_fused_key_projection_argument_validation(args, msg):
    """attnres_lrid_fused_key_projection rejects bad geometry with
    ATTNRES_ERR_INVALID_ARGUMENT and a message, before touching a device."""
    lib = N.load()
    n, din, rank, rq, heads = args
    rc = lib.attnres_lrid_fused_key_projection(n, din, rank, rq, heads, 2, None, din, None, din, 1, 1e-6,
                                               None, None, None, None)
    assert rc == ERR_INVALID_ARGUMENT
    assert msg in lib.attnres_last_error().decode()


def test_fused_key_projection_null_pointers_and_zero_tokens():
    lib = N.load()
    # zero tokens: nothing to do, no pointer needed
    assert lib.attnres_lrid_fused_key_projection(0, 384, 64, 0, 1, 2, None, 384, None, 384, 1, 1e-6,
                                                 None, None, None, None) == 0
    rc = lib.attnres_lrid_fused_key_projection(64, 384, 64, 0, 1, 2, None, 384, None, 384, 1, 1e-6,
                                               None, None, None, None)
    assert rc == ERR_INVALID_ARGUMENT and "NULL" in lib.attnres_last_error().decode()
    # key_norm needs the normalised-key and inverse-rms outputs
    fake = ctypes.c_void_p(0x1000)
    rc = lib.attnres_lrid_fused_key_projection(64, 384, 64, 0, 1, 2, fake, 384, fake, 384, 1, 1e-6,
                                               fake, None, None, None)
    assert rc == ERR_INVALID_ARGUMENT and "key_norm" in lib.attnres_last_error().decode()
