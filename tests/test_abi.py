"""The C-ABI library loads and exports every symbol include/pox_cuda.h declares (CPU only:
no compute call is made without a GPU)."""
import ctypes as C
import re

import pytest

from paraoxidizer_b200 import _lib as L
from paraoxidizer_b200.backend import CudaBackend, device_count


def test_header_declares_entry_points():
    syms = L.declared_symbols()
    for required in ("pox_cuda_create", "pox_cuda_gemv_int4", "pox_cuda_gemv_int4_outliers", "pox_cuda_gemv_int8",
                     "pox_cuda_tensor_upload", "pox_cuda_tensor_gemv", "pox_cuda_tensor_dequant"):
        assert required in syms


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    missing = [s for s in L.declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_exported_symbols_have_c_linkage():
    # nm -D shows the plain (unmangled) names for every declared entry point
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", L.LIB_PATH], capture_output=True, text=True).stdout
    names = set(re.findall(r"\b(pox_(?:cuda|file)_\w+)\b", out))
    assert set(L.declared_symbols()) <= names


def test_version_and_errors_without_gpu():
    lib = L.lib()
    assert b"sm_100a" in lib.pox_cuda_version()
    n = C.c_int(-1)
    assert lib.pox_cuda_device_count(C.byref(n)) == L.POX_OK
    assert n.value >= 0
    ctx = C.c_void_p()
    assert lib.pox_cuda_create(0, None) == L.POX_ERR_INVALID
    assert "NULL" in L.last_error()
    if n.value == 0:
        rc = lib.pox_cuda_create(0, C.byref(ctx))
        assert rc == L.POX_ERR_UNSUPPORTED and ctx.value is None
        # MetalBackend::new() -> None on a machine without the device (metal_backend.rs:193-195)
        assert CudaBackend.new(0) is None


def test_null_handles_are_rejected():
    lib = L.lib()
    assert lib.pox_cuda_tensor_info(None, None, None, None, None) == L.POX_ERR_INVALID
    assert lib.pox_cuda_tensor_gemv(None, None, None, 1, None, None) == L.POX_ERR_INVALID
    assert lib.pox_cuda_gemv_int4(None, None, 0, None, 0, 4, 4, 4, None, 0, None, 0) == L.POX_ERR_INVALID
    assert lib.pox_cuda_tensor_free(None, None) == L.POX_OK


def _prototypes():
    """{name: [parameter declarations]} of every function include/pox_cuda.h declares."""
    import re

    with open(L.HEADER) as f:
        src = re.sub(r"/\*.*?\*/", "", f.read(), flags=re.S)
    out = {}
    for m in re.finditer(r"(?:^|\n)\s*(?:const )?[a-z_0-9]+\s*\**\s*(pox_(?:cuda|file)_\w+)\s*\(([^;]*?)\);", src):
        params = " ".join(m.group(2).split())
        out[m.group(1)] = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
    return out


def test_ctypes_declarations_match_the_header():
    """Every function the Python binding declares has the header's number of parameters, and a
    pointer (or array) parameter is bound as a pointer type, a scalar as a scalar: the binding
    cannot drift from the C ABI unnoticed."""
    import ctypes as C

    protos = _prototypes()
    assert set(protos) == set(L.declared_symbols())
    lib = L.lib()
    scalars = (C.c_int, C.c_uint32, C.c_int32, C.c_size_t, C.c_float, C.c_uint64)
    checked = 0
    for name, params in protos.items():
        argtypes = getattr(getattr(lib, name), "argtypes", None)
        if argtypes is None:
            continue
        assert len(argtypes) == len(params), name
        for decl, t in zip(params, argtypes):
            is_ptr = "*" in decl or "[" in decl
            assert (t not in scalars) == is_ptr, (name, decl, t)
        checked += 1
    assert checked >= 50, checked
