"""ctypes binding of libpox_cuda.so (the C ABI declared in include/pox_cuda.h).

The library is required: importing the GPU entry points without it raises immediately
(there is no CPU fallback in this package).
"""
from __future__ import annotations

import ctypes as C
import os
import re

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libpox_cuda.so")
HEADER = os.path.join(os.path.dirname(_PKG), "include", "pox_cuda.h")

POX_OK, POX_ERR_LAYOUT, POX_ERR_UNSUPPORTED, POX_ERR_CUDA = 0, 1, 2, 3
POX_ERR_NCCL, POX_ERR_TIMEOUT, POX_ERR_OOM, POX_ERR_INVALID = 4, 5, 6, 7
POX_ERR_FORMAT, POX_ERR_INTEGRITY = 8, 9
STATUS_NAMES = {0: "OK", 1: "LAYOUT", 2: "UNSUPPORTED", 3: "CUDA", 4: "NCCL", 5: "TIMEOUT", 6: "OOM", 7: "INVALID",
                8: "FORMAT", 9: "INTEGRITY"}

# DType codes (crates/paraoxidizer-core/src/tensor.rs:4-20)
POX_F32, POX_F16, POX_BF16, POX_I8, POX_I4 = 0, 1, 2, 3, 4


class PoxError(Exception):
    """Mirror of crates/paraoxidizer-core/src/error.rs:6-58 for the codes this backend returns."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class QuantizationError(PoxError):
    """PoxError::Quantization (layout / dimension mismatch, error.rs:25-26)."""


class RuntimeBackendError(PoxError):
    """PoxError::Runtime (error.rs:50-51)."""


class TensorDesc(C.Structure):
    _fields_ = [("dtype", C.c_int), ("rows", C.c_size_t), ("cols", C.c_size_t), ("group_size", C.c_size_t),
                ("data", C.c_void_p), ("data_len", C.c_size_t), ("scales", C.c_void_p), ("scale_len", C.c_size_t),
                ("outliers", C.c_void_p), ("outlier_len", C.c_size_t)]


class GemvOp(C.Structure):
    """pox_gemv_op (include/pox_cuda.h): RMSNorm / SwiGLU fused into a GEMV's input."""

    _fields_ = [("mode", C.c_int), ("norm_w", C.c_void_p), ("eps", C.c_float), ("up", C.c_void_p),
                ("ld_x", C.c_uint32), ("ld_up", C.c_uint32)]


POX_OP_NONE, POX_OP_RMSNORM, POX_OP_SWIGLU = 0, 1, 2


class LlamaConfig(C.Structure):
    """pox_llama_config (include/pox_cuda.h): ModelConfig fields of the decode path
    (crates/paraoxidizer-core/src/arch.rs:96-112)."""

    _fields_ = [("hidden", C.c_uint32), ("intermediate", C.c_uint32), ("layers", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("vocab", C.c_uint32), ("rms_eps", C.c_float), ("rope_theta", C.c_float)]


_lib = None


def declared_symbols() -> list[str]:
    """Every function name include/pox_cuda.h declares."""
    with open(HEADER) as f:
        src = f.read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(pox_(?:cuda|file)_\w+)\s*\(", src)))


POX_COMM_NCCL, POX_COMM_PEER = 1, 2


def _declare(L):
    vp, sz, i32, u32 = C.c_void_p, C.c_size_t, C.c_int, C.c_uint32
    sig = {
        "pox_cuda_last_error": (C.c_char_p, []),
        "pox_cuda_version": (C.c_char_p, []),
        "pox_cuda_device_count": (i32, [C.POINTER(C.c_int)]),
        "pox_cuda_create": (i32, [i32, C.POINTER(vp)]),
        "pox_cuda_destroy": (None, [vp]),
        "pox_cuda_synchronize": (i32, [vp]),
        "pox_cuda_stream": (vp, [vp]),
        "pox_cuda_gemv_int4": (i32, [vp, vp, sz, vp, sz, sz, sz, sz, vp, sz, vp, sz]),
        "pox_cuda_gemv_int4_outliers": (i32, [vp, vp, sz, vp, sz, sz, sz, sz, vp, sz, vp, sz, vp, sz]),
        "pox_cuda_gemv_int8": (i32, [vp, vp, sz, vp, sz, sz, sz, vp, sz, vp, sz]),
        "pox_cuda_tensor_upload": (i32, [vp, C.POINTER(TensorDesc), C.POINTER(vp)]),
        "pox_cuda_tensor_free": (i32, [vp, vp]),
        "pox_cuda_tensor_info": (i32, [vp, C.POINTER(sz), C.POINTER(sz), C.POINTER(sz), C.POINTER(sz)]),
        "pox_cuda_tensor_gemv_kernel": (C.c_char_p, [vp, sz]),
        "pox_cuda_tensor_gemv": (i32, [vp, vp, vp, sz, vp, vp]),
        "pox_cuda_tensor_gemv_host": (i32, [vp, vp, vp, sz, vp]),
        "pox_cuda_tensor_gemv_noalloc": (i32, [vp, vp, vp, sz, vp, vp]),
        "pox_cuda_tensor_gemv_ex": (i32, [vp, vp, vp, sz, vp, C.POINTER(GemvOp), vp, vp]),
        "pox_cuda_model_create": (i32, [vp, C.POINTER(LlamaConfig), u32, u32, u32, C.POINTER(vp)]),
        "pox_cuda_model_create_tp": (i32, [vp, C.POINTER(LlamaConfig), u32, u32, u32, u32, u32, C.POINTER(vp)]),
        "pox_cuda_comm_unique_id": (i32, [vp]),
        "pox_cuda_model_comm_nccl": (i32, [vp, vp]),
        "pox_cuda_model_comm_ipc_handle": (i32, [vp, vp]),
        "pox_cuda_model_comm_peer": (i32, [vp, vp]),
        "pox_cuda_model_comm_mode": (i32, [vp, i32]),
        "pox_cuda_comm_check_missing_rank": (i32, [vp, C.POINTER(C.c_double)]),
        "pox_cuda_model_destroy": (None, [vp]),
        "pox_cuda_model_set_layer_tensors": (i32, [vp, u32, vp, vp, vp, vp, vp, vp]),
        "pox_cuda_quantize_int4": (i32, [vp, vp, sz, sz, vp, vp, vp]),
        "pox_cuda_extract_outliers": (i32, [vp, vp, sz, C.c_float, vp, sz, C.POINTER(sz)]),
        "pox_cuda_model_set_embeddings": (i32, [vp, vp, vp, vp]),
        "pox_cuda_model_set_layer": (i32, [vp, u32, C.POINTER(TensorDesc), vp, vp]),
        "pox_cuda_model_decode": (i32, [vp, u32, vp, vp, vp, vp, vp]),
        "pox_cuda_model_prefill": (i32, [vp, u32, vp, vp, vp, u32, vp, vp, vp]),
        "pox_cuda_model_decode_device": (i32, [vp, u32, vp, vp, vp, vp, vp, i32, vp]),
        "pox_cuda_model_set_persistent": (i32, [vp, i32]),
        "pox_cuda_model_step_persistent": (i32, [vp, u32]),
        "pox_cuda_model_set_state": (i32, [vp, u32, vp, vp, vp]),
        "pox_cuda_model_buffers": (i32, [vp, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(vp),
                                         C.POINTER(vp)]),
        "pox_cuda_paged_attention": (i32, [vp, vp, vp, vp, vp, vp, u32, u32, u32, u32, u32, u32, vp, vp]),
        "pox_file_open": (i32, [C.c_char_p, C.POINTER(vp)]),
        "pox_file_from_bytes": (i32, [vp, sz, C.POINTER(vp)]),
        "pox_file_close": (None, [vp]),
        "pox_file_tensor_count": (i32, [vp, C.POINTER(sz)]),
        "pox_file_tensor_meta": (i32, [vp, sz, vp]),
        "pox_file_find": (i32, [vp, C.c_char_p, C.POINTER(sz)]),
        "pox_file_tensor_data": (i32, [vp, C.c_char_p, C.POINTER(vp), C.POINTER(sz)]),
        "pox_file_scale_data": (i32, [vp, C.c_char_p, C.POINTER(vp), C.POINTER(sz)]),
        "pox_file_outlier_data": (i32, [vp, C.c_char_p, C.POINTER(vp), C.POINTER(sz)]),
        "pox_file_model_config": (i32, [vp, C.POINTER(LlamaConfig), C.POINTER(C.c_int)]),
        "pox_file_verify_integrity": (i32, [vp, i32]),
        "pox_file_tensor_shard": (i32, [vp, C.c_char_p, i32, u32, u32, vp, C.POINTER(sz), vp, C.POINTER(sz), vp,
                                        C.POINTER(sz)]),
        "pox_cuda_model_load": (i32, [vp, vp, u32, u32, u32, u32, u32, C.POINTER(vp)]),
        "pox_cuda_tensor_dequant": (i32, [vp, vp, vp, vp]),
        "pox_cuda_tensor_dequant_host": (i32, [vp, vp, vp]),
    }
    for name, (res, args) in sig.items():
        if hasattr(L, name):
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
    try:
        from . import _lib_ext
        _lib_ext.declare(L)
    except ImportError:
        pass


def lib():
    """Load libpox_cuda.so (raises if it has not been built: no silent fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m paraoxidizer_b200.build`")
        L = C.CDLL(LIB_PATH)
        _declare(L)
        _lib = L
    return _lib


def last_error() -> str:
    m = lib().pox_cuda_last_error()
    return m.decode() if m else ""


def check(rc: int) -> None:
    if rc == POX_OK:
        return
    msg = last_error()
    if rc == POX_ERR_LAYOUT:
        raise QuantizationError(rc, msg)
    raise RuntimeBackendError(rc, msg)
