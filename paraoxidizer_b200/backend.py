"""CudaBackend: the B200 backend object, shaped like the reference's MetalBackend.

Reference interfaces mirrored (paths relative to the reference repository root):
  * MetalBackend::new() -> Option<Arc<Self>>      crates/paraoxidizer-runtime/src/metal_backend.rs:64-82
  * MetalBackend::gemv_int4(...) -> Result<()>    metal_backend.rs:85-181
  * quant::gemv_int4 / gemv_int8                  crates/paraoxidizer-quant/src/kernels.rs:177-255
  * dequantize_int4_group / dequantize_int8_symmetric + SparseOutlierTable::apply_to
                                                  kernels.rs:85-173, outlier.rs:88-95
Every call goes through libpox_cuda.so; errors raise PoxError subclasses the way the reference
returns Err (QuantizationError for layout problems, RuntimeBackendError otherwise).
"""
from __future__ import annotations

import ctypes as C
from typing import Optional

import numpy as np

from . import _lib as L


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def _u8(a) -> np.ndarray:
    if a is None:
        return None
    a = np.asarray(a)
    if a.dtype != np.uint8:
        a = a.view(np.uint8) if a.flags.c_contiguous else np.ascontiguousarray(a).view(np.uint8)
    return np.ascontiguousarray(a).reshape(-1)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).reshape(-1)


def device_count() -> int:
    n = C.c_int(0)
    L.check(L.lib().pox_cuda_device_count(C.byref(n)))
    return n.value


class ResidentTensor:
    """A .pox tensor uploaded once to HBM (re-tiled weights, outlier CSR)."""

    def __init__(self, backend: "CudaBackend", handle: int, keep: tuple, dtype: int):
        self.backend = backend
        self.handle = handle
        self._keep = keep  # host slices stay alive (registry key of the host-slice calls)
        self.dtype = dtype
        rows, cols, nnz, nbytes = C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_size_t()
        L.check(L.lib().pox_cuda_tensor_info(handle, C.byref(rows), C.byref(cols), C.byref(nnz), C.byref(nbytes)))
        self.rows, self.cols, self.outlier_count, self.device_bytes = rows.value, cols.value, nnz.value, nbytes.value

    def gemv_host(self, x: np.ndarray, batch: int = 1) -> np.ndarray:
        """y[b] = W x[b] with host x ([batch][cols] f32), synchronous."""
        x = _f32(x)
        if x.size < batch * self.cols:
            raise L.QuantizationError(L.POX_ERR_LAYOUT, "x too small")
        y = np.zeros(batch * self.rows, np.float32)
        L.check(L.lib().pox_cuda_tensor_gemv_host(self.backend.ctx, self.handle, _ptr(x), batch, _ptr(y)))
        return y.reshape(batch, self.rows) if batch > 1 else y

    def gemv_device(self, x_ptr: int, batch: int, y_ptr: int, stream: int = 0) -> None:
        """Asynchronous GEMV on device pointers (x [batch][cols], y [batch][rows], f32)."""
        L.check(L.lib().pox_cuda_tensor_gemv(self.backend.ctx, self.handle, x_ptr, batch, y_ptr, stream or None))

    def gemv_kernel(self, batch: int) -> str:
        """Name of the kernel that serves a GEMV of this tensor at `batch` rows of x."""
        return L.lib().pox_cuda_tensor_gemv_kernel(self.handle, batch).decode()

    def dequant_host(self) -> np.ndarray:
        out = np.zeros(self.rows * self.cols, np.float32)
        L.check(L.lib().pox_cuda_tensor_dequant_host(self.backend.ctx, self.handle, _ptr(out)))
        return out

    def dequant_device(self, out_ptr: int, stream: int = 0) -> None:
        L.check(L.lib().pox_cuda_tensor_dequant(self.backend.ctx, self.handle, out_ptr, stream or None))

    def free(self) -> None:
        if self.handle:
            L.check(L.lib().pox_cuda_tensor_free(self.backend.ctx, self.handle))
            self.handle = None


class CudaBackend:
    """The CUDA counterpart of MetalBackend (metal_backend.rs:57-181)."""

    def __init__(self, ctx: int, device: int):
        self.ctx = ctx
        self.device = device
        self._children = []  # weak references to CudaModel objects (destroyed with the context)

    @staticmethod
    def new(device: int = 0) -> Optional["CudaBackend"]:
        """MetalBackend::new(): None when no usable device exists (metal_backend.rs:64-82, :193-195)."""
        ctx = C.c_void_p()
        rc = L.lib().pox_cuda_create(device, C.byref(ctx))
        if rc != L.POX_OK:
            return None
        return CudaBackend(ctx.value, device)

    @staticmethod
    def create(device: int = 0) -> "CudaBackend":
        """Like new() but raises with the library's message instead of returning None."""
        ctx = C.c_void_p()
        L.check(L.lib().pox_cuda_create(device, C.byref(ctx)))
        return CudaBackend(ctx.value, device)

    def check_missing_rank(self) -> float:
        """Failure-detection check of the peer exchange on this GPU (a two-rank exchange whose
        second rank never arrives must end with the bounded wait's error); returns the wait in s."""
        t = C.c_double(0.0)
        L.check(L.lib().pox_cuda_comm_check_missing_rank(self.ctx, C.byref(t)))
        return t.value

    def close(self) -> None:
        if self.ctx:
            for ref in self._children:  # pox_cuda_destroy frees the models still on the context
                child = ref()
                if child is not None:
                    child.handle = None
            self._children.clear()
            L.lib().pox_cuda_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synchronize(self) -> None:
        L.check(L.lib().pox_cuda_synchronize(self.ctx))

    @property
    def stream(self) -> int:
        return L.lib().pox_cuda_stream(self.ctx) or 0

    # ---- reference-shaped entry points --------------------------------------------------
    def gemv_int4(self, packed_weights, scale_data, rows: int, cols: int, group_size: int, x, y: np.ndarray) -> None:
        """MetalBackend::gemv_int4 (metal_backend.rs:85-181): y is written in place."""
        p, s, xf = _u8(packed_weights), _u8(scale_data), _f32(x)
        assert y.dtype == np.float32 and y.flags.c_contiguous
        L.check(L.lib().pox_cuda_gemv_int4(self.ctx, _ptr(p), p.size, _ptr(s), s.size, rows, cols, group_size,
                                           _ptr(xf), xf.size, _ptr(y), y.size))

    def gemv_int4_outliers(self, packed_weights, scale_data, group_size: int, rows: int, cols: int,
                           outlier_bytes, x, y: np.ndarray) -> None:
        """quant::gemv_int4 with Option<&SparseOutlierTable> given as .pox bytes (kernels.rs:177-226)."""
        p, s, xf = _u8(packed_weights), _u8(scale_data), _f32(x)
        o = _u8(outlier_bytes)
        assert y.dtype == np.float32 and y.flags.c_contiguous
        L.check(L.lib().pox_cuda_gemv_int4_outliers(self.ctx, _ptr(p), p.size, _ptr(s), s.size, group_size, rows,
                                                     cols, _ptr(o), 0 if o is None else o.size, _ptr(xf), xf.size,
                                                     _ptr(y), y.size))

    def gemv_int8(self, q_weights, scale_data, rows: int, cols: int, x, y: np.ndarray) -> None:
        """quant::gemv_int8 (kernels.rs:229-255)."""
        q, s, xf = _u8(q_weights), _u8(scale_data), _f32(x)
        assert y.dtype == np.float32 and y.flags.c_contiguous
        L.check(L.lib().pox_cuda_gemv_int8(self.ctx, _ptr(q), q.size, _ptr(s), s.size, rows, cols, _ptr(xf),
                                           xf.size, _ptr(y), y.size))

    # ---- residency ------------------------------------------------------------------------
    def upload(self, dtype: int, rows: int, cols: int, data, scales=None, outliers=None,
               group_size: int = 0) -> ResidentTensor:
        d, s, o = _u8(data), _u8(scales), _u8(outliers)
        desc = L.TensorDesc()
        desc.dtype, desc.rows, desc.cols, desc.group_size = dtype, rows, cols, group_size
        desc.data, desc.data_len = _ptr(d), d.size
        desc.scales, desc.scale_len = _ptr(s), 0 if s is None else s.size
        desc.outliers, desc.outlier_len = _ptr(o), 0 if o is None else o.size
        h = C.c_void_p()
        L.check(L.lib().pox_cuda_tensor_upload(self.ctx, C.byref(desc), C.byref(h)))
        return ResidentTensor(self, h.value, (d, s, o), dtype)

    def upload_int4(self, packed, scales, rows, cols, group_size, outliers=None) -> ResidentTensor:
        return self.upload(L.POX_I4, rows, cols, packed, scales, outliers, group_size)

    def upload_int8(self, q, scale, rows, cols) -> ResidentTensor:
        return self.upload(L.POX_I8, rows, cols, q, scale)

    def upload_int8_rows(self, q, row_scales, rows, cols) -> ResidentTensor:
        """INT8 with one f16 scale per output row (quant.quantize_int8_rows), the per-channel extension."""
        return self.upload(L.POX_I8, rows, cols, q, row_scales, None, 1)

    def upload_f16(self, w_bits, rows, cols) -> ResidentTensor:
        return self.upload(L.POX_F16, rows, cols, w_bits)
