"""pox_cuda_tensor_gemv_noalloc: the GEMV for callers that cannot allocate device memory while
running (an engine whose HBM is reserved at start-up, a host runtime that only hands over buffers
it owns). Its prepared-x scratch is a fixed device array instead of the tensor's buffer; its
results must match pox_cuda_tensor_gemv's within the GEMV tolerance of the other tests, on two
calls in a row (the array keeps the previous call's contents), and it must reject sizes beyond
the array with a clear error.

Collected last (file name) so that a stop-at-first-failure run has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

from paraoxidizer_b200 import _lib as L
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3


def max_rel(y, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


def test_noalloc_matches_tensor_gemv_on_two_calls():
    import torch

    be = CudaBackend.create(0)
    rng = np.random.default_rng(31)
    rows, cols = 1024, 4096
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    w.reshape(rows, cols)[:, rng.choice(cols, 20, replace=False)] *= np.float32(20.0)
    tab = Q.extract_and_zero_outliers(w, "automatic")
    packed, scales = Q.quantize_int4_group(w, 128)
    t4 = be.upload_int4(packed, scales, rows, cols, 128, Q.outliers_to_bytes(*tab))
    q8, s8 = Q.quantize_int8_symmetric(w)
    t8 = be.upload_int8(q8, s8, rows, cols)
    lib = L.lib()
    dev = torch.device("cuda", 0)
    try:
        # two calls in a row on the shared array, with different batch sizes and tensors
        for t, batch, seed in ((t4, 3, 1), (t8, 1, 2), (t4, 1, 3)):
            x = torch.from_numpy(rng.standard_normal(batch * cols, dtype=np.float32)).to(dev)
            y_ref = torch.zeros(batch * rows, dtype=torch.float32, device=dev)
            y_new = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device=dev)
            torch.cuda.synchronize()  # the library's stream does not order against torch's
            L.check(lib.pox_cuda_tensor_gemv(be.ctx, t.handle, x.data_ptr(), batch, y_ref.data_ptr(), None))
            L.check(lib.pox_cuda_tensor_gemv_noalloc(be.ctx, t.handle, x.data_ptr(), batch, y_new.data_ptr(),
                                                     None))
            be.synchronize()
            yr, yn = y_ref.cpu().numpy(), y_new.cpu().numpy()
            assert np.all(np.isfinite(yn))
            for b in range(batch):
                assert max_rel(yn[b * rows:(b + 1) * rows], yr[b * rows:(b + 1) * rows]) <= GEMV_TOL, (seed, b)

        # batch 11: two launches of up to 8 rows inside one call, both through the shared array
        batch = 11
        x = torch.from_numpy(rng.standard_normal(batch * cols, dtype=np.float32)).to(dev)
        y_ref = torch.zeros(batch * rows, dtype=torch.float32, device=dev)
        y_new = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        L.check(lib.pox_cuda_tensor_gemv(be.ctx, t8.handle, x.data_ptr(), batch, y_ref.data_ptr(), None))
        L.check(lib.pox_cuda_tensor_gemv_noalloc(be.ctx, t8.handle, x.data_ptr(), batch, y_new.data_ptr(), None))
        be.synchronize()
        yr, yn = y_ref.cpu().numpy(), y_new.cpu().numpy()
        for b in range(batch):
            assert max_rel(yn[b * rows:(b + 1) * rows], yr[b * rows:(b + 1) * rows]) <= GEMV_TOL, ("b11", b)

        # beyond the array: a clear error, nothing launched
        big = 40960
        wb = rng.standard_normal(16 * big, dtype=np.float32) * np.float32(0.02)
        pb, sb = Q.quantize_int4_group(wb, 128)
        tb = be.upload_int4(pb, sb, 16, big, 128)
        xb = torch.zeros(big, dtype=torch.float32, device=dev)
        yb = torch.zeros(16, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        rc = lib.pox_cuda_tensor_gemv_noalloc(be.ctx, tb.handle, xb.data_ptr(), 1, yb.data_ptr(), None)
        assert rc == L.POX_ERR_UNSUPPORTED
        assert "32768" in L.last_error()
        tb.free()
    finally:
        t4.free()
        t8.free()
        be.close()


def test_noalloc_f16_at_the_array_limit():
    """An F16 tensor with cols = 32768 fills the array exactly (prepared x of 8 rows as f16 hi / lo
    pairs: 1 MiB, plus 16 KiB of block metadata): accepted and equal to pox_cuda_tensor_gemv on two
    calls in a row. cols = 32800 (one 32-column block more) is rejected with POX_ERR_UNSUPPORTED."""
    import torch

    be = CudaBackend.create(0)
    lib = L.lib()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(41)
    try:
        rows, cols = 64, 32768
        wb = (rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)).astype(np.float16)
        t = be.upload_f16(wb.view(np.uint16), rows, cols)
        for batch in (8, 3):
            x = torch.from_numpy(rng.standard_normal(batch * cols, dtype=np.float32)).to(dev)
            y_ref = torch.zeros(batch * rows, dtype=torch.float32, device=dev)
            y_new = torch.full((batch * rows,), float("nan"), dtype=torch.float32, device=dev)
            torch.cuda.synchronize()
            L.check(lib.pox_cuda_tensor_gemv(be.ctx, t.handle, x.data_ptr(), batch, y_ref.data_ptr(), None))
            L.check(lib.pox_cuda_tensor_gemv_noalloc(be.ctx, t.handle, x.data_ptr(), batch, y_new.data_ptr(), None))
            be.synchronize()
            yr, yn = y_ref.cpu().numpy(), y_new.cpu().numpy()
            assert np.all(np.isfinite(yn))
            for b in range(batch):
                assert max_rel(yn[b * rows:(b + 1) * rows], yr[b * rows:(b + 1) * rows]) <= GEMV_TOL, (batch, b)
        t.free()
        cols = 32800
        wb = np.zeros(16 * cols, np.uint16)
        t = be.upload_f16(wb, 16, cols)
        x = torch.zeros(cols, dtype=torch.float32, device=dev)
        y = torch.zeros(16, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        rc = lib.pox_cuda_tensor_gemv_noalloc(be.ctx, t.handle, x.data_ptr(), 1, y.data_ptr(), None)
        assert rc == L.POX_ERR_UNSUPPORTED and "32768" in L.last_error()
        t.free()
    finally:
        be.close()


def test_noalloc_reports_an_earlier_kernel_error():
    """The call returns before its kernels run, so an error a kernel raised on the context's flag is
    returned by the next call instead of being dropped: here the flag is raised by a paged attention
    call given a page outside the pool, the next no-alloc GEMV returns it and launches nothing, and
    the call after that runs normally."""
    import torch

    be = CudaBackend.create(0)
    lib = L.lib()
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(43)
    try:
        rows, cols = 256, 1024
        w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
        packed, scales = Q.quantize_int4_group(w, 128)
        t = be.upload_int4(packed, scales, rows, cols, 128)
        heads, kvh, hd, nblk = 4, 1, 128, 2
        q = torch.zeros(heads * hd, dtype=torch.float32, device=dev)
        kp = torch.zeros(nblk * kvh * 16 * hd, dtype=torch.int16, device=dev)
        tab = torch.tensor([nblk + 7], dtype=torch.int32, device=dev)  # outside the pool
        pos = torch.tensor([3], dtype=torch.int32, device=dev)
        out = torch.zeros(heads * hd, dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        L.check(lib.pox_cuda_paged_attention(be.ctx, q.data_ptr(), kp.data_ptr(), kp.data_ptr(), tab.data_ptr(),
                                             pos.data_ptr(), 1, heads, kvh, hd, nblk, 1, out.data_ptr(), None))
        torch.cuda.synchronize()  # the attention kernel has raised the flag; nothing has read it yet
        x = torch.from_numpy(rng.standard_normal(cols, dtype=np.float32)).to(dev)
        y = torch.full((rows,), float("nan"), dtype=torch.float32, device=dev)
        rc = lib.pox_cuda_tensor_gemv_noalloc(be.ctx, t.handle, x.data_ptr(), 1, y.data_ptr(), None)
        assert rc == L.POX_ERR_INVALID, (rc, L.last_error())
        be.synchronize()
        assert torch.isnan(y).all()  # nothing was launched
        y_ref = torch.zeros(rows, dtype=torch.float32, device=dev)
        L.check(lib.pox_cuda_tensor_gemv_noalloc(be.ctx, t.handle, x.data_ptr(), 1, y.data_ptr(), None))
        L.check(lib.pox_cuda_tensor_gemv(be.ctx, t.handle, x.data_ptr(), 1, y_ref.data_ptr(), None))
        be.synchronize()
        assert max_rel(y.cpu().numpy(), y_ref.cpu().numpy()) <= GEMV_TOL
        t.free()
    finally:
        be.close()
