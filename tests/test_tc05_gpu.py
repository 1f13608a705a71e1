"""GPU parity of the small-M tensor-core path (batch >= 9 rows of x: gemm_tc05.cu, tcgen05 f16
MMA) against the oracle's quant::gemv_int4 / gemv_int8 (crates/paraoxidizer-quant/src/kernels.rs:
177-255) and the F16 projection (engine.rs:235-250), row by row of x. Bar: max|Δ| / max|ref| <= 1e-3
per row of x (the GEMV tolerance). Covers padding of the batch (9 .. 128, and 200 = two launches),
row counts that are not multiples of 128, k-splits, outliers, fused RMSNorm / SwiGLU and residual."""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import _lib as L
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def be():
    b = CudaBackend.create(0)
    yield b
    b.close()


def rel(y, ref):
    return float(np.max(np.abs(y - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


def make(be, kind, rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    if kind == "f16":
        wb = w.astype(np.float16).view(np.uint16)
        return be.upload_f16(wb, rows, cols), lambda v: O.gemv_f16(wb, rows, cols, v)
    if kind == "i8":
        q, s = Q.quantize_int8_symmetric(w)
        return be.upload_int8(q, s, rows, cols), lambda v: O.gemv_int8(q, s, rows, cols, v)
    tab = None
    if kind == "i4_outliers":
        w.reshape(rows, cols)[:, rng.choice(cols, max(4, cols // 200), replace=False)] *= np.float32(20)
        tab = Q.extract_and_zero_outliers(w, "automatic")
        assert tab is not None
    p, s = Q.quantize_int4_group(w, 128)
    t = be.upload_int4(p, s, rows, cols, 128, None if tab is None else Q.outliers_to_bytes(*tab))
    return t, lambda v: O.gemv_int4(p, s, 128, rows, cols, tab, v)


@pytest.mark.parametrize("kind,rows,cols", [("i4", 768, 1024), ("i4_outliers", 640, 2048), ("i8", 1000, 1024),
                                            ("f16", 512, 1024), ("i4", 4096, 4096), ("i4", 200, 14336),
                                            ("i8", 3000, 4096)])
@pytest.mark.parametrize("batch", [9, 16, 33, 64, 128, 200])
def test_small_m_matches_oracle(be, kind, rows, cols, batch):
    if rows * cols > 4096 * 4096 // 2 and batch not in (16, 64):
        pytest.skip("large shape: two batch sizes suffice")
    t, gemv = make(be, kind, rows, cols, 100 + batch)
    rng = np.random.default_rng(batch)
    x = (rng.standard_normal(batch * cols, dtype=np.float32) * np.float32(1.5)).reshape(batch, cols)
    x[batch // 2] *= np.float32(1e4)   # rows of very different scale share a launch
    x[batch - 1] *= np.float32(1e-6)
    y = t.gemv_host(x, batch).reshape(batch, rows)
    worst = 0.0
    for b in range(batch):
        r = rel(y[b], gemv(x[b]))
        worst = max(worst, r)
        assert r <= TOL, (kind, rows, cols, batch, b, r)
    t.free()


class Op(L.GemvOp):
    pass


@pytest.mark.parametrize("kind", ["i4_outliers", "i4"])  # f16 tiles / integer tensor cores
@pytest.mark.parametrize("batch", [12, 40])
def test_small_m_rmsnorm_residual(be, batch, kind):
    import torch

    rng = np.random.default_rng(5 + batch)
    rows, cols = 1536, 2048
    t, gemv = make(be, kind, rows, cols, 9)
    x = rng.standard_normal(batch * cols, dtype=np.float32) * np.float32(3.0)
    nw = (1.0 + 0.2 * rng.standard_normal(cols, dtype=np.float32)).astype(np.float16).view(np.uint16)
    resid = rng.standard_normal(batch * rows, dtype=np.float32)
    xd, rd, nwd = torch.from_numpy(x).cuda(), torch.from_numpy(resid).cuda(), torch.from_numpy(nw).cuda()
    yd = torch.zeros(batch * rows, dtype=torch.float32, device="cuda")
    op = Op()
    op.mode, op.eps, op.norm_w = L.POX_OP_RMSNORM, np.float32(1e-5), nwd.data_ptr()
    torch.cuda.synchronize()
    L.check(L.lib().pox_cuda_tensor_gemv_ex(be.ctx, t.handle, xd.data_ptr(), batch, yd.data_ptr(), C.byref(op),
                                            rd.data_ptr(), None))
    be.synchronize()
    y = yd.cpu().numpy().reshape(batch, rows)
    for b in range(batch):
        ref = resid[b * rows:(b + 1) * rows] + gemv(O.rms_norm(x[b * cols:(b + 1) * cols], nw, 1e-5))
        assert rel(y[b], ref) <= TOL, (b, rel(y[b], ref))
    t.free()


def test_small_m_swiglu_residual_in_place(be):
    """The decode step's down projection: x += W_down silu(g) * u, with y aliasing the residual."""
    import torch

    batch, rows, inter = 24, 1024, 1536
    rng = np.random.default_rng(3)
    t, gemv = make(be, "i4", rows, inter, 4)
    gu = rng.standard_normal(batch * 2 * inter, dtype=np.float32) * np.float32(2.0)
    x0 = rng.standard_normal(batch * rows, dtype=np.float32)
    gud, xd = torch.from_numpy(gu).cuda(), torch.from_numpy(x0.copy()).cuda()
    op = Op()
    op.mode, op.ld_x, op.ld_up, op.up = L.POX_OP_SWIGLU, 2 * inter, 2 * inter, gud.data_ptr() + inter * 4
    torch.cuda.synchronize()
    L.check(L.lib().pox_cuda_tensor_gemv_ex(be.ctx, t.handle, gud.data_ptr(), batch, xd.data_ptr(), C.byref(op),
                                            xd.data_ptr(), None))
    be.synchronize()
    y = xd.cpu().numpy().reshape(batch, rows)
    for b in range(batch):
        g = gu[b * 2 * inter:b * 2 * inter + inter]
        u = gu[b * 2 * inter + inter:(b + 1) * 2 * inter]
        ref = x0[b * rows:(b + 1) * rows] + gemv(O.swiglu(g, u))
        assert rel(y[b], ref) <= TOL, (b, rel(y[b], ref))
    t.free()


def test_small_m_agrees_with_gemv_path(be):
    """Batch 9 (small-M path) against the same rows computed 8 + 1 through the GEMV path."""
    rows, cols = 2048, 4096
    t, _ = make(be, "i4_outliers", rows, cols, 12)
    rng = np.random.default_rng(1)
    x = rng.standard_normal(9 * cols, dtype=np.float32).reshape(9, cols)
    y9 = t.gemv_host(x, 9).reshape(9, rows)
    y8 = t.gemv_host(x[:8], 8).reshape(8, rows)
    y1 = t.gemv_host(x[8:], 1).reshape(1, rows)
    ref = np.concatenate([y8, y1])
    for b in range(9):
        assert rel(y9[b], ref[b]) <= TOL
    t.free()


def test_kernel_choice_by_batch(be):
    """Which kernel serves a call: mma.sync GEMV up to batch 8, the integer tensor-core path for
    INT8 and INT4 without outliers (padded batch <= 64), the f16 tiles otherwise;
    below batch 9 the integer path takes over where it was measured faster (INT4 with K >= 8192 from
    batch 6, INT8 with >= 16 M weights from batch 2)."""
    t4, _ = make(be, "i4", 256, 1024, 1)
    t4o, _ = make(be, "i4_outliers", 256, 2048, 2)
    t8, _ = make(be, "i8", 256, 1024, 3)
    t4k, _ = make(be, "i4", 128, 8192, 4)
    t8big, _ = make(be, "i8", 4096, 4096, 5)
    assert t4.gemv_kernel(8) == "gemv_tc_kernel"
    assert t4.gemv_kernel(16) == "gemm_tq_kernel"
    assert t4.gemv_kernel(64) == "gemm_tq_kernel"
    assert t4.gemv_kernel(65) == "gemm_tc05_kernel"
    assert t4o.gemv_kernel(16) == "gemm_tc05_kernel"
    assert t8.gemv_kernel(4) == "gemv_tc_kernel"
    assert t8.gemv_kernel(64) == "gemm_tq_kernel"
    assert t8.gemv_kernel(65) == "gemm_tc05_kernel"
    assert [t4k.gemv_kernel(b) for b in (5, 6, 8)] == ["gemv_tc_kernel", "gemm_tq_kernel", "gemm_tq_kernel"]
    assert [t8big.gemv_kernel(b) for b in (1, 2)] == ["gemv_tc_kernel", "gemm_tq_kernel"]
    for t in (t4, t4o, t8, t4k, t8big):
        t.free()


@pytest.mark.parametrize("kind,rows,cols,batch", [("i4", 1000, 8192, 6), ("i4", 300, 14336, 8), ("i8", 4096, 4096, 2),
                                                  ("i8", 4100, 4096, 5)])
def test_integer_path_below_batch_9_matches_oracle(be, kind, rows, cols, batch):
    """Batches <= 8 routed to the integer tensor-core kernel keep the GEMV tolerance."""
    t, gemv = make(be, kind, rows, cols, 40 + batch)
    assert t.gemv_kernel(batch) == "gemm_tq_kernel"
    rng = np.random.default_rng(batch)
    x = (rng.standard_normal(batch * cols, dtype=np.float32) * np.float32(1.5)).reshape(batch, cols)
    y = t.gemv_host(x, batch).reshape(batch, rows)
    for b in range(batch):
        assert rel(y[b], gemv(x[b])) <= TOL, (kind, rows, cols, batch, b)
    t.free()
