"""GPU parity of the GEMV with fused input operations (pox_cuda_tensor_gemv_ex) against the oracle:
RMSNorm (crates/paraoxidizer-runtime/src/engine.rs:294-350) or SwiGLU (engine.rs:671-677) applied to
x before the product, and a residual added after it (engine.rs:646-648, 682-684). Bar: max|Δ| /
max|ref| <= 1e-3 (the GEMV tolerance)."""
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


def run_ex(be, t, x, batch, op=None, resid=None, rows=None):
    import torch

    dev = torch.device("cuda", 0)
    xd = torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(dev)
    rd = None if resid is None else torch.from_numpy(np.ascontiguousarray(resid, np.float32)).to(dev)
    yd = torch.zeros(batch * rows, dtype=torch.float32, device=dev)
    keep = []
    if op is not None:
        for k in ("norm_w", "up"):
            v = getattr(op, k + "_host", None)
            if v is not None:
                td = torch.from_numpy(v).to(dev)
                keep.append(td)
                setattr(op, k, td.data_ptr())
    torch.cuda.synchronize()
    L.check(L.lib().pox_cuda_tensor_gemv_ex(be.ctx, t.handle, xd.data_ptr(), batch, yd.data_ptr(),
                                            None if op is None else C.byref(op),
                                            None if rd is None else rd.data_ptr(), None))
    be.synchronize()
    return yd.cpu().numpy().reshape(batch, rows)


class Op(L.GemvOp):
    pass


@pytest.mark.parametrize("kind", ["i4", "i4_outliers", "f16"])
@pytest.mark.parametrize("batch", [1, 3])
def test_gemv_rmsnorm_residual(be, kind, batch):
    rng = np.random.default_rng(41 + batch)
    rows, cols = 384, 1024
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    if kind == "f16":
        wb = w.astype(np.float16).view(np.uint16)
        t = be.upload_f16(wb, rows, cols)
        gemv = lambda v: O.gemv_f16(wb, rows, cols, v)
    else:
        tab = None
        if kind == "i4_outliers":
            w.reshape(rows, cols)[:, rng.choice(cols, 8, replace=False)] *= np.float32(20)
            tab = Q.extract_and_zero_outliers(w, "automatic")
        p, s = Q.quantize_int4_group(w, 128)
        t = be.upload_int4(p, s, rows, cols, 128, None if tab is None else Q.outliers_to_bytes(*tab))
        gemv = lambda v: O.gemv_int4(p, s, 128, rows, cols, tab, v)
    x = rng.standard_normal(batch * cols, dtype=np.float32) * np.float32(3.0)
    nw = (1.0 + 0.2 * rng.standard_normal(cols, dtype=np.float32)).astype(np.float16).view(np.uint16)
    resid = rng.standard_normal(batch * rows, dtype=np.float32)
    op = Op()
    op.mode, op.eps = L.POX_OP_RMSNORM, np.float32(1e-5)
    op.norm_w_host = nw
    y = run_ex(be, t, x, batch, op, resid, rows)
    for b in range(batch):
        xn = O.rms_norm(x[b * cols:(b + 1) * cols], nw, 1e-5)
        ref = resid[b * rows:(b + 1) * rows] + gemv(xn)
        assert rel(y[b], ref) <= TOL, (kind, b, rel(y[b], ref))
    t.free()


@pytest.mark.parametrize("batch", [1, 2, 9])
def test_gemv_swiglu(be, batch):
    rng = np.random.default_rng(7 + batch)
    rows, inter = 256, 512
    w = rng.standard_normal(rows * inter, dtype=np.float32) * np.float32(0.02)
    p, s = Q.quantize_int4_group(w, 128)
    t = be.upload_int4(p, s, rows, inter, 128)
    gu = rng.standard_normal(batch * 2 * inter, dtype=np.float32) * np.float32(2.0)  # [batch][gate | up]
    import torch

    op = Op()
    op.mode, op.ld_x, op.ld_up = L.POX_OP_SWIGLU, 2 * inter, 2 * inter
    gud = torch.from_numpy(gu).cuda()
    op.up = gud.data_ptr() + inter * 4
    yd = torch.zeros(batch * rows, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    L.check(L.lib().pox_cuda_tensor_gemv_ex(be.ctx, t.handle, gud.data_ptr(), batch, yd.data_ptr(), C.byref(op),
                                            None, None))
    be.synchronize()
    y = yd.cpu().numpy().reshape(batch, rows)
    for b in range(batch):
        g = gu[b * 2 * inter:b * 2 * inter + inter]
        u = gu[b * 2 * inter + inter:(b + 1) * 2 * inter]
        ref = O.gemv_int4(p, s, 128, rows, inter, None, O.swiglu(g, u))
        assert rel(y[b], ref) <= TOL, (b, rel(y[b], ref))
    t.free()
