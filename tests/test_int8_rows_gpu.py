"""INT8 with one f16 scale per output row (the per-output-channel layout of the benchmark's INT8
configuration; the reference's .pox INT8 is per tensor, kernels.rs:131-154, so this is an extension
whose oracle applies the reference's gemv_int8 arithmetic, kernels.rs:229-255, with the row's scale).

Bars: the host quantizer equals the oracle's bit for bit; dequantization is bit-exact; GEMV outputs
within max |y - ref| / max |ref| <= 1e-3 per row of x on every kernel that serves INT8 (the batch <= 8
GEMV, the integer tcgen05 kernel up to a padded batch of 64, the f16 tiles above), including a
matrix whose rows differ in scale by orders of magnitude.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu
GEMV_TOL = 1e-3
POOL = ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def be():
    b = CudaBackend.create(0)
    yield b
    b.close()


def max_rel(y, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


def make(rows, cols, seed, spread=False):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    if spread:  # row magnitudes over four decades: a per-tensor scale would flush the small rows
        w.reshape(rows, cols)[:] *= (10.0 ** rng.uniform(-2, 2, rows)).astype(np.float32)[:, None]
    q, s = Q.quantize_int8_rows(w, rows, cols)
    qo, so = O.quantize_int8_rows(w, rows, cols)
    assert np.array_equal(q, qo) and np.array_equal(s, so)
    return q, s


@pytest.fixture(scope="module")
def mlp(be):
    rows, cols = 14336, 4096
    q, s = make(rows, cols, 5)
    t = be.upload_int8_rows(q, s, rows, cols)
    yield t, q, s
    t.free()


@pytest.mark.parametrize("batch", [1, 4, 16, 64])
def test_int8_rows_14336x4096(be, mlp, batch):
    t, q, s = mlp
    rng = np.random.default_rng(batch)
    x = rng.standard_normal((batch, 4096), dtype=np.float32).astype(np.float16).astype(np.float32)
    y = t.gemv_host(x, batch).reshape(batch, 14336)
    refs = list(POOL.map(lambda v: O.gemv_int8_rows(q, s, 14336, 4096, v), x))
    for b in range(batch):
        assert max_rel(y[b], refs[b]) <= GEMV_TOL, (batch, b, t.gemv_kernel(batch))


@pytest.mark.parametrize("rows,cols,batch", [(1000, 1024, 3), (333, 1024, 40), (300, 4096, 128), (70, 96, 2),
                                             (513, 640, 9)])
def test_int8_rows_shapes_and_dequant(be, rows, cols, batch):
    q, s = make(rows, cols, rows + cols, spread=True)
    t = be.upload_int8_rows(q, s, rows, cols)
    rng = np.random.default_rng(batch)
    x = rng.standard_normal((batch, cols), dtype=np.float32)
    y = np.asarray(t.gemv_host(x, batch)).reshape(batch, rows)
    for b in range(batch):
        ref = O.gemv_int8_rows(q, s, rows, cols, x[b])
        assert max_rel(y[b], ref) <= GEMV_TOL, (rows, cols, batch, b, t.gemv_kernel(batch))
    deq = t.dequant_host()
    ref_d = O.dequantize_int8_rows(q, s, rows, cols)
    assert np.array_equal(deq.view(np.uint32), ref_d.view(np.uint32))
    t.free()


def test_int8_rows_layout_errors(be):
    from paraoxidizer_b200 import _lib as L

    q, s = make(16, 64, 1)
    with pytest.raises(L.QuantizationError):
        be.upload_int8_rows(q, s[:10], 16, 64)  # fewer than rows x 2 scale bytes
    with pytest.raises(L.PoxError):
        be.upload(L.POX_I8, 16, 64, q, s, None, 2)  # group_size 2: neither layout
