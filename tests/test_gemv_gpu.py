"""GPU parity of the CUDA GEMV / dequantization path against the oracle, through the C ABI.

Bars: dequantized weights and outlier tables bit-exact; GEMV outputs
within max|y - ref| / max|ref| <= 1e-3 (fp32 accumulation), where ref is the oracle's
restatement of quant::gemv_int4 / gemv_int8 (crates/paraoxidizer-quant/src/kernels.rs:177-255).
"""
import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import QuantizationError, quant as Q
from paraoxidizer_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3


@pytest.fixture(scope="module")
def be():
    b = CudaBackend.create(0)  # raises (no fallback) when the GPU or library is unusable
    yield b
    b.close()


def max_rel(y, ref):
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


def make_w(rows, cols, seed, hot_cols=0):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    if hot_cols:
        hot = rng.choice(cols, hot_cols, replace=False)
        w.reshape(rows, cols)[:, hot] *= np.float32(20.0)
    return w


def make_x(cols, batch=1, seed=1):
    rng = np.random.default_rng(seed)
    return rng.standard_normal(batch * cols, dtype=np.float32).astype(np.float16).astype(np.float32)


def oracle_rowwise_dequant(packed, scales, gs, rows, cols):
    """dequantize_int4_group applied row by row, as gemv_int4 slices the buffers
    (kernels.rs:192-208)."""
    rb, sb = (cols + 1) // 2, ((cols + gs - 1) // gs) * 4
    return np.concatenate([O.dequantize_int4_group(packed[r * rb:(r + 1) * rb], scales[r * sb:(r + 1) * sb], gs, cols)
                           for r in range(rows)])


def i4_case(rows, cols, gs, seed=0, hot_cols=0, policy=None):
    w = make_w(rows, cols, seed, hot_cols)
    tab = Q.extract_and_zero_outliers(w, policy) if policy else None
    if cols % gs == 0:
        packed, scales = Q.quantize_int4_group(w, gs)
    else:
        # groups of the flat quantizer would straddle rows: quantize row by row so the buffers
        # have the per-row layout gemv_int4 reads (kernels.rs:191-200)
        parts = [Q.quantize_int4_group(w[r * cols:(r + 1) * cols], gs) for r in range(rows)]
        packed = np.concatenate([p for p, _ in parts])
        scales = np.concatenate([s for _, s in parts])
    ob = Q.outliers_to_bytes(*tab) if tab is not None else None
    return packed, scales, tab, ob


def test_gemv_int4_metal_entry_4096x4096(be):
    # workload: 4096x4096 INT4 g128, no outliers, x ~ N(0,1) fp16 (reference CPU-runnable case)
    rows = cols = 4096
    packed, scales, _, _ = i4_case(rows, cols, 128)
    x = make_x(cols)
    y = np.zeros(rows, np.float32)
    be.gemv_int4(packed, scales, rows, cols, 128, x, y)
    ref = O.gemv_int4(packed, scales, 128, rows, cols, None, x)
    assert max_rel(y, ref) <= GEMV_TOL
    # x enters the integer MMAs as a 15-bit per-128-block quantization (two exact int8 limbs):
    # ~2^-15 of the block max per element, i.e. ~5e-5 of max|y| here (20x inside the bar)
    assert max_rel(y, ref) <= 2.5e-4


def test_gemv_int4_metal_backend_case(be):
    """The reference's own test of its GPU GEMV (metal_backend.rs:226-246), through the call that
    mirrors MetalBackend::gemv_int4: 32 x 64 weights sin(0.05 i), x = cos(0.1 i), INT4 groups of
    32. The reference asserts sum |y| > 0.01; here y is also held to the oracle."""
    rows, cols, gs = 32, 64, 32
    w = np.sin(np.arange(rows * cols, dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    x = np.cos(np.arange(cols, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    packed, scales = Q.quantize_int4_group(w, gs)
    y = np.zeros(rows, np.float32)
    be.gemv_int4(packed, scales, rows, cols, gs, x, y)
    assert float(np.sum(np.abs(y))) > 0.01
    assert max_rel(y, O.gemv_int4(packed, scales, gs, rows, cols, None, x)) <= GEMV_TOL


def test_gemv_int4_outliers_4096x14336(be):
    # workload: 4096x14336 INT4 g128, 0.5% of input channels x20, 3.5-sigma extraction
    rows, cols = 4096, 14336
    packed, scales, tab, ob = i4_case(rows, cols, 128, seed=2, hot_cols=72, policy="automatic")
    assert tab is not None and 150_000 < tab[0].size < 300_000
    x = make_x(cols, seed=3)
    y = np.zeros(rows, np.float32)
    be.gemv_int4_outliers(packed, scales, 128, rows, cols, ob, x, y)
    ref = O.gemv_int4(packed, scales, 128, rows, cols, tab, x)
    assert max_rel(y, ref) <= GEMV_TOL
    t = be.upload_int4(packed, scales, rows, cols, 128, ob)
    assert t.outlier_count == tab[0].size
    deq = t.dequant_host()
    ref_d = O.dequantize_int4_group(packed, scales, 128, rows * cols)
    O.outliers_apply(tab[0], tab[1], ref_d)
    assert np.array_equal(deq.view(np.uint32), ref_d.view(np.uint32))
    t.free()


@pytest.mark.parametrize("rows,cols,gs", [(1000, 4096, 128), (33, 512, 256), (16, 128, 128), (7, 384, 256),
                                          (300, 320, 64), (17, 301, 32), (5, 200, 2)])
def test_gemv_int4_shapes_and_dequant(be, rows, cols, gs):
    packed, scales, tab, ob = i4_case(rows, cols, gs, seed=rows + cols, hot_cols=max(1, cols // 64),
                                      policy="automatic")
    x = make_x(cols, seed=4)
    t = be.upload_int4(packed, scales, rows, cols, gs, ob)
    y = t.gemv_host(x)
    ref = O.gemv_int4(packed, scales, gs, rows, cols, tab, x)
    assert max_rel(y, ref) <= GEMV_TOL
    deq = t.dequant_host()
    ref_d = oracle_rowwise_dequant(packed, scales, gs, rows, cols)
    if tab is not None:
        O.outliers_apply(tab[0], tab[1], ref_d)
    assert np.array_equal(deq.view(np.uint32), ref_d.view(np.uint32))
    t.free()


@pytest.mark.parametrize("batch", [1, 2, 3, 4, 5, 8, 11])
def test_gemv_int4_batched(be, batch):
    rows, cols = 1024, 2048
    packed, scales, tab, ob = i4_case(rows, cols, 128, seed=7, hot_cols=10, policy="automatic")
    x = make_x(cols, batch, seed=8)
    t = be.upload_int4(packed, scales, rows, cols, 128, ob)
    y = np.asarray(t.gemv_host(x, batch)).reshape(batch, rows)
    for b in range(batch):
        ref = O.gemv_int4(packed, scales, 128, rows, cols, tab, x[b * cols:(b + 1) * cols])
        assert max_rel(y[b], ref) <= GEMV_TOL, b
    t.free()


@pytest.mark.parametrize("batch", [1, 4])
def test_gemv_int8_14336x4096(be, batch):
    # workload: INT8 14336x4096, per-tensor f32 scale (the .pox INT8 layout), x fp16 N(0,1)
    rows, cols = 14336, 4096
    w = make_w(rows, cols, seed=9)
    q, s = Q.quantize_int8_symmetric(w)
    x = make_x(cols, batch, seed=10)
    if batch == 1:
        y = np.zeros(rows, np.float32)
        be.gemv_int8(q, s, rows, cols, x, y)
        ys = [y]
    else:
        t = be.upload_int8(q, s, rows, cols)
        ys = list(np.asarray(t.gemv_host(x, batch)).reshape(batch, rows))
        t.free()
    for b in range(batch):
        ref = O.gemv_int8(q, s, rows, cols, x[b * cols:(b + 1) * cols])
        assert max_rel(ys[b], ref) <= GEMV_TOL


@pytest.mark.parametrize("rows,cols", [(64, 4096), (1000, 256), (33, 100)])
def test_gemv_int8_shapes_and_dequant(be, rows, cols):
    w = make_w(rows, cols, seed=11)
    q, s = Q.quantize_int8_symmetric(w)
    x = make_x(cols, seed=12)
    t = be.upload_int8(q, s, rows, cols)
    y = t.gemv_host(x)
    assert max_rel(y, O.gemv_int8(q, s, rows, cols, x)) <= GEMV_TOL
    deq = t.dequant_host()
    assert np.array_equal(deq.view(np.uint32), O.dequantize_int8_symmetric(q, s).view(np.uint32))
    t.free()


@pytest.mark.parametrize("rows,cols", [(1000, 4096), (50, 96), (8, 100)])
def test_gemv_f16(be, rows, cols):
    rng = np.random.default_rng(13)
    wb = (rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)).astype(np.float16).view(np.uint16)
    x = rng.standard_normal(cols, dtype=np.float32)
    t = be.upload_f16(wb, rows, cols)
    y = t.gemv_host(x)
    assert max_rel(y, O.gemv_f16(wb, rows, cols, x)) <= GEMV_TOL
    t.free()


def test_outlier_table_semantics(be):
    # duplicates: the last entry for a slot wins (kernels.rs:213-217 applies in table order);
    # indices >= rows*cols never match a row and are ignored
    rows, cols, gs = 32, 256, 128
    packed, scales, _, _ = i4_case(rows, cols, gs, seed=21)
    idx = np.array([5, 300, 5, 999_999, 8191, 300], np.uint32)
    val = np.array([1.0, -2.0, 3.0, 9.0, 0.5, 4.0], np.float16).view(np.uint16)
    ob = Q.outliers_to_bytes(idx, val)
    x = make_x(cols, seed=22)
    y = np.zeros(rows, np.float32)
    be.gemv_int4_outliers(packed, scales, gs, rows, cols, ob, x, y)
    ref = O.gemv_int4(packed, scales, gs, rows, cols, (idx, val), x)
    assert max_rel(y, ref) <= GEMV_TOL
    t = be.upload_int4(packed, scales, rows, cols, gs, ob)
    assert t.outlier_count == 3
    deq = t.dequant_host()
    assert deq[5] == 3.0 and deq[300] == 4.0 and deq[8191] == 0.5
    t.free()


def test_layout_errors(be):
    rows, cols, gs = 16, 256, 128
    packed, scales, _, _ = i4_case(rows, cols, gs, seed=23)
    x = make_x(cols)
    y = np.full(rows, 7.0, np.float32)
    with pytest.raises(QuantizationError):  # metal_backend.rs:104-108
        be.gemv_int4(packed, scales[:-1], rows, cols, gs, x, y)
    with pytest.raises(QuantizationError):
        be.gemv_int4(packed[:-1], scales, rows, cols, gs, x, y)
    with pytest.raises(QuantizationError):  # x shorter than cols
        be.gemv_int4(packed, scales, rows, cols, gs, x[:-1], y)
    with pytest.raises(QuantizationError):  # outlier table whose count runs past the buffer
        bad = Q.outliers_to_bytes(np.array([1, 2], np.uint32), np.array([0, 0], np.uint16))[:-1]
        be.gemv_int4_outliers(packed, scales, gs, rows, cols, bad, x, y)
    be.gemv_int4(packed, scales, 0, cols, gs, x, y)  # rows == 0 -> Ok, nothing written
    assert np.all(y == 7.0)
    with pytest.raises(QuantizationError):
        be.gemv_int8(np.zeros(10, np.uint8), np.zeros(4, np.uint8), 4, 4, np.zeros(4, np.float32), y)


def test_registered_host_slices_reuse_resident_copy(be):
    rows, cols, gs = 512, 1024, 128
    packed, scales, _, _ = i4_case(rows, cols, gs, seed=24)
    t = be.upload_int4(packed, scales, rows, cols, gs)
    x = make_x(cols, seed=25)
    y = np.zeros(rows, np.float32)
    be.gemv_int4(t._keep[0], t._keep[1], rows, cols, gs, x, y)
    assert np.array_equal(y, t.gemv_host(x))
    assert max_rel(y, O.gemv_int4(packed, scales, gs, rows, cols, None, x)) <= GEMV_TOL
    t.free()


def test_host_slice_calls_replay_as_one_graph(be):
    """From the second host-slice call of a batch on, the x preparation and GEMV are replayed as one
    CUDA graph on the same staging buffers: every call's y must follow that call's x, across batch
    changes (a new batch is launched directly, then cached) and a larger x that regrows the staging."""
    rows, cols, gs = 1024, 2048, 128
    packed, scales, tab, ob = i4_case(rows, cols, gs, seed=31, hot_cols=6, policy="automatic")
    t = be.upload_int4(packed, scales, rows, cols, gs, ob)
    for i, batch in enumerate((1, 1, 1, 3, 3, 1, 8, 8, 1)):
        x = make_x(cols, batch, seed=40 + i)
        y = np.asarray(t.gemv_host(x, batch)).reshape(batch, rows)
        for b in range(batch):
            ref = O.gemv_int4(packed, scales, gs, rows, cols, tab, x[b * cols:(b + 1) * cols])
            assert max_rel(y[b], ref) <= GEMV_TOL, (i, batch, b)
    t.free()


def test_replayed_host_graph_reads_each_calls_x(be):
    """Host-slice calls from the second on replay one graph over the same mapped staging. Six calls
    in a row with a new x each, for INT4 (integer x preparation), INT8 and F16 (the f16 hi / lo
    preparation): every y must follow its own call's x, never the previous call's."""
    rows, cols = 512, 4096
    rng = np.random.default_rng(77)
    w = make_w(rows, cols, 78)
    packed, scales = Q.quantize_int4_group(w, 128)
    q8, s8 = Q.quantize_int8_symmetric(w)
    wb = w.astype(np.float16).view(np.uint16)
    cases = [(be.upload_int4(packed, scales, rows, cols, 128), lambda x: O.gemv_int4(packed, scales, 128, rows, cols, None, x)),
             (be.upload_int8(q8, s8, rows, cols), lambda x: O.gemv_int8(q8, s8, rows, cols, x)),
             (be.upload_f16(wb, rows, cols), lambda x: O.gemv_f16(wb, rows, cols, x))]
    for t, ref in cases:
        for i in range(6):
            x = rng.standard_normal(cols, dtype=np.float32) * np.float32(1 + i)
            assert max_rel(t.gemv_host(x), ref(x)) <= GEMV_TOL, (t, i)
        t.free()
