"""Pins the oracle (oracle/pox_oracle.c) against the reference's own known-answer tests.

The reference holds no golden output vectors; its hot-path tests are tolerance and exact-index
assertions on deterministic inputs. Each test below restates one of them on the same input
formula and asserts the same bound, so the oracle is pinned to everything the reference's
tests pin.
"""
import numpy as np
import pytest

from oracle import oracle as O


def test_int4_group_roundtrip_kat():
    # tests/test_quant_and_security.rs:14-44
    w = (np.sin(np.arange(512, dtype=np.float32) * np.float32(0.05)) * np.float32(2.5)).astype(np.float32)
    for gs in (32, 64, 128, 256):
        packed, scales = O.quantize_int4_group(w, gs)
        assert packed.size == (w.size + 1) // 2
        deq = O.dequantize_int4_group(packed, scales, gs, w.size)
        assert np.max(np.abs(w - deq)) < 0.25, gs


def test_int8_roundtrip_kat():
    # tests/test_quant_and_security.rs:47-67
    w = (np.cos(np.arange(256, dtype=np.float32) * np.float32(0.1)) * np.float32(1.8)).astype(np.float32)
    q, s = O.quantize_int8_symmetric(w)
    deq = O.dequantize_int8_symmetric(q, s)
    assert np.max(np.abs(w - deq)) < 0.03


def test_outlier_extraction_kat():
    # tests/test_quant_and_security.rs:70-95
    w = (np.sin(np.arange(200, dtype=np.float32) * np.float32(0.1)) * np.float32(0.2)).astype(np.float32)
    w[50] = 15.0
    w[120] = -18.0
    orig = w.copy()
    t = O.extract_and_zero_outliers(w, "automatic")
    assert t is not None
    idx, val = t
    assert list(idx) == [50, 120]
    assert w[50] == 0.0 and w[120] == 0.0
    b = O.outliers_to_bytes(idx, val)
    assert b.size == 4 + 6 * 2
    idx2, val2 = O.outliers_from_bytes(b)
    assert len(idx2) == 2
    O.outliers_apply(idx2, val2, w)
    assert abs(w[50] - orig[50]) < 0.01 and abs(w[120] - orig[120]) < 0.01


def test_outlier_policy_names():
    # outlier.rs:17-34
    assert O.sigma_for_policy("conservative") == 4.5
    assert O.sigma_for_policy("Automatic") == 3.5
    assert O.sigma_for_policy("aggressive") == 2.8
    assert O.sigma_for_policy("3.5") == 3.5
    assert O.sigma_for_policy("none") is None


def test_outlier_from_bytes_edges():
    # outlier.rs:112-127: < 4 bytes -> empty, truncated count -> Err
    assert len(O.outliers_from_bytes(np.zeros(3, np.uint8))[0]) == 0
    bad = np.zeros(10, np.uint8)
    bad[0] = 2  # claims 2 entries = 16 bytes
    with pytest.raises(ValueError):
        O.outliers_from_bytes(bad)


def test_dot_product_kat():
    # tests/test_quant_and_security.rs:98-111
    a = (np.arange(128, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    b = np.cos(np.arange(128, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    scalar = np.float32(0)
    for x, y in zip(a, b):
        scalar = np.float32(scalar + np.float32(x * y))
    assert abs(O.dot_product_simd(a, b) - scalar) < 1e-4
    assert abs(O.dot_product_simd(a, b, neon=True) - scalar) < 1e-4


def _degradation_weights(rows=512, cols=256):
    # tests/test_model_degradation.rs:67-82 (computed in f64 then cast, as the reference)
    i = np.arange(rows * cols, dtype=np.float64)
    u1 = np.minimum(np.abs(np.sin(i * 31415.92)) * 0.999 + 0.0001, 0.9999)
    u2 = np.minimum(np.abs(np.cos(i * 27182.81)) * 0.999 + 0.0001, 0.9999)
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    w = (z * 0.04).astype(np.float32)
    w[::1500] *= np.float32(3.5)
    return w


def _metrics(o, r):
    o = o.astype(np.float64)
    r = r.astype(np.float64)
    err = np.abs(o - r)
    cos = np.dot(o, r) / (np.linalg.norm(o) * np.linalg.norm(r))
    sqnr = 10 * np.log10(np.sum(o * o) / np.sum(err * err))
    return cos, sqnr


def test_layer_degradation_bounds():
    # tests/test_model_degradation.rs:61-345: weight cosine >= 0.995, SQNR >= 20 dB,
    # activation MSE < 1e-3 for INT8, INT4-g128 and INT4-g128 + outliers.
    rows, cols = 512, 256
    w = _degradation_weights(rows, cols)
    t = np.arange(64 * cols, dtype=np.float32)
    acts = (np.sin(t * np.float32(0.37)) * np.float32(0.5) + np.cos(t * np.float32(0.11)) * np.float32(0.2)).astype(np.float32).reshape(64, cols)
    base = acts @ w.reshape(rows, cols).T
    q, s = O.quantize_int8_symmetric(w)
    d8 = O.dequantize_int8_symmetric(q, s)
    p, sc = O.quantize_int4_group(w, 128)
    d4 = O.dequantize_int4_group(p, sc, 128, w.size)
    wz = w.copy()
    tab = O.extract_and_zero_outliers(wz, "automatic")
    p2, sc2 = O.quantize_int4_group(wz, 128)
    d4o = O.dequantize_int4_group(p2, sc2, 128, w.size)
    if tab is not None:
        O.outliers_apply(tab[0], tab[1], d4o)
    for d in (d8, d4, d4o):
        cos, sqnr = _metrics(w, d)
        assert cos >= 0.995 and sqnr >= 20.0
        y = acts @ d.reshape(rows, cols).T
        assert np.mean((y - base) ** 2) < 1e-3


def test_f16_conversion_matches_ieee():
    # half 2.7.1 f16::from_f32 is IEEE round-to-nearest-even; numpy's float16 cast is an
    # independent IEEE implementation. Edge cases plus 2M random bit patterns.
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 2**32, size=2_000_000, dtype=np.uint64).astype(np.uint32)
    edge = np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x477FE000, 0x477FF000, 0x477FEFFF,
                     0x33000000, 0x33000001, 0x32FFFFFF, 0x38800000, 0x387FFFFF, 0x33800000,
                     0x3F800000, 0x3F801000, 0x3F803000, 0x00000001, 0x00800000], np.uint32)
    bits = np.concatenate([edge, bits])
    f = bits.view(np.float32)
    finite = np.isfinite(f)
    with np.errstate(over="ignore"):
        ref = f[finite].astype(np.float16).view(np.uint16)
    got = O.f32_to_f16_bits(f[finite])
    assert np.array_equal(got, ref)
    # NaN stays NaN (quiet), inf stays inf
    nan_bits = O.f32_to_f16_bits(np.array([np.nan, np.inf, -np.inf], np.float32))
    assert (nan_bits[0] & 0x7C00) == 0x7C00 and (nan_bits[0] & 0x3FF) != 0
    assert nan_bits[1] == 0x7C00 and nan_bits[2] == 0xFC00
    # f16 -> f32 is exact for all 65536 patterns
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    back = O.f16_bits_to_f32(allh)
    ref32 = allh.view(np.float16).astype(np.float32)
    ok = ~np.isnan(ref32)
    assert np.array_equal(back[ok].view(np.uint32), ref32[ok].view(np.uint32))
    assert np.all(np.isnan(back[~ok]))


def test_gemv_int4_matches_dequant_dot():
    # kernels.rs:177-226: y[r] = dot_product_simd(dequant(row) with outliers replaced, x)
    rng = np.random.default_rng(1)
    rows, cols, gs = 24, 256, 64
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    w[rng.choice(rows * cols, 10, replace=False)] = np.float32(1.5)
    tab = O.extract_and_zero_outliers(w, "automatic")
    assert tab is not None and len(tab[0]) >= 10
    p, s = O.quantize_int4_group(w, gs)
    x = rng.standard_normal(cols, dtype=np.float32)
    y = O.gemv_int4(p, s, gs, rows, cols, tab, x)
    d = O.dequantize_int4_group(p, s, gs, rows * cols)
    O.outliers_apply(tab[0], tab[1], d)
    for r in range(rows):
        assert y[r] == np.float32(O.dot_product_simd(d[r * cols:(r + 1) * cols], x))


def metal_test_case():
    """Inputs of the reference's own GEMV backend test (metal_backend.rs:226-246): 32 x 64 weights
    sin(0.05 i), x = cos(0.1 i), INT4 groups of 32."""
    rows, cols, gs = 32, 64, 32
    w = np.sin(np.arange(rows * cols, dtype=np.float32) * np.float32(0.05)).astype(np.float32)
    x = np.cos(np.arange(cols, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    return rows, cols, gs, w, x


def test_metal_backend_case_kat():
    # metal_backend.rs:226-246: quantize_int4_group(&weights, 32), gemv_int4, then "sum |y| > 0.01"
    rows, cols, gs, w, x = metal_test_case()
    p, s = O.quantize_int4_group(w, gs)
    y = O.gemv_int4(p, s, gs, rows, cols, None, x)
    assert float(np.sum(np.abs(y))) > 0.01
    d = O.dequantize_int4_group(p, s, gs, rows * cols)
    for r in range(rows):
        assert y[r] == np.float32(O.dot_product_simd(d[r * cols:(r + 1) * cols], x))
