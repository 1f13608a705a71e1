"""The oracle's decode primitives against independent float64 restatements of the same
mathematics (CPU). The reference ships no golden vectors for these, so this pins the oracle's C
code to the formulas of engine.rs it cites, within float32 rounding:

* GQA attention (engine.rs:580-641): softmax(q k / sqrt(d)) v over positions 0..=pos, query head
  h reading kv head h / (heads per kv head);
* RoPE on interleaved pairs (engine.rs:353-408), angle pos / theta^(2i/d) formed in f32 as the
  reference forms it;
* RMSNorm with an f16 weight (engine.rs:294-350) and SwiGLU (engine.rs:671-677).
"""
import numpy as np
import pytest

from oracle import oracle as O


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


@pytest.mark.parametrize("nq,nkv,hd,pos", [(32, 8, 128, 0), (32, 8, 128, 700), (8, 8, 64, 33), (64, 8, 128, 129),
                                           (4, 1, 32, 5)])
def test_attention_matches_float64_softmax(nq, nkv, hd, pos):
    rng = np.random.default_rng(nq * 1000 + pos)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    kc = rng.standard_normal((pos + 1) * nkv * hd).astype(np.float32)
    vc = rng.standard_normal((pos + 1) * nkv * hd).astype(np.float32)
    got = O.attention(q, kc, vc, nq, nkv, hd, pos)
    G = nq // nkv
    k = kc.astype(np.float64).reshape(pos + 1, nkv, hd)
    v = vc.astype(np.float64).reshape(pos + 1, nkv, hd)
    ref = np.zeros((nq, hd))
    for h in range(nq):
        s = k[:, h // G, :] @ q[h * hd:(h + 1) * hd].astype(np.float64) / np.sqrt(hd)
        p = np.exp(s - s.max())
        ref[h] = (p / p.sum()) @ v[:, h // G, :]
    assert rel(got, ref.ravel()) <= 2e-6


@pytest.mark.parametrize("pos", [0, 1, 17, 63])
@pytest.mark.parametrize("hd,theta", [(128, 500000.0), (64, 10000.0)])
def test_rope_matches_rotation(pos, hd, theta):
    nq, nkv = 4, 2
    rng = np.random.default_rng(pos + hd)
    q = rng.standard_normal(nq * hd).astype(np.float32)
    k = rng.standard_normal(nkv * hd).astype(np.float32)
    gq, gk = O.rope(q, k, nq, nkv, hd, pos, theta)
    i = np.arange(hd // 2)
    freq = np.float32(1.0) / np.power(np.float32(theta), (2 * i).astype(np.float32) / np.float32(hd))
    ang = (np.float32(pos) * freq.astype(np.float32)).astype(np.float64)
    c, s = np.cos(ang), np.sin(ang)

    def rot(v, n):
        v = v.astype(np.float64).reshape(n, hd // 2, 2)
        out = np.empty_like(v)
        out[..., 0] = v[..., 0] * c - v[..., 1] * s
        out[..., 1] = v[..., 0] * s + v[..., 1] * c
        return out.ravel()

    # numpy's f32 power and the C library's powf may differ by an ulp of the frequency (<= 1):
    # that moves the angle by up to pos x 1.2e-7 rad
    tol = 2e-6 + pos * 1.2e-7
    assert rel(gq, rot(q, nq)) <= tol and rel(gk, rot(k, nkv)) <= tol
    if pos == 0:
        assert np.array_equal(gq, q) and np.array_equal(gk, k)


def test_rms_norm_and_swiglu_match_float64():
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(4096) * 3).astype(np.float32)
    wb = (1 + 0.1 * rng.standard_normal(4096)).astype(np.float16).view(np.uint16)
    got = O.rms_norm(x, wb, 1e-5)
    xd = x.astype(np.float64)
    ref = xd / np.sqrt(np.mean(xd * xd) + 1e-5) * wb.view(np.float16).astype(np.float64)
    assert rel(got, ref) <= 2e-6
    assert rel(O.rms_norm(x, None, 1e-5), xd / np.sqrt(np.mean(xd * xd) + 1e-5)) <= 2e-6
    g = np.concatenate([rng.standard_normal(1000) * 4, [-100.0, -30.0, 0.0, 30.0]]).astype(np.float32)
    u = rng.standard_normal(g.size).astype(np.float32)
    gd = g.astype(np.float64)
    assert rel(O.swiglu(g, u), gd / (1 + np.exp(-gd)) * u.astype(np.float64)) <= 2e-6


@pytest.mark.parametrize("rows,cols", [(64, 4096), (33, 100)])
def test_gemv_int8_and_f16_match_float64(rows, cols):
    # kernels.rs:229-255 (INT8: q * scale per element, f32 dot) and engine.rs:235-250 (F16 rows)
    rng = np.random.default_rng(rows + cols)
    w = rng.standard_normal(rows * cols).astype(np.float32) * np.float32(0.02)
    x = rng.standard_normal(cols).astype(np.float32)
    q, s = O.quantize_int8_symmetric(w)
    wq = O.dequantize_int8_symmetric(q, s).astype(np.float64).reshape(rows, cols)
    # f32 sums of up to 4096 products: a few 1e-6 of max |y| (measured 2.2e-6 at 4096)
    assert rel(O.gemv_int8(q, s, rows, cols, x), wq @ x.astype(np.float64)) <= 1e-5
    wb = w.astype(np.float16).view(np.uint16)
    ref = wb.view(np.float16).astype(np.float64).reshape(rows, cols) @ x.astype(np.float64)
    assert rel(O.gemv_f16(wb, rows, cols, x), ref) <= 1e-5
