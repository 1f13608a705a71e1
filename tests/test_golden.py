"""The committed fixtures of tests/golden/ (made by tests/golden/make_golden.py from the oracle)
recomputed on the CPU: the oracle must still produce them, and the product's host quantizer must
produce the same packed nibbles, scales, int8 bytes and outlier table from the same weights.
Arithmetic without libm calls (quantization, GEMVs) is compared bit for bit; attention and
forward_token, which call expf / cosf / sinf / powf, within 1e-6 of max |value|."""
import os

import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200.synth import make_llama, oracle_weights

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def g():
    import sys

    sys.path.insert(0, os.path.join(HERE, "golden"))
    import make_golden

    with np.load(os.path.join(HERE, "golden", "oracle_vectors.npz")) as z:
        d = {k: z[k] for k in z.files}
    d["_mod"] = make_golden
    return d


def same_bits(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.dtype == b.dtype and a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def close(a, b, tol=1e-6):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return a.shape == b.shape and float(np.max(np.abs(a - b))) <= tol * float(np.max(np.abs(b)))


def test_quantizers_reproduce_the_fixtures(g):
    assert g["i4_idx"].size >= 12  # the fixture's weights carry outliers
    w = g["i4_w"].copy()
    idx, val = O.extract_and_zero_outliers(w, "automatic")
    assert same_bits(idx, g["i4_idx"]) and same_bits(val, g["i4_val"])
    p, s = O.quantize_int4_group(w, 64)
    assert same_bits(p, g["i4_packed"]) and same_bits(s, g["i4_scales"])
    wq = g["i4_w"].copy()
    tq = Q.extract_and_zero_outliers(wq, "automatic")
    pq, sq = Q.quantize_int4_group(wq, 64)
    assert same_bits(tq[0].astype(g["i4_idx"].dtype), g["i4_idx"]) and same_bits(tq[1], g["i4_val"])
    assert same_bits(pq, g["i4_packed"]) and same_bits(sq, g["i4_scales"])
    q8, s8 = Q.quantize_int8_symmetric(g["i8_w"])
    assert same_bits(q8, g["i8_q"]) and same_bits(s8, g["i8_scale"])


def test_gemvs_reproduce_the_fixtures(g):
    y4 = O.gemv_int4(g["i4_packed"], g["i4_scales"], 64, 64, 256, (g["i4_idx"], g["i4_val"]), g["i4_x"])
    assert same_bits(y4, g["i4_y"])
    assert same_bits(O.gemv_int8(g["i8_q"], g["i8_scale"], 48, 200, g["i8_x"]), g["i8_y"])
    assert same_bits(O.gemv_f16(g["f16_w"], 40, 96, g["f16_x"]), g["f16_y"])


def test_attention_and_forward_reproduce_the_fixtures(g):
    assert close(O.attention(g["att_q"], g["att_k"], g["att_v"], 8, 2, 64, 40), g["att_out"])
    mg = g["_mod"]
    m = O.OracleModel(mg.FORWARD_CFG, oracle_weights(make_llama(mg.FORWARD_CFG, seed=mg.FORWARD_SEED,
                                                                outlier_policy="automatic", norm_jitter=0.1)), 16)
    got = np.stack([m.forward_token(t, i) for i, t in enumerate(mg.FORWARD_TOKENS)])
    assert close(got, g["fwd_logits"])
    assert [int(np.argmax(r)) for r in got] == [int(np.argmax(r)) for r in g["fwd_logits"]]
