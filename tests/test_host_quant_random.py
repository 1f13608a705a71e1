"""Randomized agreement of the product's quantize-time tools (paraoxidizer_b200.quant, numpy)
with the oracle's C restatement of the same reference functions, bit for bit:
quantize_int4_group (kernels.rs:26-82), quantize_int8_symmetric (kernels.rs:131-154) and
extract_and_zero_outliers (outlier.rs:57-85). Inputs mix the cases the reference's loops treat
specially: exact .5 ties, +0 / -0, subnormals, values near the f16 range, NaN and +-inf."""
import warnings

import numpy as np
from hypothesis import given, settings, strategies as st

from oracle import oracle as O
from paraoxidizer_b200 import quant as Q

SPECIAL = np.array([0.0, -0.0, 0.5, -0.5, 1.5, -2.5, 1e-40, -1e-40, 6.0e4, -6.0e4, 1e30, np.nan, np.inf, -np.inf],
                   np.float32)


def draw_weights(seed: int, n: int, mode: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if mode == 0:  # the path's weights
        w = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    elif mode == 1:  # few distinct values: ties everywhere
        w = rng.integers(-3, 4, n).astype(np.float32) * np.float32(0.25)
    elif mode == 2:  # wide dynamic range
        w = (rng.standard_normal(n) * 10.0 ** rng.integers(-30, 30, n)).astype(np.float32)
    else:  # the path's weights with special values sprinkled in
        w = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
        k = max(1, n // 16)
        w[rng.integers(0, n, k)] = SPECIAL[rng.integers(0, SPECIAL.size, k)]
    return np.ascontiguousarray(w, np.float32)


@settings(max_examples=150, deadline=None)
@given(seed=st.integers(0, 2**31 - 1), n=st.integers(1, 3000), gs=st.sampled_from([2, 4, 32, 64, 128, 256]),
       mode=st.integers(0, 3))
def test_int4_group_quantizer_agrees(seed, n, gs, mode):
    w = draw_weights(seed, n, mode)
    p1, s1 = Q.quantize_int4_group(w, gs)
    p2, s2 = O.quantize_int4_group(w, gs)
    assert np.array_equal(p1, p2) and np.array_equal(s1, s2)


@settings(max_examples=150, deadline=None)
@given(seed=st.integers(0, 2**31 - 1), n=st.integers(1, 3000), mode=st.integers(0, 3))
def test_int8_symmetric_quantizer_agrees(seed, n, mode):
    w = draw_weights(seed, n, mode)
    q1, s1 = Q.quantize_int8_symmetric(w)
    q2, s2 = O.quantize_int8_symmetric(w)
    assert np.array_equal(q1, q2) and np.array_equal(s1, s2)


@settings(max_examples=100, deadline=None)
@given(seed=st.integers(0, 2**31 - 1), n=st.integers(2, 3000), mode=st.integers(0, 3),
       policy=st.sampled_from(["automatic", "conservative", "aggressive"]), hot=st.integers(0, 8))
def test_outlier_extraction_agrees(seed, n, mode, policy, hot):
    # with inf / NaN in the tensor (mode 3) or a variance that overflows (mode 2) the mean and
    # threshold stop being finite; both sides must still select and zero the same entries
    w = draw_weights(seed, n, mode)
    if hot:
        rng = np.random.default_rng(seed + 1)
        w[rng.integers(0, n, hot)] *= np.float32(50.0)
    a, b = w.copy(), w.copy()
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", RuntimeWarning)  # f32 overflow is part of the reference's arithmetic
        t1 = Q.extract_and_zero_outliers(a, policy)
    t2 = O.extract_and_zero_outliers(b, policy)
    assert (t1 is None) == (t2 is None)
    if t1 is not None:
        assert np.array_equal(t1[0], t2[0]) and np.array_equal(t1[1], t2[1])
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
