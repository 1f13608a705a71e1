"""Host checks of numeric arguments the kernels rely on (no GPU).

The tensor-core attention feeds q and the softmax weights p to f16 MMAs as two f16 terms,
hi = f16(x) and lo = f16(x - hi). The sum keeps about 22 significant bits of x for |x| >= 2^-4;
below that lo falls among f16's subnormals and the error stays under 2^-24 in absolute terms,
negligible next to the larger terms of the same dot product (|q| runs to tens, p to 1).
"""
import numpy as np


def split(x):
    hi = x.astype(np.float16)
    lo = (x - hi.astype(np.float32)).astype(np.float16)
    return hi, lo


def test_hi_lo_f16_error_bounds():
    rng = np.random.default_rng(0)
    # roped q values (|q| up to a few tens) and softmax weights (0 .. 1, down to e^-10)
    x = np.concatenate([rng.standard_normal(200_000).astype(np.float32) * np.float32(8.0),
                        np.exp(-rng.random(200_000) * 10).astype(np.float32)])
    hi, lo = split(x)
    err = np.abs(hi.astype(np.float64) + lo.astype(np.float64) - x.astype(np.float64))
    ax = np.abs(x.astype(np.float64))
    assert np.all(err <= np.maximum(ax * 2.0 ** -21, 2.0 ** -24))
    assert np.all(err[ax >= 2.0 ** -4] <= ax[ax >= 2.0 ** -4] * 2.0 ** -21)


def test_hi_alone_is_only_11_bits():
    # why the lo term is needed: f16 alone is off by up to 2^-11 relative
    x = np.float32(1.0) + np.arange(1, 1000, dtype=np.float32) * np.float32(2.0 ** -20)
    hi, _ = split(x)
    rel = np.abs(hi.astype(np.float64) - x) / x
    assert rel.max() > 2.0 ** -13
