"""The product's quantize-time tools (paraoxidizer_b200.quant) and paged bookkeeping against
the oracle and the reference's known answers. Bit-exact: packed nibbles, f16 scale/min bytes,
int8 bytes, outlier indices and values."""
import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200.paged import BlockManager, BlockTable, OutOfBlocks


@pytest.mark.parametrize("n,gs", [(512, 32), (512, 64), (4096, 128), (4096 + 37, 128), (1000, 256), (129, 128),
                                  (7, 4), (1, 128)])
def test_quantize_int4_bit_exact(n, gs):
    rng = np.random.default_rng(n * 7 + gs)
    w = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    p1, s1 = Q.quantize_int4_group(w, gs)
    p2, s2 = O.quantize_int4_group(w, gs)
    assert np.array_equal(p1, p2) and np.array_equal(s1, s2)


def test_quantize_int4_degenerate_and_special_groups():
    gs = 16
    w = np.zeros(16 * 8, np.float32)
    w[16:32] = 3.0                       # constant group: max = min + 1e-4
    w[32:48] = np.linspace(-1, 1, 16)
    w[40] = np.nan                       # NaN skipped by min/max, quantizes to 0
    w[48:64] = -0.0
    w[50] = 0.0                          # first of -0.0/+0.0 wins
    w[64:80] = np.float32(1e30)
    w[70] = np.inf
    w[80:96] = np.float32(0.5) * np.arange(16, dtype=np.float32)  # exact .5 ties
    p1, s1 = Q.quantize_int4_group(w, gs)
    p2, s2 = O.quantize_int4_group(w, gs)
    assert np.array_equal(p1, p2) and np.array_equal(s1, s2)


def test_quantize_int8_bit_exact():
    rng = np.random.default_rng(3)
    for w in (rng.standard_normal(100_000, dtype=np.float32) * np.float32(0.02),
              np.zeros(64, np.float32),
              np.array([0.5, -0.5, 1.5, -2.5, np.nan, 127.0], np.float32)):
        q1, s1 = Q.quantize_int8_symmetric(w)
        q2, s2 = O.quantize_int8_symmetric(w)
        assert np.array_equal(q1, q2) and np.array_equal(s1, s2)


@pytest.mark.parametrize("policy", ["automatic", "conservative", "aggressive"])
def test_extract_outliers_bit_exact(policy):
    rng = np.random.default_rng(5)
    rows, cols = 64, 1024
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    hot = rng.choice(cols, 8, replace=False)
    w.reshape(rows, cols)[:, hot] *= np.float32(20.0)
    a, b = w.copy(), w.copy()
    t1 = Q.extract_and_zero_outliers(a, policy)
    t2 = O.extract_and_zero_outliers(b, policy)
    assert t1 is not None and t2 is not None
    assert np.array_equal(t1[0], t2[0]) and np.array_equal(t1[1], t2[1])
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert np.array_equal(Q.outliers_to_bytes(*t1), O.outliers_to_bytes(*t2))


def test_extract_outliers_kat_and_none():
    # tests/test_quant_and_security.rs:70-95 on the product side
    w = (np.sin(np.arange(200, dtype=np.float32) * np.float32(0.1)) * np.float32(0.2)).astype(np.float32)
    w[50], w[120] = 15.0, -18.0
    idx, _ = Q.extract_and_zero_outliers(w, "automatic")
    assert list(idx) == [50, 120] and w[50] == 0 and w[120] == 0
    assert Q.extract_and_zero_outliers(np.ones(10, np.float32), "automatic") is None
    assert Q.extract_and_zero_outliers(np.ones(10, np.float32), "disabled") is None


def test_paged_block_table_kat():
    # crates/paraoxidizer-runtime/src/paged_cache.rs:223-250
    m = BlockManager(total_blocks=4, block_size=16)
    t = BlockTable(16)
    for _ in range(20):
        t.append_token(m)
    assert len(t.allocated_block_ids) == 2 and t.sequence_len == 20
    assert m.available_blocks() == 2
    t.free(m)
    assert t.sequence_len == 0 and m.available_blocks() == 4


def test_paged_out_of_blocks():
    m = BlockManager(total_blocks=1, block_size=16)
    t = BlockTable(16)
    for _ in range(16):
        t.append_token(m)
    with pytest.raises(OutOfBlocks):
        t.append_token(m)
