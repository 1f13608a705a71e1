"""GPU outlier extraction (pox_cuda_extract_outliers) against the oracle's restatement of
SparseOutlierTable::extract_and_zero_outliers (crates/paraoxidizer-quant/src/outlier.rs:57-85).

Bar: bit-exact -- the same .pox table bytes (indices, f16 values, order) and the same zeroed weights,
bit for bit, on the benchmark's 4096x14336 matrix with 0.5% of its input channels x20 (the 3.5-sigma
"Automatic" policy), the reference's own spike test, lengths that are not multiples of the kernels'
chunks, the other policies, inputs with no outlier and NaN.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import _lib as L
from paraoxidizer_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    b = CudaBackend.create(0)
    yield b
    b.close()


def gpu_extract(be, w, sigma):
    import torch

    wd = torch.from_numpy(w.copy()).cuda()
    torch.cuda.synchronize()
    n = C.c_size_t(0)
    cap = 4 + 6 * w.size
    buf = np.zeros(cap, np.uint8)
    L.check(L.lib().pox_cuda_extract_outliers(be.ctx, wd.data_ptr(), w.size, np.float32(sigma), buf.ctypes.data, cap,
                                              C.byref(n)))
    return (buf[:n.value] if n.value else None), wd.cpu().numpy()


def oracle_extract(w, policy):
    ref = w.copy()
    tab = O.extract_and_zero_outliers(ref, policy)
    return (None if tab is None else O.outliers_to_bytes(*tab)), ref


def check(be, w, policy):
    sigma = O.sigma_for_policy(policy)
    got_tab, got_w = gpu_extract(be, w, sigma)
    ref_tab, ref_w = oracle_extract(w, policy)
    if ref_tab is None:
        assert got_tab is None
    else:
        assert got_tab is not None and np.array_equal(got_tab, ref_tab)
    assert np.array_equal(got_w.view(np.uint32), ref_w.view(np.uint32))
    return 0 if ref_tab is None else int(ref_tab[:4].view(np.uint32)[0])


def test_benchmark_matrix_automatic(be):
    rng = np.random.default_rng(0)
    rows, cols = 4096, 14336
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    w.reshape(rows, cols)[:, rng.choice(cols, 72, replace=False)] *= np.float32(20.0)
    n = check(be, w, "automatic")
    assert 150_000 < n < 300_000


@pytest.mark.parametrize("policy", ["conservative", "automatic", "aggressive"])
@pytest.mark.parametrize("n", [1, 3, 1023, 1025, 4096, 4097, 100_003])
def test_lengths_and_policies(be, policy, n):
    rng = np.random.default_rng(n)
    w = rng.standard_normal(n, dtype=np.float32) * np.float32(0.05)
    w[rng.integers(0, n, max(1, n // 500))] *= np.float32(30.0)
    check(be, w, policy)


def test_reference_spike_case(be):
    # test_quant_and_security.rs:70-95: sin-shaped weights with spikes at 50 and 120 -> exactly those two
    w = (np.sin(np.arange(512, dtype=np.float32) * np.float32(0.05)) * np.float32(0.1)).astype(np.float32)
    w[50], w[120] = 10.0, -12.0
    tab, _ = gpu_extract(be, w, O.sigma_for_policy("automatic"))
    assert int(tab[:4].view(np.uint32)[0]) == 2
    assert list(tab[4:12].view(np.uint32)) == [50, 120]
    check(be, w, "automatic")


def test_no_outliers_nan_and_small_buffer(be):
    import torch

    check(be, np.full(5000, 0.25, np.float32), "automatic")   # std 0: strict > finds nothing -> None
    w = np.random.default_rng(1).standard_normal(3000).astype(np.float32)
    w[17] = np.nan                                            # NaN sum: every comparison false -> None
    check(be, w, "automatic")
    n = C.c_size_t(7)
    assert L.lib().pox_cuda_extract_outliers(be.ctx, None, 0, np.float32(3.5), None, 0, C.byref(n)) == L.POX_OK
    assert n.value == 0
    # a buffer too small: POX_ERR_LAYOUT with the size, the weights untouched
    w = np.random.default_rng(2).standard_normal(10000).astype(np.float32)
    w[::97] *= 50
    wd = torch.from_numpy(w.copy()).cuda()
    torch.cuda.synchronize()
    buf = np.zeros(8, np.uint8)
    rc = L.lib().pox_cuda_extract_outliers(be.ctx, wd.data_ptr(), w.size, np.float32(3.5), buf.ctypes.data, 8,
                                           C.byref(n))
    assert rc == L.POX_ERR_LAYOUT and n.value > 8
    assert np.array_equal(wd.cpu().numpy().view(np.uint32), w.view(np.uint32))
