"""Failure detection of the peer exchange on one GPU, without faulting it.

A two-rank allreduce whose second rank never arrives (its arrival flags are a buffer nothing
writes) must end by itself: the kernel's bounded arrival wait runs out, raises the context's
error flag and the sticky abort word, and returns. The host reads that status, and the same
context then serves a GEMV whose result matches the oracle.
"""
import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu


def test_missing_rank_times_out_and_context_stays_usable():
    be = CudaBackend.create(0)
    try:
        waited = be.check_missing_rank()
        assert 0.3 < waited < 20.0, waited  # about two seconds at the B200's clocks
        rng = np.random.default_rng(5)
        rows, cols = 256, 1024
        w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
        p, s = Q.quantize_int4_group(w, 128)
        t = be.upload_int4(p, s, rows, cols, 128)
        x = rng.standard_normal(cols, dtype=np.float32).astype(np.float16).astype(np.float32)
        y = t.gemv_host(x)
        ref = O.gemv_int4(p, s, 128, rows, cols, None, x)
        assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) <= 1e-3
        assert be.check_missing_rank() > 0.3  # a second check starts from a fresh abort word
        t.free()
    finally:
        be.close()
