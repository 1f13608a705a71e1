"""paraoxidizer_b200: B200-native (sm_100a) CUDA backend for ParaOxidizer's decode hot path.

The compute lives in libpox_cuda.so (hand-written CUDA behind the C ABI of
include/pox_cuda.h); this package is its host-side mirror of the reference's runtime
interfaces (MetalBackend, quant::gemv_*, PagedKvCache, PoxEngine::forward_token).
"""
from ._lib import PoxError, QuantizationError, RuntimeBackendError, POX_F16, POX_I4, POX_I8  # noqa: F401

__version__ = "0.1.0"


def backend(device: int = 0):
    """CudaBackend.new(device): None when no usable B200 is present."""
    from .backend import CudaBackend

    return CudaBackend.new(device)
