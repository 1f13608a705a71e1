"""GPU quantizer (pox_cuda_quantize_int4) bit-exact with quantize_int4_group
(crates/paraoxidizer-quant/src/kernels.rs:26-82), and uploads from device payloads equal uploads
from host payloads."""
import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import _lib as L
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    b = CudaBackend.create(0)
    yield b
    b.close()


def gpu_quantize(be, w, gs):
    import torch

    wd = torch.from_numpy(np.ascontiguousarray(w, np.float32)).cuda()
    pd = torch.zeros(w.size // 2, dtype=torch.uint8, device="cuda")
    sd = torch.zeros(w.size // gs * 4, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    L.check(L.lib().pox_cuda_quantize_int4(be.ctx, wd.data_ptr(), w.size, gs, pd.data_ptr(), sd.data_ptr(), None))
    be.synchronize()
    return pd.cpu().numpy(), sd.cpu().numpy()


@pytest.mark.parametrize("gs", [32, 64, 128, 256])
def test_quantizer_bit_exact(be, gs):
    rng = np.random.default_rng(gs)
    n = gs * 997
    w = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    g = w.reshape(-1, gs)
    g[0] = 0.0                        # constant group: max = min + 1e-4 (kernels.rs:50-52)
    g[1] = 0.0
    g[1, ::2] = -0.0                  # +0 / -0 ties: the first of equal values is kept
    g[2] = np.float32(3.0)
    g[3, 5] = np.float32(np.nan)      # NaN is skipped by min / max and quantizes to 0
    g[4, :] = np.float32(1e-9) * np.arange(gs, dtype=np.float32)  # range below 1e-8
    g[5, 7] = np.float32(70000.0)     # one large value: coarse scale
    g[6] = rng.standard_normal(gs).astype(np.float32) * np.float32(1e4)
    ref_p, ref_s = Q.quantize_int4_group(w, gs)
    orc_p, orc_s = O.quantize_int4_group(w, gs)
    assert np.array_equal(ref_p, orc_p) and np.array_equal(ref_s, orc_s)
    p, s = gpu_quantize(be, w, gs)
    assert np.array_equal(p, ref_p)
    bad = np.nonzero((s.view(np.uint32) != ref_s.view(np.uint32)))[0]
    detail = [(int(i), hex(int(s.view(np.uint32)[i])), hex(int(ref_s.view(np.uint32)[i]))) for i in bad[:8]]
    assert bad.size == 0, (bad.size, detail)


def test_upload_from_device_payload(be):
    import torch

    rng = np.random.default_rng(3)
    rows, cols = 512, 2048
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    p, s = Q.quantize_int4_group(w, 128)
    th = be.upload_int4(p, s, rows, cols, 128)
    pd, sd = torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda()
    torch.cuda.synchronize()
    desc = L.TensorDesc()
    desc.dtype, desc.rows, desc.cols, desc.group_size = L.POX_I4, rows, cols, 128
    desc.data, desc.data_len, desc.scales, desc.scale_len = pd.data_ptr(), p.size, sd.data_ptr(), s.size
    import ctypes as C

    h = C.c_void_p()
    L.check(L.lib().pox_cuda_tensor_upload(be.ctx, C.byref(desc), C.byref(h)))
    x = rng.standard_normal(cols, dtype=np.float32)
    y_host = th.gemv_host(x)
    y_dev = np.zeros(rows, np.float32)
    L.check(L.lib().pox_cuda_tensor_gemv_host(be.ctx, h.value, x.ctypes.data, 1, y_dev.ctypes.data))
    assert np.array_equal(y_host, y_dev)
    L.check(L.lib().pox_cuda_tensor_free(be.ctx, h.value))
    th.free()
