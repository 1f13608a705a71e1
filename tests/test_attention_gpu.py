"""Kernel-level parity of the paged decode attention (pox_cuda_paged_attention) against the oracle.

Reference: the attention of PoxEngine::forward_token (crates/paraoxidizer-runtime/src/engine.rs:
580-641) over a contiguous f32 KvCache; the CUDA kernels read fp16 pages of 16 tokens through a
block table (crates/paraoxidizer-runtime/src/paged_cache.rs:149-162). The oracle runs on the same
K/V values (the f16 pages converted exactly to f32), so the comparison isolates the attention
arithmetic. Bar: max |out - ref| / max |ref| <= 1e-3 per batch row (fp32 accumulate).

Block tables are scattered and out of order: sequence b's pages are a random permutation drawn
from the whole pool, so consecutive positions live in unrelated pages.
"""
import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import _lib as L
from paraoxidizer_b200.backend import CudaBackend

pytestmark = pytest.mark.gpu

ATTN_TOL = 1e-3
PAGE = 16


def max_rel(y, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(np.asarray(y, np.float64) - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


@pytest.fixture(scope="module")
def be():
    b = CudaBackend.create(0)
    yield b
    b.close()


def _case(rng, contexts, heads, kv_heads, hd, extra_blocks=3):
    """Random q, K/V pages with scattered block tables; returns host arrays and the oracle output."""
    B = len(contexts)
    mbps = max((c + PAGE - 1) // PAGE for c in contexts) + 1
    need = sum((c + PAGE - 1) // PAGE for c in contexts)
    nblk = need + extra_blocks
    perm = rng.permutation(nblk)
    tab = np.full((B, mbps), -1, np.int32)
    o = 0
    for b, c in enumerate(contexts):
        n = (c + PAGE - 1) // PAGE
        tab[b, :n] = perm[o:o + n]
        o += n
    # K/V values: N(0, 1) keys and values, stored as f16 (pages hold garbage beyond each context)
    kp = rng.standard_normal((nblk, kv_heads, PAGE, hd), dtype=np.float32).astype(np.float16)
    vp = rng.standard_normal((nblk, kv_heads, PAGE, hd), dtype=np.float32).astype(np.float16)
    q = (rng.standard_normal((B, heads, hd), dtype=np.float32) * np.float32(1.5)).astype(np.float32)
    pos = np.array([c - 1 for c in contexts], np.uint32)
    ref = np.zeros((B, heads, hd), np.float32)
    for b, c in enumerate(contexts):
        # contiguous f32 cache [t][kv_head][hd] of this sequence, as the reference's KvCache holds it
        kc = np.stack([kp[tab[b, t // PAGE], :, t % PAGE, :] for t in range(c)]).astype(np.float32)
        vc = np.stack([vp[tab[b, t // PAGE], :, t % PAGE, :] for t in range(c)]).astype(np.float32)
        ref[b] = O.attention(q[b].reshape(-1), kc.reshape(-1), vc.reshape(-1), heads, kv_heads, hd,
                             c - 1).reshape(heads, hd)
    return q, kp, vp, tab, pos, nblk, mbps, ref


def _run(be, q, kp, vp, tab, pos, heads, kv_heads, hd, nblk, mbps):
    import torch

    dev = torch.device("cuda", 0)
    qd = torch.from_numpy(q).to(dev)
    kd = torch.from_numpy(np.ascontiguousarray(kp).view(np.int16)).to(dev)
    vd = torch.from_numpy(np.ascontiguousarray(vp).view(np.int16)).to(dev)
    td = torch.from_numpy(tab).to(dev)
    pd = torch.from_numpy(pos.view(np.int32)).to(dev)
    out = torch.full(q.shape, float("nan"), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()  # the library's stream does not order against torch's
    rc = L.lib().pox_cuda_paged_attention(be.ctx, qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), td.data_ptr(),
                                          pd.data_ptr(), q.shape[0], heads, kv_heads, hd, nblk, mbps,
                                          out.data_ptr(), None)
    return rc, out


# (contexts per batch row, heads, kv_heads, head_dim): G = 4 and 8 query heads per kv head of 128
# (the tensor-core kernel), G = 2 (the FMA kernel), head_dim 64; contexts 1, 17, 640 and 4096.
CASES = [
    ((1, 17, 640), 32, 8, 128),     # Llama-3-8B head layout
    ((4096,), 32, 8, 128),
    ((1, 17, 640), 16, 2, 128),     # G = 8 (Llama-3-70B layout, 2 kv heads)
    ((4096, 33), 8, 1, 128),
    ((1, 17, 640, 4096), 8, 4, 128),  # G = 2: FMA kernel
    ((1, 17, 640, 4096), 16, 2, 64),  # head_dim 64, G = 8
    ((5, 64, 65), 4, 4, 32),        # head_dim 32, one query head per kv head; split boundaries
]


@pytest.mark.parametrize("contexts,heads,kv_heads,hd", CASES)
def test_paged_attention_matches_oracle(be, contexts, heads, kv_heads, hd):
    rng = np.random.default_rng(sum(contexts) + heads * 7 + hd)
    q, kp, vp, tab, pos, nblk, mbps, ref = _case(rng, contexts, heads, kv_heads, hd)
    rc, out = _run(be, q, kp, vp, tab, pos, heads, kv_heads, hd, nblk, mbps)
    L.check(rc)
    be.synchronize()
    y = out.cpu().numpy()
    assert np.all(np.isfinite(y))
    for b in range(len(contexts)):
        err = max_rel(y[b], ref[b])
        assert err <= ATTN_TOL, (contexts[b], b, err)


def test_paged_attention_rejects_bad_pages_on_device(be):
    """A page entry outside [0, num_blocks) or a position beyond the block table is caught by the
    kernel (no access outside the buffers), reported by the next synchronize as POX_ERR_INVALID, and
    the context stays usable."""
    rng = np.random.default_rng(3)
    heads, kv_heads, hd = 8, 2, 128
    q, kp, vp, tab, pos, nblk, mbps, ref = _case(rng, (40, 20), heads, kv_heads, hd)
    bad = tab.copy()
    bad[0, 1] = nblk + 5  # page 1 of row 0 (positions 16-31) outside the pool
    rc, _ = _run(be, q, kp, vp, bad, pos, heads, kv_heads, hd, nblk, mbps)
    L.check(rc)
    with pytest.raises(L.PoxError) as ei:
        be.synchronize()
    assert ei.value.code == L.POX_ERR_INVALID and "block-table entry" in str(ei.value)
    bad = tab.copy()
    bad[1, 0] = -1
    rc, _ = _run(be, q, kp, vp, bad, pos, heads, kv_heads, hd, nblk, mbps)
    L.check(rc)
    with pytest.raises(L.PoxError):
        be.synchronize()
    far = pos.copy()
    far[1] = mbps * PAGE + 3  # beyond the block table: that row's output is 0
    rc, out = _run(be, q, kp, vp, tab, far, heads, kv_heads, hd, nblk, mbps)
    L.check(rc)
    with pytest.raises(L.PoxError) as ei:
        be.synchronize()
    assert "beyond its block table" in str(ei.value)
    assert np.all(out.cpu().numpy()[1] == 0.0)
    # still usable: a valid call matches the oracle
    rc, out = _run(be, q, kp, vp, tab, pos, heads, kv_heads, hd, nblk, mbps)
    L.check(rc)
    be.synchronize()
    y = out.cpu().numpy()
    for b in range(2):
        assert max_rel(y[b], ref[b]) <= ATTN_TOL


def test_paged_attention_argument_checks(be):
    rng = np.random.default_rng(4)
    q, kp, vp, tab, pos, nblk, mbps, _ = _case(rng, (3,), 24, 2, 128)  # 12 query heads per kv head
    rc, _ = _run(be, q, kp, vp, tab, pos, 24, 2, 128, nblk, mbps)
    assert rc == L.POX_ERR_UNSUPPORTED
    q, kp, vp, tab, pos, nblk, mbps, _ = _case(rng, (3,), 4, 2, 96)
    rc, _ = _run(be, q, kp, vp, tab, pos, 4, 2, 96, nblk, mbps)
    assert rc == L.POX_ERR_UNSUPPORTED
    assert L.lib().pox_cuda_paged_attention(be.ctx, None, None, None, None, None, 1, 4, 2, 128, 1, 1, None,
                                            None) == L.POX_ERR_INVALID
    assert L.lib().pox_cuda_paged_attention(be.ctx, None, None, None, None, None, 0, 4, 2, 128, 1, 1, None,
                                            None) == L.POX_OK
