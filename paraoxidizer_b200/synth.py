"""Synthetic Llama-architecture weights in the .pox layout, for tests and benchmarks.

Random-init N(0, sigma) f32 projections quantized with the reference's quantizer
(quantize_int4_group, crates/paraoxidizer-quant/src/kernels.rs:26-82; optional outlier extraction,
outlier.rs:57-85), f16 embedding / lm_head, f16 norms (1.0 like the reference's fixtures,
tests/common/mod.rs) -- there is no network for real checkpoints.
"""
from __future__ import annotations

import numpy as np

from . import quant as Q


def _f16(a) -> np.ndarray:
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def make_llama(cfg: dict, seed: int = 0, sigma: float = 0.02, group_size: int = 128, outlier_policy=None,
               norm_jitter: float = 0.0) -> dict:
    rng = np.random.default_rng(seed)
    H, I, V = cfg["hidden"], cfg["inter"], cfg["vocab"]
    hd = H // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    shapes = {"q": (qd, H), "k": (kvd, H), "v": (kvd, H), "o": (H, qd), "gate": (I, H), "up": (I, H), "down": (H, I)}
    layers = []
    for _ in range(cfg["layers"]):
        lay = {}
        for name, (r, c) in shapes.items():
            w = rng.standard_normal(r * c, dtype=np.float32) * np.float32(sigma)
            tab = Q.extract_and_zero_outliers(w, outlier_policy) if outlier_policy else None
            packed, scales = Q.quantize_int4_group(w, group_size)
            lay[name] = {"packed": packed, "scales": scales, "rows": r, "cols": c, "group_size": group_size,
                         "outliers": None if tab is None else tab,
                         "outlier_bytes": None if tab is None else Q.outliers_to_bytes(*tab)}
        jit = (lambda: 1.0 + norm_jitter * rng.standard_normal(H, dtype=np.float32)) if norm_jitter else (
            lambda: np.ones(H, np.float32))
        lay["attn_norm"] = _f16(jit())
        lay["mlp_norm"] = _f16(jit())
        layers.append(lay)
    embed = _f16(rng.standard_normal(V * H, dtype=np.float32) * np.float32(sigma))
    lm_head = _f16(rng.standard_normal(V * H, dtype=np.float32) * np.float32(sigma))
    final_norm = _f16(np.ones(H, np.float32))
    return {"layers": layers, "embed": embed, "lm_head": lm_head, "final_norm": final_norm}


def load_into(model, weights: dict) -> None:
    """Uploads make_llama() weights into a CudaModel."""
    for l, lay in enumerate(weights["layers"]):
        proj = {}
        for name in ("q", "k", "v", "o", "gate", "up", "down"):
            t = dict(lay[name])
            t["outliers"] = t.get("outlier_bytes")
            proj[name] = t
        model.set_layer(l, proj, lay["attn_norm"], lay["mlp_norm"])
    model.set_embeddings(weights["embed"], weights["final_norm"], weights["lm_head"])


def oracle_weights(weights: dict) -> dict:
    """The same weights in the form oracle.OracleModel takes (outliers as (idx, val) arrays)."""
    out = {"embed": weights["embed"], "lm_head": weights["lm_head"], "final_norm": weights["final_norm"], "layers": []}
    for lay in weights["layers"]:
        d = {"attn_norm": lay["attn_norm"], "mlp_norm": lay["mlp_norm"]}
        for name in ("q", "k", "v", "o", "gate", "up", "down"):
            t = lay[name]
            d[name] = {"packed": t["packed"], "scales": t["scales"], "rows": t["rows"], "cols": t["cols"],
                       "group_size": t["group_size"], "outliers": t["outliers"]}
        out["layers"].append(d)
    return out


def build_llama_on_device(backend, cfg: dict, max_batch: int, kv_blocks: int, max_blocks_per_seq: int, seed: int = 0,
                          sigma: float = 0.02, tp_rank: int = 0, tp_size: int = 1, outlier_sigma=None):
    """A CudaModel with random-init N(0, sigma) weights generated on the GPU: projections quantized
    INT4 g128 by the GPU quantizer (bit-exact with quantize_int4_group) and uploaded from device
    memory; embedding and lm_head f16; norms 1.0. q/k/v and gate/up are drawn as stacked
    tensors (per-row quantization makes that identical to quantizing them separately).
    With tp_size > 1 only rank tp_rank's shard is drawn (shapes of tp.shard_llama; the draws
    differ from the whole model's, which a throughput benchmark does not need).
    With outlier_sigma (3.5 = the Automatic policy) each drawn projection first loses the values
    with |w - mean| > outlier_sigma * std to an f16 outlier table (extract_and_zero_outliers,
    outlier.rs:57-85, over the stacked tensor, with torch's mean / std instead of the sequential
    f32 sums: the table is for throughput, not parity); those tensors are uploaded from host
    memory, as the outlier upload requires."""
    import ctypes as C

    import torch

    from . import _lib as L
    from .model import CudaModel

    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed * 1000 + tp_rank)
    H, I, V = cfg["hidden"], cfg["inter"] // tp_size, cfg["vocab"] // tp_size
    hd = H // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd // tp_size, cfg["n_kv_heads"] * hd // tp_size
    model = CudaModel(backend, cfg, max_batch, kv_blocks, max_blocks_per_seq, tp_rank=tp_rank, tp_size=tp_size)
    lib = L.lib()

    def tensor(rows, cols):
        w = torch.randn(rows * cols, device="cuda", generator=gen, dtype=torch.float32).mul_(sigma)
        table = None
        if outlier_sigma:
            mean = w.mean()
            thr = outlier_sigma * w.std(correction=0)
            idx = torch.nonzero((w - mean).abs() > thr).flatten()
            vals = w[idx].half()
            w[idx] = 0.0
            n = idx.numel()
            table = np.empty(4 + 6 * n, np.uint8)
            table[:4] = np.frombuffer(np.uint32(n).tobytes(), np.uint8)
            table[4:4 + 4 * n] = idx.to(torch.int32).cpu().numpy().view(np.uint8)
            table[4 + 4 * n:] = vals.cpu().numpy().view(np.uint8)
            del idx, vals
            outlier_bytes[0] += table.size
        p = torch.empty(rows * cols // 2, dtype=torch.uint8, device="cuda")
        s = torch.empty(rows * cols // 128 * 4, dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        L.check(lib.pox_cuda_quantize_int4(backend.ctx, w.data_ptr(), rows * cols, 128, p.data_ptr(), s.data_ptr(),
                                           None))
        backend.synchronize()
        del w
        d = L.TensorDesc()
        d.dtype, d.rows, d.cols, d.group_size = L.POX_I4, rows, cols, 128
        if table is None:
            d.data, d.data_len, d.scales, d.scale_len = p.data_ptr(), p.numel(), s.data_ptr(), s.numel()
        else:
            ph, sh = p.cpu().numpy(), s.cpu().numpy()
            d.data, d.data_len = ph.ctypes.data, ph.size
            d.scales, d.scale_len = sh.ctypes.data, sh.size
            d.outliers, d.outlier_len = table.ctypes.data, table.size
        h = C.c_void_p()
        L.check(lib.pox_cuda_tensor_upload(backend.ctx, C.byref(d), C.byref(h)))
        return h.value

    ones = np.ones(H, np.float32).astype(np.float16).view(np.uint16)
    outlier_bytes = [0]
    weight_bytes = 0
    for l in range(cfg["layers"]):
        shapes = [(qd + 2 * kvd, H), (H, qd), (2 * I, H), (H, I)]
        hs = [tensor(r, c) for r, c in shapes]
        weight_bytes += sum(r * c // 2 + r * c // 128 * 4 for r, c in shapes)
        model.set_layer_tensors(l, *hs, ones, ones)
    embed = torch.randn(cfg["vocab"] * H, device="cuda", generator=gen).mul_(sigma).half()
    head = torch.randn(V * H, device="cuda", generator=gen).mul_(sigma).half()
    fn = torch.ones(H, device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()
    model.set_embeddings_device(embed.data_ptr(), fn.data_ptr(), head.data_ptr())
    del embed, head, fn
    torch.cuda.empty_cache()
    model.weight_bytes = weight_bytes + outlier_bytes[0] + V * H * 2 + (2 * cfg["layers"] + 1) * H * 2
    return model
