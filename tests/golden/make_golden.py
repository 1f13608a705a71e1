"""Writes tests/golden/oracle_vectors.npz: small seeded inputs of the decode path and the oracle's
outputs on them (INT4 quantization with outliers and its GEMV, INT8 and F16 GEMVs, GQA attention,
and a 2-layer model's forward_token logits).

The reference is Rust with no toolchain here, so these are outputs of the oracle (the C
restatement of the reference's path), not of the reference itself: they pin the oracle against
later changes, next to the reference's own known-answer tests. Run from the repository root:
    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from paraoxidizer_b200.synth import make_llama, oracle_weights  # noqa: E402

FORWARD_CFG = {"hidden": 256, "inter": 512, "layers": 2, "n_heads": 8, "n_kv_heads": 2, "vocab": 300,
               "rms_eps": 1e-5, "rope_theta": 500000.0}
FORWARD_SEED = 11
FORWARD_TOKENS = [7, 250, 3, 99, 42, 42, 180, 5]


def vectors() -> dict:
    rng = np.random.default_rng(2024)
    out = {}
    # INT4 group 64 with a 3.5-sigma outlier table, 64 x 256
    w = rng.standard_normal(64 * 256, dtype=np.float32) * np.float32(0.02)
    w[rng.choice(w.size, 12, replace=False)] = np.float32(0.9)
    w_in = w.copy()  # extraction zeroes the outliers in place
    idx, val = O.extract_and_zero_outliers(w, "automatic")
    p, s = O.quantize_int4_group(w, 64)
    x = rng.standard_normal(256, dtype=np.float32)
    out.update(i4_w=w_in, i4_idx=idx, i4_val=val, i4_packed=p, i4_scales=s, i4_x=x,
               i4_y=O.gemv_int4(p, s, 64, 64, 256, (idx, val), x))
    # INT8 per tensor, 48 x 200
    w8 = rng.standard_normal(48 * 200, dtype=np.float32) * np.float32(0.02)
    q8, s8 = O.quantize_int8_symmetric(w8)
    x8 = rng.standard_normal(200, dtype=np.float32)
    out.update(i8_w=w8, i8_q=q8, i8_scale=s8, i8_x=x8, i8_y=O.gemv_int8(q8, s8, 48, 200, x8))
    # F16 rows, 40 x 96
    wb = (rng.standard_normal(40 * 96, dtype=np.float32) * np.float32(0.02)).astype(np.float16).view(np.uint16)
    xf = rng.standard_normal(96, dtype=np.float32)
    out.update(f16_w=wb, f16_x=xf, f16_y=O.gemv_f16(wb, 40, 96, xf))
    # GQA attention: 8 query heads over 2 kv heads of 64, positions 0..40
    q = rng.standard_normal(8 * 64, dtype=np.float32)
    kc = rng.standard_normal(41 * 2 * 64, dtype=np.float32)
    vc = rng.standard_normal(41 * 2 * 64, dtype=np.float32)
    out.update(att_q=q, att_k=kc, att_v=vc, att_out=O.attention(q, kc, vc, 8, 2, 64, 40))
    # forward_token of a 2-layer model (weights regenerated from FORWARD_SEED by make_llama)
    m = O.OracleModel(FORWARD_CFG, oracle_weights(make_llama(FORWARD_CFG, seed=FORWARD_SEED,
                                                             outlier_policy="automatic", norm_jitter=0.1)), 16)
    out["fwd_logits"] = np.stack([m.forward_token(t, i) for i, t in enumerate(FORWARD_TOKENS)])
    return out


if __name__ == "__main__":
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle_vectors.npz")
    np.savez_compressed(path, **vectors())
    print(path, os.path.getsize(path), "bytes")
