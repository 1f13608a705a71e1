"""Tensor-parallel shards of .pox payloads (host side, numpy) for decode on 1/2/4/8 GPUs of a node.

The reference decodes on one device. The split is the standard one for a Llama block, chosen so
that every .pox payload (row-major packed nibbles, flat groups of group_size along K, kernels.rs:
26-82; outlier table of flat indices, outlier.rs:88-127) shards without re-quantization:

* row split (q, k, v, gate, up and the lm_head): rank r takes rows [r0, r1), a contiguous byte
  range of the packed nibbles and of the scale words; outlier indices in [r0 K, r1 K) shift by
  -r0 K.
* column split (o, down): rank r takes columns [c0, c1) of every row, c0 and c1 multiples of the
  group size, so the groups are whole; outlier index r K + c becomes r (c1 - c0) + (c - c0).
  Each rank's partial product is summed over ranks by the decode step's allreduce.

Index order is preserved, so the "last entry wins" rule of the replace step (kernels.rs:211-219)
still holds in every shard, and a shard dequantizes bit-exactly to the same slice of the whole
tensor's dequantization.
"""
from __future__ import annotations

import numpy as np

from . import quant as Q

ROW_SPLIT = ("q", "k", "v", "gate", "up")
COL_SPLIT = ("o", "down")


def _with_outliers(t: dict, idx, val) -> dict:
    if t.get("outliers") is None:
        return t
    t["outliers"] = (idx, val) if len(idx) else None
    t["outlier_bytes"] = Q.outliers_to_bytes(idx, val) if len(idx) else None
    return t


def shard_rows(t: dict, r0: int, r1: int) -> dict:
    """Rows [r0, r1) of an INT4 .pox tensor dict (make_llama layout)."""
    K, gs = t["cols"], t["group_size"]
    assert K % 2 == 0 and K % gs == 0, "groups must line up with rows"
    rb, sb = K // 2, K // gs * 4
    out = {"packed": np.ascontiguousarray(np.asarray(t["packed"], np.uint8)[r0 * rb:r1 * rb]),
           "scales": np.ascontiguousarray(np.asarray(t["scales"], np.uint8)[r0 * sb:r1 * sb]),
           "rows": r1 - r0, "cols": K, "group_size": gs, "outliers": t.get("outliers"), "outlier_bytes": None}
    if t.get("outliers") is not None:
        idx, val = (np.asarray(a) for a in t["outliers"])
        keep = (idx >= r0 * K) & (idx < r1 * K)
        out = _with_outliers(out, (idx[keep] - r0 * K).astype(np.uint32), val[keep].astype(np.uint16))
    return out


def shard_cols(t: dict, c0: int, c1: int) -> dict:
    """Columns [c0, c1) of every row of an INT4 .pox tensor dict; c0, c1 multiples of the group size."""
    R, K, gs = t["rows"], t["cols"], t["group_size"]
    assert c0 % gs == 0 and c1 % gs == 0 and K % gs == 0, "column shards must hold whole groups"
    p = np.asarray(t["packed"], np.uint8).reshape(R, K // 2)[:, c0 // 2:c1 // 2]
    s = np.asarray(t["scales"], np.uint8).reshape(R, K // gs * 4)[:, c0 // gs * 4:c1 // gs * 4]
    out = {"packed": np.ascontiguousarray(p).reshape(-1), "scales": np.ascontiguousarray(s).reshape(-1),
           "rows": R, "cols": c1 - c0, "group_size": gs, "outliers": t.get("outliers"), "outlier_bytes": None}
    if t.get("outliers") is not None:
        idx, val = (np.asarray(a) for a in t["outliers"])
        r, c = idx // K, idx % K
        keep = (c >= c0) & (c < c1)
        nidx = (r[keep] * (c1 - c0) + (c[keep] - c0)).astype(np.uint32)
        out = _with_outliers(out, nidx, val[keep].astype(np.uint16))
    return out


def check_tp(cfg: dict, tp: int) -> None:
    if tp < 1 or tp > 8:
        raise ValueError("tensor parallel size must be 1..8")
    if cfg["n_heads"] % tp or cfg["n_kv_heads"] % tp or cfg["vocab"] % tp or cfg["inter"] % (128 * tp):
        raise ValueError(f"tp={tp} needs heads, kv heads and vocab divisible by it and the FFN size by 128 x it")


def shard_ranges(cfg: dict, tp: int, rank: int) -> dict:
    """Row / column ranges of rank `rank`: {"q": (r0, r1), "k": ..., "o": (c0, c1), ...}."""
    check_tp(cfg, tp)
    H, I, V = cfg["hidden"], cfg["inter"], cfg["vocab"]
    hd = H // cfg["n_heads"]
    qd, kvd, Il, Vl = cfg["n_heads"] * hd // tp, cfg["n_kv_heads"] * hd // tp, I // tp, V // tp
    return {"q": (rank * qd, (rank + 1) * qd), "k": (rank * kvd, (rank + 1) * kvd),
            "v": (rank * kvd, (rank + 1) * kvd), "gate": (rank * Il, (rank + 1) * Il),
            "up": (rank * Il, (rank + 1) * Il), "o": (rank * qd, (rank + 1) * qd), "down": (rank * Il, (rank + 1) * Il),
            "lm_head": (rank * Vl, (rank + 1) * Vl)}


def shard_llama(weights: dict, cfg: dict, tp: int, rank: int) -> dict:
    """Rank `rank`'s shard of make_llama() weights, in the same dict layout (embedding and norms
    replicated, lm_head rows of the rank's vocab slice)."""
    rg = shard_ranges(cfg, tp, rank)
    H = cfg["hidden"]
    layers = []
    for lay in weights["layers"]:
        d = {"attn_norm": lay["attn_norm"], "mlp_norm": lay["mlp_norm"]}
        for name in ROW_SPLIT:
            d[name] = shard_rows(lay[name], *rg[name])
        for name in COL_SPLIT:
            d[name] = shard_cols(lay[name], *rg[name])
        layers.append(d)
    v0, v1 = rg["lm_head"]
    head = np.asarray(weights["lm_head"], np.uint16)[v0 * H:v1 * H]
    return {"layers": layers, "embed": weights["embed"], "final_norm": weights["final_norm"],
            "lm_head": np.ascontiguousarray(head)}


def pick_greedy(pairs) -> int:
    """The cross-rank greedy pick the decode step runs on the GPU: pairs[r] = (best logit, token
    index in the whole vocabulary) of rank r; the larger logit wins, then the smaller index -- the
    first maximum of the concatenated logits (sampler.rs:55-65)."""
    best = None
    for v, i in pairs:
        if best is None or v > best[0] or (v == best[0] and i < best[1]):
            best = (float(v), int(i))
    return best[1]
