"""Tensor-parallel decode, host side (CPU, no GPU): the .pox shard layout and the split of the
decode step, checked against the oracle.

* Every shard of an INT4 tensor with outliers dequantizes bit-exactly to the same slice of the
  whole tensor's dequantization (kernels.rs:85-128 + outlier.rs:88-95).
* 2, 4 and 8 gloo ranks run forward_token (engine.rs:411-716) split the way the CUDA decode step
  splits it -- column-split q/k/v/gate/up/lm_head, row-split o/down summed by an allreduce after
  each, the greedy pick over the ranks' (logit, token) pairs -- through the oracle's primitives,
  and match the oracle's unsplit forward_token: logits within 1e-4 and the same greedy tokens.
"""
import os
import socket

import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200 import tp as TP
from paraoxidizer_b200.synth import make_llama, oracle_weights

CFG = {"hidden": 256, "inter": 512, "layers": 2, "n_heads": 8, "n_kv_heads": 2, "vocab": 1000,
       "rms_eps": 1e-5, "rope_theta": 500000.0}
CFGS = {2: CFG, 4: dict(CFG, hidden=512, n_kv_heads=4),  # 4 ranks: one kv head and 128 columns of o/down each
        # 8 ranks: the shapes of the benchmark's 8-rank tp_check (two query heads of 64 and one kv
        # head per rank, 128 columns of o and 256 of down per rank)
        8: dict(CFG, hidden=1024, inter=2048, n_heads=16, n_kv_heads=8)}


def _dequant(t):
    d = O.dequantize_int4_group(t["packed"], t["scales"], t["group_size"], t["rows"] * t["cols"])
    if t.get("outliers") is not None:
        O.outliers_apply(t["outliers"][0], t["outliers"][1], d)
    return d.reshape(t["rows"], t["cols"])


def _tensor(rows, cols, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal(rows * cols, dtype=np.float32) * np.float32(0.02)
    w[rng.integers(0, w.size, 40)] *= np.float32(30.0)
    tab = Q.extract_and_zero_outliers(w, "aggressive")
    p, s = Q.quantize_int4_group(w, 128)
    return {"packed": p, "scales": s, "rows": rows, "cols": cols, "group_size": 128, "outliers": tab,
            "outlier_bytes": Q.outliers_to_bytes(*tab)}


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_shards_dequantize_to_slices(tp):
    t = _tensor(64, 1024, 7)
    assert t["outliers"] is not None and len(t["outliers"][0]) > 10
    full = _dequant(t)
    rs, cs = t["rows"] // tp, t["cols"] // tp
    for r in range(tp):
        a = TP.shard_rows(t, r * rs, (r + 1) * rs)
        assert np.array_equal(_dequant(a).view(np.uint32), full[r * rs:(r + 1) * rs].view(np.uint32))
        b = TP.shard_cols(t, r * cs, (r + 1) * cs)
        assert np.array_equal(_dequant(b).view(np.uint32), full[:, r * cs:(r + 1) * cs].view(np.uint32))
        if b["outliers"] is not None:  # the .pox table bytes agree with the (idx, val) arrays
            assert np.array_equal(b["outlier_bytes"], Q.outliers_to_bytes(*b["outliers"]))


def test_shard_ranges_reject_bad_tp():
    with pytest.raises(ValueError):
        TP.shard_ranges(CFG, 3, 0)  # 8 heads, 2 kv heads: not divisible by 3
    with pytest.raises(ValueError):
        TP.shard_ranges(CFG, 4, 0)  # 2 kv heads


def test_pick_greedy_first_maximum():
    assert TP.pick_greedy([(1.0, 5), (2.0, 900), (2.0, 700)]) == 700
    assert TP.pick_greedy([(3.0, 10), (3.0, 600)]) == 10


def _tp_forward(w, cfg, tp, rank, tok, pos, kc, vc):
    """forward_token split across `tp` ranks (this is rank `rank`); the allreduce and the gather go
    through torch.distributed."""
    import torch
    import torch.distributed as dist

    H = cfg["hidden"]
    hd = H // cfg["n_heads"]
    nq, nkv = cfg["n_heads"] // tp, cfg["n_kv_heads"] // tp
    eps, theta = cfg["rms_eps"], cfg["rope_theta"]
    x = O.f16_bits_to_f32(np.asarray(w["embed"]).reshape(-1, H)[tok % cfg["vocab"]]).astype(np.float32)

    def gemv(t, v):
        return O.gemv_int4(t["packed"], t["scales"], t["group_size"], t["rows"], t["cols"], t.get("outliers"), v)

    def allreduce(partial):
        tt = torch.from_numpy(np.ascontiguousarray(partial, np.float32))
        dist.all_reduce(tt)
        return tt.numpy()

    for l, lay in enumerate(w["layers"]):
        h = O.rms_norm(x, lay["attn_norm"], eps)
        q, k = O.rope(gemv(lay["q"], h), gemv(lay["k"], h), nq, nkv, hd, pos, theta)
        kc[l, pos], vc[l, pos] = k.reshape(nkv, hd), gemv(lay["v"], h).reshape(nkv, hd)
        att = O.attention(q, kc[l, :pos + 1], vc[l, :pos + 1], nq, nkv, hd, pos)
        part = gemv(lay["o"], att)
        x = allreduce(x + part if rank == 0 else part)
        h = O.rms_norm(x, lay["mlp_norm"], eps)
        part = gemv(lay["down"], O.swiglu(gemv(lay["gate"], h), gemv(lay["up"], h)))
        x = allreduce(x + part if rank == 0 else part)
    h = O.rms_norm(x, w["final_norm"], eps)
    Vl = cfg["vocab"] // tp
    logits = O.gemv_f16(w["lm_head"], Vl, H, h)
    logits[~np.isfinite(logits)] = 0.0
    j = int(np.argmax(logits))  # numpy argmax is the first maximum
    pairs = [None] * tp
    dist.all_gather_object(pairs, (float(logits[j]), rank * Vl + j))
    return logits, TP.pick_greedy(pairs)


def _rank_main(rank, world, port, outdir):
    cfg = CFGS[world]
    import torch.distributed as dist

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        w = make_llama(cfg, seed=4, outlier_policy="automatic", norm_jitter=0.1)
        shard = TP.shard_llama(oracle_weights(w), cfg, world, rank)
        hd = cfg["hidden"] // cfg["n_heads"]
        steps = 5
        kc = np.zeros((cfg["layers"], steps, cfg["n_kv_heads"] // world, hd), np.float32)
        vc = np.zeros_like(kc)
        tok = 17
        out_logits, out_next = [], []
        for pos in range(steps):
            logits, nxt = _tp_forward(shard, cfg, world, rank, tok, pos, kc, vc)
            out_logits.append(logits)
            out_next.append(nxt)
            tok = nxt
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), logits=np.stack(out_logits), next=np.array(out_next))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_gloo_matches_oracle(tmp_path, world):
    import torch.multiprocessing as mp

    cfg = CFGS[world]
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(res[0]["next"], res[r]["next"])  # every rank picks the same tokens
    w = make_llama(cfg, seed=4, outlier_policy="automatic", norm_jitter=0.1)
    ref = O.OracleModel(cfg, oracle_weights(w), max_seq=8)
    Vl = cfg["vocab"] // world
    tok = 17
    for pos in range(len(res[0]["next"])):
        full = ref.forward_token(tok, pos)
        got = np.concatenate([res[r]["logits"][pos] for r in range(world)])
        assert np.max(np.abs(got - full)) <= 1e-4, pos
        for r in range(world):
            assert np.allclose(res[r]["logits"][pos], full[r * Vl:(r + 1) * Vl], atol=1e-4)
        assert int(res[0]["next"][pos]) == O.argmax(full)
        tok = int(res[0]["next"][pos])
