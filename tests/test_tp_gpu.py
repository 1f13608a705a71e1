"""Tensor-parallel decode on 2, 4 and 8 GPUs of one node against the oracle (each size skipped
with fewer GPUs).

One process per GPU, each a CudaModel rank holding its shards (tp.shard_llama); the
exchanges run once over NCCL and once over CUDA IPC peer memory. Every rank's vocab slice of the
logits must be within the end-to-end bar (1e-2 max abs) of the oracle's forward_token
(engine.rs:411-716, K/V rounded to f16), teacher-forced on the oracle's tokens, and both ranks must
return identical greedy tokens equal to the oracle's wherever its top-2 margin exceeds the bar.
The model grows with the rank count so that every rank holds at least one kv head and 128-column
slices of o_proj and down_proj.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

E2E_TOL = 1e-2
CFG = {"hidden": 512, "inter": 1024, "layers": 2, "n_heads": 4, "n_kv_heads": 2, "vocab": 1000,
       "rms_eps": 1e-5, "rope_theta": 500000.0}
CFGS = {2: CFG,
        4: dict(CFG, n_heads=8, n_kv_heads=4),
        8: dict(CFG, hidden=1024, inter=2048, n_heads=16, n_kv_heads=8)}
PROMPTS = (5, 140, 19)
STEPS = 10


def _gpus():
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _oracle_feed(cfg):
    """Token feeds of the three sequences: prompt, then the oracle's greedy continuation."""
    from oracle import oracle as O
    from paraoxidizer_b200.synth import make_llama, oracle_weights

    w = make_llama(cfg, seed=21, outlier_policy="automatic", norm_jitter=0.1)
    rng = np.random.default_rng(8)
    feeds, logits = [], []
    for n in PROMPTS:
        ref = O.OracleModel(cfg, oracle_weights(w), max_seq=256, kv_f16=True)
        feed = list(rng.integers(0, cfg["vocab"], n))
        out = []
        for t in range(n + STEPS):
            lg = ref.forward_token(int(feed[t]), t)
            out.append(lg)
            if t + 1 >= n:
                feed.append(int(np.argmax(lg)))
        feeds.append(feed[:n + STEPS])  # the last greedy token is never fed
        logits.append(np.stack(out))
    return w, feeds, logits


def _rank_main(rank, world, port, outdir, feeds, mode):
    cfg = CFGS[world]
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    from paraoxidizer_b200 import tp as TP
    from paraoxidizer_b200.backend import CudaBackend
    from paraoxidizer_b200.model import CudaModel
    from paraoxidizer_b200.synth import load_into, make_llama

    be = CudaBackend.create(rank)
    try:
        w = make_llama(cfg, seed=21, outlier_policy="automatic", norm_jitter=0.1)
        model = CudaModel(be, cfg, max_batch=3, kv_blocks=48, max_blocks_per_seq=16, tp_rank=rank, tp_size=world)
        load_into(model, TP.shard_llama(w, cfg, world, rank))
        model.init_comm(modes=(mode,))
        seqs = [model.new_sequence() for _ in feeds]
        horizon = max(len(f) for f in feeds)
        logs = {i: [] for i in range(len(feeds))}
        nexts = {i: [] for i in range(len(feeds))}
        for t in range(horizon):
            active = [i for i in range(len(feeds)) if t < len(feeds[i])]
            lg, nx = model.decode([feeds[i][t] for i in active], [seqs[i] for i in active])
            for j, i in enumerate(active):
                logs[i].append(lg[j])
                nexts[i].append(int(nx[j]))
        np.savez(os.path.join(outdir, f"{mode}_rank{rank}.npz"),
                 **{f"l{i}": np.stack(logs[i]) for i in logs}, **{f"n{i}": np.array(nexts[i]) for i in nexts})
        model.close()
    finally:
        be.close()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode", ["peer", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_matches_oracle(tmp_path, world, mode):
    import torch.multiprocessing as mp

    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    w, feeds, ref_logits = _oracle_feed(CFGS[world])
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), feeds, mode), nprocs=world, join=True,
                       start_method="spawn")
    res = [np.load(tmp_path / f"{mode}_rank{r}.npz") for r in range(world)]
    Vl = CFGS[world]["vocab"] // world
    agree = total = 0
    for i, feed in enumerate(feeds):
        for r in range(1, world):
            assert np.array_equal(res[0][f"n{i}"], res[r][f"n{i}"])
        for r in range(world):
            err = np.max(np.abs(res[r][f"l{i}"] - ref_logits[i][:, r * Vl:(r + 1) * Vl]))
            assert err <= E2E_TOL, (mode, i, r, err)
        for t in range(len(feed)):
            ref = ref_logits[i][t]
            top = np.sort(ref)[-2:]
            if top[1] - top[0] > E2E_TOL:
                total += 1
                agree += int(res[0][f"n{i}"][t]) == int(np.argmax(ref))
    assert total > 0 and agree == total, (agree, total)
