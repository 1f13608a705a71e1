"""GPU parity of the batched decode step (CudaModel) against the oracle's forward_token.

Reference: PoxEngine::forward_token (crates/paraoxidizer-runtime/src/engine.rs:411-716) over a
KvCache (engine.rs:10-84); the CUDA path keeps K/V in fp16 pages of 16 tokens, so the oracle runs
with K/V rounded to f16 on store. Bar: end-to-end logits within 1e-2 max abs per step,
teacher-forced on the oracle's tokens, and identical greedy tokens wherever the oracle's top-2
margin exceeds the tolerance.
"""
import numpy as np
import pytest

from oracle import oracle as O
from paraoxidizer_b200.backend import CudaBackend
from paraoxidizer_b200.model import CudaModel
from paraoxidizer_b200.synth import load_into, make_llama, oracle_weights

pytestmark = pytest.mark.gpu

E2E_TOL = 1e-2

CONFIGS = {
    # head_dim 128, 2 query heads per kv head
    "hd128": {"hidden": 512, "inter": 1024, "layers": 2, "n_heads": 4, "n_kv_heads": 2, "vocab": 1000,
              "rms_eps": 1e-5, "rope_theta": 500000.0},
    # the reference's synthetic Llama fixture shape (tests/common/mod.rs:32-163): d 256, 8 / 2 heads
    "fixture": {"hidden": 256, "inter": 512, "layers": 2, "n_heads": 8, "n_kv_heads": 2, "vocab": 1000,
                "rms_eps": 1e-5, "rope_theta": 500000.0},
    # head_dim 64, 8 query heads per kv head
    "hd64": {"hidden": 512, "inter": 512, "layers": 1, "n_heads": 8, "n_kv_heads": 1, "vocab": 512,
             "rms_eps": 1e-5, "rope_theta": 10000.0},
    # the Llama-3-70B head layout (head_dim 128, 8 query heads per kv head; one kv head, as each
    # rank holds at tensor-parallel 8), scaled down
    "l70": {"hidden": 1024, "inter": 2048, "layers": 2, "n_heads": 8, "n_kv_heads": 1, "vocab": 1000,
            "rms_eps": 1e-5, "rope_theta": 500000.0},
    # the Llama-3-8B head layout (head_dim 128, 4 query heads per kv head), scaled down
    "l8": {"hidden": 512, "inter": 1024, "layers": 2, "n_heads": 4, "n_kv_heads": 1, "vocab": 1000,
           "rms_eps": 1e-5, "rope_theta": 500000.0},
}


@pytest.fixture(scope="module")
def be():
    b = CudaBackend.create(0)
    yield b
    b.close()


@pytest.mark.parametrize("name,outliers,nseq", [("hd128", None, 3), ("hd128", "automatic", 3), ("fixture", None, 3),
                                                ("hd64", "aggressive", 3), ("hd128", "automatic", 11),
                                                ("hd64", None, 10), ("l70", "automatic", 3), ("l70", "automatic", 17),
                                                ("l70", None, 12), ("l8", "automatic", 3), ("l8", None, 9)])
def test_decode_matches_forward_token(be, name, outliers, nseq):
    """nseq 3: the batch <= 8 GEMV path; nseq 9-17: the small-M tensor-core paths (batch >= 9
    while every sequence is active; f16 tiles with outliers, the integer kernel without). Head
    layouts with 4-8 query heads of 128 per kv head (l8, l70) take the tensor-core attention."""
    cfg = CONFIGS[name]
    w = make_llama(cfg, seed=11, outlier_policy=outliers, norm_jitter=0.1)
    model = CudaModel(be, cfg, max_batch=nseq, kv_blocks=16 * nseq, max_blocks_per_seq=16)
    load_into(model, w)
    ow = oracle_weights(w)
    rng = np.random.default_rng(5)
    # sequences of different lengths; one runs past 128 positions so attention uses several splits
    lens = (6, 150, 21) if nseq == 3 else tuple(int(v) for v in rng.integers(12, 40, nseq - 1)) + (140,)
    prompts = [list(rng.integers(0, cfg["vocab"], n)) for n in lens]
    steps = 12
    oracles = [O.OracleModel(cfg, ow, max_seq=256, kv_f16=True) for _ in prompts]
    seqs = [model.new_sequence() for _ in prompts]
    feeds = [list(p) for p in prompts]
    worst = 0.0
    agree = total = 0
    horizon = max(len(p) for p in prompts) + steps
    for t in range(horizon):
        active = [i for i in range(len(prompts)) if t < len(prompts[i]) + steps]
        tokens = [int(feeds[i][t]) for i in active]
        logits, nxt = model.decode(tokens, [seqs[i] for i in active])
        for j, i in enumerate(active):
            ref = oracles[i].forward_token(tokens[j], t)
            err = float(np.max(np.abs(logits[j] - ref)))
            worst = max(worst, err)
            assert err <= E2E_TOL, (name, i, t, err)
            top = np.sort(ref)[-2:]
            ref_tok = int(np.argmax(ref))
            if top[1] - top[0] > E2E_TOL:
                total += 1
                agree += int(nxt[j]) == ref_tok
            if t + 1 >= len(prompts[i]):  # greedy continuation, teacher-forced on the oracle's token
                feeds[i].append(ref_tok)
    assert total > 0 and agree == total, (agree, total)
    model.close()


@pytest.mark.parametrize("name,nseq", [("l8", 1), ("l8", 2), ("l8", 4), ("l70", 1), ("l70", 3)])
def test_persistent_decode_matches_forward_token(be, name, nseq):
    """Batch 1-4 without outliers runs every layer as one persistent kernel (grid barriers between the
    projections, attention items combined by the last split of each kv head). Contexts up to 170
    positions put 3 attention splits in a sequence; every step is checked against the oracle, and the
    per-projection launches of the same model (persistent kernel off) agree within 5e-3."""
    cfg = CONFIGS[name]
    w = make_llama(cfg, seed=23, norm_jitter=0.1)
    model = CudaModel(be, cfg, max_batch=8, kv_blocks=32 * nseq, max_blocks_per_seq=16)
    load_into(model, w)
    assert not model.step_persistent(nseq)  # opt-in
    model.set_persistent(True)
    assert model.step_persistent(nseq)
    ow = oracle_weights(w)
    rng = np.random.default_rng(40 + nseq)
    lens = (150, 7, 70, 33)[:nseq]
    prompts = [list(rng.integers(0, cfg["vocab"], n)) for n in lens]
    steps = 20
    oracles = [O.OracleModel(cfg, ow, max_seq=256, kv_f16=True) for _ in prompts]
    seqs = [model.new_sequence() for _ in prompts]
    feeds = [list(p) for p in prompts]
    horizon = max(len(p) for p in prompts) + steps
    outs = {}
    for t in range(horizon):
        active = [i for i in range(nseq) if t < len(prompts[i]) + steps]
        tokens = [int(feeds[i][t]) for i in active]
        logits, nxt = model.decode(tokens, [seqs[i] for i in active])
        for j, i in enumerate(active):
            ref = oracles[i].forward_token(tokens[j], t)
            err = float(np.max(np.abs(logits[j] - ref)))
            assert err <= E2E_TOL, (name, nseq, i, t, err)
            outs[(i, t)] = logits[j].copy()
            if t + 1 >= len(prompts[i]):
                feeds[i].append(int(np.argmax(ref)))
    # the per-projection launches on the same weights and inputs: the same logits up to the order of
    # the RMSNorm sums and of the partial reductions
    model.set_persistent(False)
    assert not model.step_persistent(nseq)
    seqs2 = [model.new_sequence() for _ in prompts]
    worst = 0.0
    for t in range(horizon):
        active = [i for i in range(nseq) if t < len(prompts[i]) + steps]
        logits, _ = model.decode([int(feeds[i][t]) for i in active], [seqs2[i] for i in active])
        for j, i in enumerate(active):
            worst = max(worst, float(np.max(np.abs(logits[j] - outs[(i, t)]))))
    assert worst <= 5e-3, worst
    model.close()


@pytest.mark.parametrize("name", ["l8", "l70"])
def test_decode_long_context_capacity(be, name):
    """A model whose block tables reach 1280 positions (20 attention splits) merges the splits in the
    combine kernel; up to 16 splits the tensor-core attention merges them itself. Both against the
    oracle, at batch 2."""
    cfg = CONFIGS[name]
    w = make_llama(cfg, seed=29, norm_jitter=0.1)
    model = CudaModel(be, cfg, max_batch=2, kv_blocks=40, max_blocks_per_seq=80)
    load_into(model, w)
    ow = oracle_weights(w)
    rng = np.random.default_rng(31)
    prompts = [list(rng.integers(0, cfg["vocab"], n)) for n in (140, 9)]
    steps = 6
    oracles = [O.OracleModel(cfg, ow, max_seq=256, kv_f16=True) for _ in prompts]
    seqs = [model.new_sequence() for _ in prompts]
    feeds = [list(p) for p in prompts]
    for t in range(max(len(p) for p in prompts) + steps):
        active = [i for i in range(2) if t < len(prompts[i]) + steps]
        tokens = [int(feeds[i][t]) for i in active]
        logits, _ = model.decode(tokens, [seqs[i] for i in active])
        for j, i in enumerate(active):
            ref = oracles[i].forward_token(tokens[j], t)
            assert float(np.max(np.abs(logits[j] - ref))) <= E2E_TOL, (name, i, t)
            if t + 1 >= len(prompts[i]):
                feeds[i].append(int(np.argmax(ref)))
    model.close()


# The Llama-3-8B widths (d 4096, 32 / 8 heads of 128, FFN 14336, vocab 128256, f16 embedding and
# lm_head), two layers so the oracle's scalar forward_token stays within seconds per token.
LLAMA8B_2L = {"hidden": 4096, "inter": 14336, "layers": 2, "n_heads": 32, "n_kv_heads": 8, "vocab": 128256,
              "rms_eps": 1e-5, "rope_theta": 500000.0}


@pytest.fixture(scope="module")
def llama8b_2l(be):
    w = make_llama(LLAMA8B_2L, seed=17, norm_jitter=0.1)
    model = CudaModel(be, LLAMA8B_2L, max_batch=32, kv_blocks=64, max_blocks_per_seq=2)
    load_into(model, w)
    yield model, oracle_weights(w)
    model.close()


@pytest.mark.parametrize("nseq", [1, 9, 32])
def test_decode_llama8b_widths(be, llama8b_2l, nseq):
    """Every kernel of the step at its Llama-3-8B size (the batch <= 8 GEMV at 1, the integer small-M
    kernel and the f16 lm_head tiles at 9 and 32, the tensor-core attention with 4 query heads per
    kv head): 3-5 prompt tokens then 5 greedy steps per sequence, teacher-forced on the oracle."""
    from concurrent.futures import ThreadPoolExecutor
    import os

    model, ow = llama8b_2l
    cfg = LLAMA8B_2L
    rng = np.random.default_rng(100 + nseq)
    prompts = [list(rng.integers(0, cfg["vocab"], int(n))) for n in rng.integers(3, 6, nseq)]
    steps = 5
    oracles = [O.OracleModel(cfg, ow, max_seq=32, kv_f16=True) for _ in prompts]
    seqs = [model.new_sequence() for _ in prompts]
    feeds = [list(p) for p in prompts]
    pool = ThreadPoolExecutor(max_workers=min(32, os.cpu_count() or 1))  # the oracle releases the GIL
    agree = total = 0
    worst = 0.0
    for t in range(max(len(p) for p in prompts) + steps):
        active = [i for i in range(nseq) if t < len(prompts[i]) + steps]
        tokens = [int(feeds[i][t]) for i in active]
        logits, nxt = model.decode(tokens, [seqs[i] for i in active])
        refs = list(pool.map(lambda j: oracles[active[j]].forward_token(tokens[j], t), range(len(active))))
        for j, i in enumerate(active):
            ref = refs[j]
            err = float(np.max(np.abs(logits[j] - ref)))
            worst = max(worst, err)
            assert err <= E2E_TOL, (nseq, i, t, err)
            top = np.sort(ref)[-2:]
            ref_tok = int(np.argmax(ref))
            if top[1] - top[0] > E2E_TOL:
                total += 1
                agree += int(nxt[j]) == ref_tok
            if t + 1 >= len(prompts[i]):
                feeds[i].append(ref_tok)
    pool.shutdown()
    for sq in seqs:
        sq.free(model.blocks)
    print(f"llama-8b widths, batch {nseq}: worst logit |diff| {worst:.2e}, greedy agreement {agree}/{total}")
    assert total > 0 and agree == total, (agree, total)


@pytest.mark.parametrize("name,max_batch", [("l8", 96), ("l8", 16), ("l70", 64), ("hd64", 32), ("fixture", 40)])
def test_prefill_matches_forward_token(be, name, max_batch):
    """Prompts fed in passes of up to max_batch rows (rows of several sequences together, a sequence
    split across passes when max_batch is small) give the last prompt token's logits of the oracle's
    token-by-token forward_token; decode steps continue from the pages prefill wrote."""
    cfg = CONFIGS[name]
    w = make_llama(cfg, seed=12, outlier_policy="automatic", norm_jitter=0.1)
    model = CudaModel(be, cfg, max_batch=max_batch, kv_blocks=48, max_blocks_per_seq=16)
    load_into(model, w)
    ow = oracle_weights(w)
    rng = np.random.default_rng(9)
    prompts = [list(int(t) for t in rng.integers(0, cfg["vocab"], n)) for n in (5, 70, 19)]
    oracles = [O.OracleModel(cfg, ow, max_seq=256, kv_f16=True) for _ in prompts]
    seqs = [model.new_sequence() for _ in prompts]
    logits, nxt = model.prefill(prompts, seqs)
    feeds = []
    for i, p in enumerate(prompts):
        for t, tok in enumerate(p):
            ref = oracles[i].forward_token(tok, t)
        err = float(np.max(np.abs(logits[i] - ref)))
        assert err <= E2E_TOL, (name, i, err)
        top = np.sort(ref)[-2:]
        if top[1] - top[0] > E2E_TOL:
            assert int(nxt[i]) == int(np.argmax(ref))
        feeds.append(int(np.argmax(ref)))
    for step in range(4):  # decode continues over the prefilled pages
        pos = [len(p) + step for p in prompts]
        lg, nx = model.decode(feeds, seqs)
        for i in range(3):
            ref = oracles[i].forward_token(feeds[i], pos[i])
            assert float(np.max(np.abs(lg[i] - ref))) <= E2E_TOL, (name, i, step)
            feeds[i] = int(np.argmax(ref))
    model.close()


def test_decode_from_pox_file(be, tmp_path):
    """The model read from a .pox file (pox_cuda_model_load over the C++ container reader: mmap,
    tensor index, one verify_integrity) decodes like forward_token on the same weights."""
    from paraoxidizer_b200.pox_format import PoxFile, llama_pox_bytes

    cfg = CONFIGS["l8"]
    w = make_llama(cfg, seed=13, outlier_policy="automatic", norm_jitter=0.1)
    path = tmp_path / "llama.pox"
    path.write_bytes(llama_pox_bytes(cfg, w))
    f = PoxFile.open(str(path))
    f.verify_integrity()
    model = CudaModel.from_pox(be, f, max_batch=3, kv_blocks=48, max_blocks_per_seq=16)
    f.close()  # the model holds its own copies on the GPU
    assert model.cfg["hidden"] == cfg["hidden"] and model.cfg["vocab"] == cfg["vocab"]
    ow = oracle_weights(w)
    rng = np.random.default_rng(6)
    prompts = [list(rng.integers(0, cfg["vocab"], n)) for n in (4, 70, 19)]
    oracles = [O.OracleModel(cfg, ow, max_seq=256, kv_f16=True) for _ in prompts]
    seqs = [model.new_sequence() for _ in prompts]
    feeds = [list(p) for p in prompts]
    steps = 6
    for t in range(max(len(p) for p in prompts) + steps):
        active = [i for i in range(3) if t < len(prompts[i]) + steps]
        tokens = [int(feeds[i][t]) for i in active]
        logits, nxt = model.decode(tokens, [seqs[i] for i in active])
        for j, i in enumerate(active):
            ref = oracles[i].forward_token(tokens[j], t)
            assert float(np.max(np.abs(logits[j] - ref))) <= E2E_TOL, (i, t)
            if t + 1 >= len(prompts[i]):
                feeds[i].append(int(np.argmax(ref)))
    model.close()


def test_decode_rejects_bad_inputs(be):
    from paraoxidizer_b200 import _lib as L

    cfg = CONFIGS["fixture"]
    model = CudaModel(be, cfg, max_batch=2, kv_blocks=4, max_blocks_per_seq=2)
    load_into(model, make_llama(cfg, seed=3))
    seq = model.new_sequence()
    with pytest.raises(L.PoxError):
        model.decode([1, 2, 3], [seq, seq, seq])  # batch above max_batch
    seq.sequence_len = 40  # position 40 needs a third page: beyond max_blocks_per_seq
    seq.allocated_block_ids = [0, 1]
    with pytest.raises(L.PoxError):
        model.decode([1], [seq])
    # set_state: every page up to a row's next position must be a block (BlockTable pads with -1)
    s2 = model.new_sequence()
    s2.sequence_len, s2.allocated_block_ids = 16, [0]  # position 16 needs page 1, which has no block
    with pytest.raises(L.PoxError) as ei:
        model.set_state([1], [s2])
    assert ei.value.code == L.POX_ERR_INVALID
    # the device path advances positions on the GPU: a step that reaches a page without a block, or a
    # position beyond the block table, is caught by the attention kernel (nothing outside the KV pages
    # is touched) and reported by the next synchronize; the context stays usable
    s3 = model.new_sequence()
    s3.sequence_len, s3.allocated_block_ids = 15, [1]
    model.set_state([1], [s3])
    model.decode_device(1, True)  # position 15 (page 0 = block 1), then advances to 16
    be.synchronize()
    model.decode_device(1, True)  # position 16: page 1 is -1
    with pytest.raises(L.PoxError) as ei:
        be.synchronize()
    assert ei.value.code == L.POX_ERR_INVALID and "block-table entry" in str(ei.value)
    s4 = model.new_sequence()
    s4.sequence_len, s4.allocated_block_ids = 31, [2, 3]
    model.set_state([1], [s4])
    model.decode_device(1, True)  # position 31, the last the table holds
    be.synchronize()
    model.decode_device(1, True)  # position 32 = 16 x max_blocks_per_seq
    with pytest.raises(L.PoxError) as ei:
        be.synchronize()
    assert "beyond its block table" in str(ei.value)
    logits, _ = model.decode([5], [model.new_sequence()])  # usable afterwards
    assert np.all(np.isfinite(logits))
    model.close()
