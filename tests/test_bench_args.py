"""Host-side checks of bench.py's decode workloads (no GPU): the batches, context and outlier
setting each workload runs with, and that the 70B workload is the Llama-3-70B layout."""
from types import SimpleNamespace

import bench


def args(**kw):
    base = dict(decode_model="llama8b", decode_batches=None, decode_prefill=None)
    base.update(kw)
    return SimpleNamespace(**base)


def test_default_decode_workload_is_llama8b():
    a = args()
    assert bench.decode_batches(a) == (1, 8, 32)
    kw = bench.decode_kwargs(a)
    assert kw["cfg"] is bench.LLAMA_8B and kw["prefill"] == 512
    assert kw["prefill_mode"] == "tokens" and kw["outlier_sigma"] is None


def test_llama70b_workload():
    a = args(decode_model="llama70b")
    assert bench.decode_batches(a) == (1, 16, 64)
    kw = bench.decode_kwargs(a)
    cfg = kw["cfg"]
    assert (cfg["hidden"], cfg["inter"], cfg["layers"], cfg["n_heads"], cfg["n_kv_heads"], cfg["vocab"]) == \
        (8192, 28672, 80, 64, 8, 128256)
    assert kw["prefill"] == 4096 and kw["prefill_mode"] == "reserve" and kw["outlier_sigma"] == 3.5


def test_overrides_and_none():
    assert bench.decode_batches(args(decode_batches="none")) == ()
    assert bench.decode_batches(args(decode_batches="2,4")) == (2, 4)
    assert bench.decode_kwargs(args(decode_prefill=64))["prefill"] == 64


def test_tp_check_models_shard_at_their_rank_counts():
    """The tensor-parallel check's small models give every rank a kv head, whole 128-column groups
    of o_proj / down_proj and an equal vocab slice (tp.check_tp), at 2, 4 and 8 ranks."""
    from paraoxidizer_b200 import tp as TP

    for world, cfg in bench.TP_CHECK_CFGS.items():
        TP.check_tp(cfg, world)
        assert cfg["n_kv_heads"] >= world and (cfg["hidden"] // cfg["n_heads"]) * cfg["n_heads"] // world % 128 == 0


def test_optional_sections_record_failures():
    assert bench._section("ok", lambda: {"a": 1}) == {"a": 1}

    def boom():
        raise RuntimeError("device lost")

    r = bench._section("decode", boom)
    assert r == {"error": "RuntimeError: device lost"}
