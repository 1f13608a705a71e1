"""The .pox container reader (libpox_cuda.so's pox_file_*) on the CPU, against files laid out by the
writer restatement (paraoxidizer_b200.pox_format.PoxWriter, pox.rs:397-606).

Reference behaviour checked (crates/paraoxidizer-format/src/pox.rs): the header's magic / version
(:40-55), section bounds -> Security errors (:184-226), zero-copy accessors returning None for empty
scale / outlier sections or unknown names (:311-353), verify_integrity's SHA-256 over data || scales ||
outliers and the first mismatch reported (:356-383); ModelConfig from the metadata. Tensor-parallel
shards of INT4 payloads must equal tp.py's numpy sharding byte for byte.
"""
import hashlib
import os
import struct

import numpy as np
import pytest

from paraoxidizer_b200 import _lib as L
from paraoxidizer_b200 import quant as Q
from paraoxidizer_b200 import tp as TP
from paraoxidizer_b200.pox_format import PoxFile, PoxWriter, llama_pox_bytes, model_config_dict
from paraoxidizer_b200.synth import make_llama

CFG = {"hidden": 256, "inter": 512, "layers": 2, "n_heads": 4, "n_kv_heads": 2, "vocab": 300, "rms_eps": 1e-5,
       "rope_theta": 500000.0}


@pytest.fixture(scope="module")
def model():
    w = make_llama(CFG, seed=5, outlier_policy="automatic", norm_jitter=0.1)
    return w, llama_pox_bytes(CFG, w)


def test_header_and_layout(model):
    _, b = model
    assert b[:4] == b"POX\x01" and struct.unpack_from("<I", b, 4)[0] == 1
    f = PoxFile.from_bytes(b)
    hdr = struct.unpack_from("<12Q", b, 16)
    data_off = hdr[6]
    for t in f.tensors:
        assert t["data_offset"] % 64 == 0 and t["data_offset"] >= data_off
        if t["scale_len"]:
            assert t["scale_offset"] % 64 == 0
    names = {t["name"] for t in f.tensors}
    assert "model.layers.1.mlp.down_proj.weight" in names and "lm_head.weight" in names
    cfg = f.model_config()
    assert (cfg["hidden"], cfg["inter"], cfg["layers"], cfg["n_heads"], cfg["n_kv_heads"], cfg["vocab"]) == \
        (256, 512, 2, 4, 2, 300)
    assert abs(cfg["rms_eps"] - 1e-5) < 1e-12 and cfg["rope_theta"] == 500000.0 and not cfg["tie_word_embeddings"]
    f.close()


def test_payload_slices_round_trip(model, tmp_path):
    w, b = model
    p = tmp_path / "m.pox"
    p.write_bytes(b)
    f = PoxFile.open(str(p))  # mmap path
    t = w["layers"][1]["o"]
    name = "model.layers.1.self_attn.o_proj.weight"
    assert np.array_equal(f.get_tensor_data(name), t["packed"])
    assert np.array_equal(f.get_scale_data(name), t["scales"])
    ob = f.get_outlier_data(name)
    if t["outlier_bytes"] is None:
        assert ob is None
    else:
        assert np.array_equal(ob, t["outlier_bytes"])
    # F16 tensors carry no scales: None, like get_scale_data of scale_len 0
    assert f.get_scale_data("model.norm.weight") is None and f.get_outlier_data("model.norm.weight") is None
    assert np.array_equal(f.get_tensor_data("lm_head.weight").view(np.uint16), w["lm_head"])
    assert f.get_tensor_data("no.such.tensor") is None
    meta = f.tensors[f.tensor_map[name]]
    assert meta["dtype"] == L.POX_I4 and meta["group_size"] == 128 and meta["shape"] == [256, 256]
    h = hashlib.sha256(t["packed"].tobytes() + t["scales"].tobytes() +
                       (b"" if t["outlier_bytes"] is None else t["outlier_bytes"].tobytes())).hexdigest()
    assert meta["sha256"] == h
    f.verify_integrity()
    f.verify_integrity(threads=1)
    f.close()


def test_integrity_mismatch_names_the_tensor(model):
    _, b = model
    f = PoxFile.from_bytes(b)
    t = f.tensors[f.tensor_map["model.layers.0.mlp.up_proj.weight"]]
    bad = bytearray(b)
    bad[t["scale_offset"] + 3] ^= 0x10  # one bit of one scale word
    g = PoxFile.from_bytes(bytes(bad))
    with pytest.raises(L.PoxError) as ei:
        g.verify_integrity()
    assert ei.value.code == L.POX_ERR_INTEGRITY and "model.layers.0.mlp.up_proj.weight" in str(ei.value)
    f.close()
    g.close()


def test_malformed_containers(model):
    _, b = model
    cases = {
        "short": b[:100],
        "magic": b"POX\x02" + b[4:],
        "version": b[:4] + struct.pack("<I", 2) + b[8:],
    }
    hdr = list(struct.unpack_from("<12Q", b, 16))
    for i, what in ((1, "Metadata"), (3, "Tensor index"), (5, "Quant plan"), (9, "Manifest")):
        h = list(hdr)
        h[i] = len(b)  # section runs past the end: out of bounds
        cases[what] = b[:16] + struct.pack("<12Q", *h) + b[112:]
    broken = bytearray(b)
    broken[hdr[2]] = ord("{")  # the index is no longer a JSON array
    cases["index"] = bytes(broken)
    for what, data in cases.items():
        with pytest.raises(L.PoxError) as ei:
            PoxFile.from_bytes(data)
        assert ei.value.code == L.POX_ERR_FORMAT, what
    with pytest.raises(L.PoxError):
        PoxFile.open("/nonexistent/model.pox")


def test_payload_past_the_end_is_none():
    """An index entry whose data range runs past the file: the accessor returns None (pox.rs:311-321)
    and verify_integrity reports the missing data (:358-361)."""
    meta = {"model_config": model_config_dict(CFG), "total_parameters": 0, "quantized_by": "t", "timestamp_utc": 0,
            "original_format": "t", "base_model_name": "t"}
    w = PoxWriter(meta, {"default_precision": "F16", "group_size": 0, "outlier_strategy": "Disabled",
                         "layer_assignments": {}}, "r")
    w.add_tensor("a", (4,), L.POX_F16, 0, np.arange(4, dtype=np.uint16))
    w.tensors[0]["data_len"] = 1 << 40
    f = PoxFile.from_bytes(w.write_to_bytes())
    assert f.get_tensor_data("a") is None
    with pytest.raises(L.PoxError) as ei:
        f.verify_integrity()
    assert ei.value.code == L.POX_ERR_FORMAT and "Missing data" in str(ei.value)


@pytest.mark.parametrize("tp", [2, 4, 8])
def test_shards_equal_tp_py(model, tp):
    w, b = model
    f = PoxFile.from_bytes(b)
    for key, nm, split in (("q", "self_attn.q_proj", 0), ("gate", "mlp.gate_proj", 0), ("o", "self_attn.o_proj", 1),
                           ("down", "mlp.down_proj", 1)):
        t = w["layers"][0][key]
        R, K = t["rows"], t["cols"]
        if split == 1 and K % (128 * tp):
            continue
        for r in range(tp):
            d, s, o = f.shard(f"model.layers.0.{nm}.weight", split, r, tp)
            ref = TP.shard_rows(t, R // tp * r, R // tp * (r + 1)) if split == 0 else \
                TP.shard_cols(t, K // tp * r, K // tp * (r + 1))
            assert np.array_equal(d, ref["packed"]) and np.array_equal(s, ref["scales"]), (key, r)
            if ref["outliers"] is None:
                assert o is None, (key, r)
            else:
                assert np.array_equal(o, Q.outliers_to_bytes(*ref["outliers"])), (key, r)
    f.close()


def test_ffi_symbols_declared():
    for name in ("pox_file_open", "pox_file_from_bytes", "pox_file_close", "pox_file_tensor_meta",
                 "pox_file_verify_integrity", "pox_file_tensor_shard", "pox_cuda_model_load"):
        assert name in L.declared_symbols()
        assert hasattr(L.lib(), name)


def _named_container(name: str) -> bytes:
    meta = {"model_config": model_config_dict(CFG), "total_parameters": 0, "quantized_by": "t", "timestamp_utc": 0,
            "original_format": "t", "base_model_name": "t"}
    w = PoxWriter(meta, {"default_precision": "F16", "group_size": 0, "outlier_strategy": "Disabled",
                         "layer_assignments": {}}, "r")
    w.add_tensor(name, (4,), L.POX_F16, 0, np.arange(4, dtype=np.uint16))
    return w.write_to_bytes()


def test_json_strings_follow_the_reference_parser():
    """The container's JSON is read as serde_json::from_slice reads it (pox.rs:184-226): strings
    are UTF-8 (multibyte names kept), a \\u surrogate pair decodes to one character, and invalid
    UTF-8 or a lone surrogate is a format error rather than a name with stray bytes."""
    b = _named_container("w.层.XXXXXXXXXXXX")
    assert PoxFile.from_bytes(b).tensors[0]["name"] == "w.层.XXXXXXXXXXXX"
    pair = b.replace(b"XXXXXXXXXXXX", b"\\ud835\\udd38")  # same length: offsets stay valid
    assert PoxFile.from_bytes(pair).tensors[0]["name"] == "w.层.\U0001d538"
    bad = {"invalid UTF-8": b.replace("层".encode(), b"\xff\xfe\xfd"),
           "overlong": b.replace("层".encode(), b"\xe0\x80\xaf"),
           "encoded surrogate": b.replace("层".encode(), b"\xed\xa0\x80"),
           "lone trailing surrogate": b.replace(b"XXXXXXXXXXXX", b"\\udd38\\ud835"),
           "lone leading surrogate": b.replace(b"XXXXXXXXXXXX", b"\\ud835abcdef")}
    for what, data in bad.items():
        assert len(data) == len(b), what
        with pytest.raises(L.PoxError) as ei:
            PoxFile.from_bytes(data)
        assert ei.value.code == L.POX_ERR_FORMAT, what


def test_mutated_containers_open_or_fail_cleanly():
    """Seeded corruption of a small container (bytes overwritten, header fields set to extremes,
    truncation): every file either opens, with every accessor, shard and verify_integrity then
    returning data or an error, or is rejected with a PoxError. Nothing reads out of bounds."""
    import random

    cfg = dict(CFG, layers=1, vocab=64)
    b = llama_pox_bytes(cfg, make_llama(cfg, seed=1, outlier_policy="automatic"))
    rng = random.Random(7)
    opened = 0
    for _ in range(300):
        d = bytearray(b)
        kind = rng.randrange(3)
        if kind == 0:
            for _ in range(rng.randrange(1, 8)):
                d[rng.randrange(len(d))] = rng.randrange(256)
        elif kind == 1:
            d = d[:rng.randrange(len(d))]
        else:
            struct.pack_into("<Q", d, 16 + 8 * rng.randrange(12),
                             rng.choice([0, 1, 2**63, 2**64 - 1, len(b), rng.randrange(2**64)]))
        try:
            f = PoxFile.from_bytes(bytes(d))
        except L.PoxError:
            continue
        opened += 1
        for t in f.tensors:
            for fn in (f.get_tensor_data, f.get_scale_data, f.get_outlier_data):
                try:
                    v = fn(t["name"])
                    if v is not None and v.size:
                        _ = int(v[0]) + int(v[-1])
                except L.PoxError:
                    pass
            try:
                f.shard(t["name"], 1, 1, 2)
            except L.PoxError:
                pass
        for call in (f.model_config, f.verify_integrity):
            try:
                call()
            except L.PoxError:
                pass
        f.close()
    assert opened > 0


def _container(edit=None, replace=()) -> bytes:
    """A one-tensor container; edit(writer) changes its sections before writing, then each
    (old, new) byte replacement of equal length is applied (offsets stay valid)."""
    meta = {"model_config": model_config_dict(CFG), "total_parameters": 0, "quantized_by": "t",
            "timestamp_utc": 10, "original_format": "t", "base_model_name": "t"}
    w = PoxWriter(meta, {"default_precision": "F16", "group_size": 0, "outlier_strategy": "Disabled",
                         "layer_assignments": {}}, "r")
    w.add_tensor("a", (4,), L.POX_F16, 0, np.arange(4, dtype=np.uint16))
    if edit:
        edit(w)
    b = w.write_to_bytes()
    for old, new in replace:
        assert len(old) == len(new) and old in b
        b = b.replace(old, new)
    return b


def _opens(b: bytes) -> bool:
    try:
        PoxFile.from_bytes(b).close()
        return True
    except L.PoxError as e:
        assert e.code == L.POX_ERR_FORMAT
        return False


def test_sections_deserialize_like_the_reference_structs():
    """Each JSON section must deserialize into the reference's typed struct (pox.rs:119-158,
    arch.rs:94-112, tensor.rs:114-128; serde derive): required fields present and unique, integers
    as non-negative integer literals, enums by variant name; unknown fields are ignored, optional
    fields may be absent or null."""
    def meta(key, value=None, drop=False):
        def f(w):
            if drop:
                del w.metadata[key]
            else:
                w.metadata[key] = value
        return f

    def cfg(key, value=None, drop=False):
        def f(w):
            if drop:
                del w.metadata["model_config"][key]
            else:
                w.metadata["model_config"][key] = value
        return f

    def man(key, value):
        def f(w):
            w.manifest[key] = value
        return f

    def tensor(key, value):
        def f(w):
            w.tensors[0][key] = value
        return f

    def sig(value):
        def f(w):
            w.signature = value
        return f

    accepted = {
        "as written": _container(),
        "unknown fields": _container(meta("extra", {"x": [1, 2]})),
        "optional ids absent": _container(lambda w: [w.metadata["model_config"].pop(k) for k in ("eos_token_id",
                                                                                                 "bos_token_id")]),
        "u32 at its maximum": _container(cfg("eos_token_id", 2**32 - 1)),
        "f64 given an integer": _container(cfg("rms_norm_eps", 0)),
        "calibration hash null": _container(man("calibration_sha256", None)),
        "calibration hash absent": _container(lambda w: w.manifest.pop("calibration_sha256")),
        "calibration hash string": _container(man("calibration_sha256", "ab")),
        "signature block": _container(sig({"public_key_hex": "ab", "signature_hex": "cd"})),
        "integer -0": _container(replace=[(b'"timestamp_utc":10', b'"timestamp_utc":-0')]),
        "duplicate unknown field": _container(lambda w: w.tensors[0].update(zzzz=1, yyyy=1),
                                              [(b'"yyyy":1', b'"zzzz":1')]),
    }
    for what, b in accepted.items():
        assert _opens(b), what
    rejected = {
        "metadata field missing": _container(meta("quantized_by", drop=True)),
        "config field missing": _container(cfg("vocab_size", drop=True)),
        "integer given a fraction": _container(meta("total_parameters", 1000.0)),
        "integer given a sign": _container(meta("timestamp_utc", -1)),
        "leading zero": _container(replace=[(b'"timestamp_utc":10', b'"timestamp_utc":01')]),
        "u32 overflow": _container(cfg("eos_token_id", 2**32)),
        "string given a number": _container(meta("quantized_by", 5)),
        "bool given a number": _container(cfg("tie_word_embeddings", 0)),
        "unknown architecture": _container(cfg("architecture", "Llama2")),
        "unknown group size": _container(tensor("group_size", "G16")),
        "duplicate tensor field": _container(tensor("data_lex", 5), [(b'"data_lex"', b'"data_len"')]),
        "shape of floats": _container(tensor("shape", [4.0])),
        "calibration hash number": _container(man("calibration_sha256", 5)),
        "tensor hash not a string": _container(man("tensor_hashes", {"a": 1})),
        "quant plan group size string": _container(lambda w: w.quant_plan.update(group_size="G32")),
        "signature field missing": _container(sig({"public_key_hex": "ab"})),
    }
    for what, b in rejected.items():
        assert not _opens(b), what
