"""The .pox container: a writer that lays files out as the reference's PoxWriter does, and a reader over
libpox_cuda.so's C++ parser (pox_file_*), mirroring PoxFile.

Reference (paths relative to the reference repository root):
  * PoxHeader                 crates/paraoxidizer-format/src/pox.rs:23-113 (128 bytes, little endian)
  * PoxFile::{open, from_bytes, get_*_data, verify_integrity}   pox.rs:171-383
  * PoxWriter::{new, add_tensor, write_to_bytes}                 pox.rs:397-606
  * TensorMeta / DType / QuantGroupSize   crates/paraoxidizer-core/src/tensor.rs:4-128
  * ModelConfig                           crates/paraoxidizer-core/src/arch.rs:96-112

The writer produces test and benchmark artifacts (there is no network for real checkpoints); the
layout is the format's: header, metadata JSON, quant plan JSON, 64-byte aligned payloads, tensor index
JSON with absolute offsets, manifest JSON (artifact SHA-256 of everything after the header up to the
index), optional signature JSON.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import struct
from typing import Optional

import numpy as np

from . import _lib as L

MAGIC = b"POX\x01"
VERSION = 1
HEADER_SIZE = 128
ALIGN = 64

DTYPE_NAMES = {L.POX_F32: "F32", L.POX_F16: "F16", L.POX_BF16: "BF16", L.POX_I8: "I8", L.POX_I4: "I4"}
GROUP_NAMES = {0: "None", 32: "G32", 64: "G64", 128: "G128", 256: "G256"}


def _json(obj) -> bytes:
    """Compact JSON, fields in declaration order (serde_json::to_vec of the reference's structs)."""
    return json.dumps(obj, separators=(",", ":"), ensure_ascii=False).encode()


def _pad(buf: bytearray, align: int = ALIGN) -> None:
    r = len(buf) % align
    if r:
        buf.extend(b"\0" * (align - r))


def model_config_dict(cfg: dict, max_position_embeddings: int = 8192, tie_word_embeddings: bool = False) -> dict:
    """ModelConfig (arch.rs:96-112) of a decode configuration dict (hidden, inter, layers, ...)."""
    return {"architecture": "Llama", "hidden_size": cfg["hidden"], "intermediate_size": cfg["inter"],
            "num_hidden_layers": cfg["layers"], "num_attention_heads": cfg["n_heads"],
            "num_key_value_heads": cfg["n_kv_heads"], "vocab_size": cfg["vocab"],
            "max_position_embeddings": max_position_embeddings, "rms_norm_eps": float(cfg.get("rms_eps", 1e-5)),
            "rope_theta": float(cfg.get("rope_theta", 500000.0)), "tie_word_embeddings": tie_word_embeddings,
            "eos_token_id": 2, "bos_token_id": 1}


class PoxWriter:
    """Builder of .pox bytes with the reference writer's layout (pox.rs:397-606)."""

    def __init__(self, metadata: dict, quant_plan: dict, run_id: str):
        self.metadata = metadata
        self.quant_plan = quant_plan
        self.manifest = {"run_id": run_id, "source_model_sha256": "", "calibration_sha256": None,
                         "compiler_version": "0.1.0", "target_arch": "x86_64", "tensor_hashes": {},
                         "artifact_sha256": ""}
        self.signature = None
        self.tensors: list[dict] = []
        self.payload = bytearray()

    def add_tensor(self, name: str, shape, dtype: int, group_size: int, data, scales=None, outliers=None) -> None:
        """add_tensor (pox.rs:442-505): SHA-256 of data || scales || outliers, each chunk 64-byte aligned."""
        d = np.ascontiguousarray(data).view(np.uint8).reshape(-1).tobytes()
        s = None if scales is None else np.ascontiguousarray(scales).view(np.uint8).reshape(-1).tobytes()
        o = None if outliers is None else np.ascontiguousarray(outliers).view(np.uint8).reshape(-1).tobytes()
        h = hashlib.sha256(d)
        if s is not None:
            h.update(s)
        if o is not None:
            h.update(o)
        digest = h.hexdigest()
        self.manifest["tensor_hashes"][name] = digest
        _pad(self.payload)
        data_off = len(self.payload)
        self.payload.extend(d)
        scale_off = scale_len = outl_off = outl_len = 0
        if s is not None:
            _pad(self.payload)
            scale_off, scale_len = len(self.payload), len(s)
            self.payload.extend(s)
        if o is not None:
            _pad(self.payload)
            outl_off, outl_len = len(self.payload), len(o)
            self.payload.extend(o)
        self.tensors.append({"name": name, "shape": [int(v) for v in shape], "dtype": DTYPE_NAMES[dtype],
                             "group_size": GROUP_NAMES[group_size], "data_offset": data_off, "data_len": len(d),
                             "scale_offset": scale_off, "scale_len": scale_len, "outlier_offset": outl_off,
                             "outlier_len": outl_len, "sha256": digest})

    def write_to_bytes(self) -> bytes:
        """write_to_bytes (pox.rs:516-606)."""
        out = bytearray(HEADER_SIZE)
        meta = _json(self.metadata)
        meta_off = len(out)
        out.extend(meta)
        _pad(out)
        plan = _json(self.quant_plan)
        plan_off = len(out)
        out.extend(plan)
        _pad(out)
        data_off = len(out)
        out.extend(self.payload)
        _pad(out)
        for t in self.tensors:  # absolute offsets
            t["data_offset"] += data_off
            if t["scale_len"] > 0:
                t["scale_offset"] += data_off
            if t["outlier_len"] > 0:
                t["outlier_offset"] += data_off
        index = _json(self.tensors)
        index_off = len(out)
        out.extend(index)
        _pad(out)
        self.manifest["artifact_sha256"] = hashlib.sha256(bytes(out[HEADER_SIZE:])).hexdigest()
        man = _json(self.manifest)
        man_off = len(out)
        out.extend(man)
        _pad(out)
        sig_off = sig_len = 0
        if self.signature is not None:
            sig = _json(self.signature)
            sig_off, sig_len = len(out), len(sig)
            out.extend(sig)
        header = MAGIC + struct.pack("<III", VERSION, 0, 0) + struct.pack(
            "<12Q", meta_off, len(meta), index_off, len(index), plan_off, len(plan), data_off, len(self.payload),
            man_off, len(man), sig_off, sig_len)
        header += b"\0" * (HEADER_SIZE - len(header))
        out[:HEADER_SIZE] = header
        return bytes(out)

    def write_to_file(self, path: str) -> None:
        with open(path, "wb") as f:
            f.write(self.write_to_bytes())


def llama_pox_bytes(cfg: dict, weights: dict, run_id: str = "pox-run-synthetic") -> bytes:
    """A make_llama() model as .pox bytes under the engine's tensor names (engine.rs:424-713): INT4
    projections with their outlier tables, F16 embedding / lm_head / norms."""
    H, V = cfg["hidden"], cfg["vocab"]
    meta = {"model_config": model_config_dict(cfg), "total_parameters": 0, "quantized_by": "paraoxidizer_b200",
            "timestamp_utc": 0, "original_format": "Synthetic", "base_model_name": "random-init"}
    plan = {"default_precision": "INT4", "group_size": 128, "outlier_strategy": "Automatic", "layer_assignments": {}}
    w = PoxWriter(meta, plan, run_id)
    w.add_tensor("model.embed_tokens.weight", (V, H), L.POX_F16, 0, weights["embed"])
    names = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
             "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}
    for l, lay in enumerate(weights["layers"]):
        w.add_tensor(f"model.layers.{l}.input_layernorm.weight", (H,), L.POX_F16, 0, lay["attn_norm"])
        for key, nm in names.items():
            t = lay[key]
            w.add_tensor(f"model.layers.{l}.{nm}.weight", (t["rows"], t["cols"]), L.POX_I4, t["group_size"],
                         t["packed"], t["scales"], t.get("outlier_bytes"))
        w.add_tensor(f"model.layers.{l}.post_attention_layernorm.weight", (H,), L.POX_F16, 0, lay["mlp_norm"])
    w.add_tensor("model.norm.weight", (H,), L.POX_F16, 0, weights["final_norm"])
    w.add_tensor("lm_head.weight", (V, H), L.POX_F16, 0, weights["lm_head"])
    return w.write_to_bytes()


class PoxFileMeta(C.Structure):
    """pox_tensor_meta (include/pox_cuda.h): TensorMeta of one index entry."""

    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int), ("group_size", C.c_uint32), ("rank", C.c_uint32),
                ("dims", C.c_uint64 * 8), ("data_offset", C.c_uint64), ("data_len", C.c_uint64),
                ("scale_offset", C.c_uint64), ("scale_len", C.c_uint64), ("outlier_offset", C.c_uint64),
                ("outlier_len", C.c_uint64), ("sha256", C.c_char_p)]


class PoxFile:
    """PoxFile (pox.rs:159-383) over the library's parser: the payload accessors return zero-copy numpy
    views of the mapped file (None where the reference returns None)."""

    def __init__(self, handle: int):
        self.handle = handle
        n = C.c_size_t()
        L.check(L.lib().pox_file_tensor_count(handle, C.byref(n)))
        self.tensors = []
        for i in range(n.value):
            m = PoxFileMeta()
            L.check(L.lib().pox_file_tensor_meta(handle, i, C.byref(m)))
            self.tensors.append({"name": m.name.decode(), "dtype": m.dtype, "group_size": m.group_size,
                                 "shape": [int(m.dims[j]) for j in range(m.rank)], "data_offset": m.data_offset,
                                 "data_len": m.data_len, "scale_offset": m.scale_offset, "scale_len": m.scale_len,
                                 "outlier_offset": m.outlier_offset, "outlier_len": m.outlier_len,
                                 "sha256": m.sha256.decode()})
        self.tensor_map = {t["name"]: i for i, t in enumerate(self.tensors)}

    @staticmethod
    def open(path: str) -> "PoxFile":
        h = C.c_void_p()
        L.check(L.lib().pox_file_open(path.encode(), C.byref(h)))
        return PoxFile(h.value)

    @staticmethod
    def from_bytes(b: bytes) -> "PoxFile":
        h = C.c_void_p()
        buf = (C.c_uint8 * len(b)).from_buffer_copy(b) if len(b) else None
        L.check(L.lib().pox_file_from_bytes(buf, len(b), C.byref(h)))
        return PoxFile(h.value)

    def close(self) -> None:
        if self.handle:
            L.lib().pox_file_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _slice(self, fn, name: str) -> Optional[np.ndarray]:
        p, n = C.c_void_p(), C.c_size_t()
        L.check(fn(self.handle, name.encode(), C.byref(p), C.byref(n)))
        if not p.value:
            return None
        return np.ctypeslib.as_array((C.c_uint8 * n.value).from_address(p.value)) if n.value else np.zeros(0, np.uint8)

    def get_tensor_data(self, name: str) -> Optional[np.ndarray]:
        return self._slice(L.lib().pox_file_tensor_data, name)

    def get_scale_data(self, name: str) -> Optional[np.ndarray]:
        return self._slice(L.lib().pox_file_scale_data, name)

    def get_outlier_data(self, name: str) -> Optional[np.ndarray]:
        return self._slice(L.lib().pox_file_outlier_data, name)

    def model_config(self) -> dict:
        c = L.LlamaConfig()
        tie = C.c_int()
        L.check(L.lib().pox_file_model_config(self.handle, C.byref(c), C.byref(tie)))
        return {"hidden": c.hidden, "inter": c.intermediate, "layers": c.layers, "n_heads": c.heads,
                "n_kv_heads": c.kv_heads, "vocab": c.vocab, "rms_eps": c.rms_eps, "rope_theta": c.rope_theta,
                "tie_word_embeddings": bool(tie.value)}

    def verify_integrity(self, threads: int = 0) -> None:
        L.check(L.lib().pox_file_verify_integrity(self.handle, threads))

    def shard(self, name: str, split: int, rank: int, tp: int):
        """(data, scales, outliers or None) of rank's shard (split 0 rows, 1 columns) of an INT4 tensor."""
        sizes = [C.c_size_t(0), C.c_size_t(0), C.c_size_t(0)]
        rc = L.lib().pox_file_tensor_shard(self.handle, name.encode(), split, rank, tp, None, C.byref(sizes[0]),
                                           None, C.byref(sizes[1]), None, C.byref(sizes[2]))
        if rc not in (L.POX_OK, L.POX_ERR_LAYOUT):
            L.check(rc)
        bufs = [np.zeros(max(1, s.value), np.uint8) for s in sizes]
        L.check(L.lib().pox_file_tensor_shard(self.handle, name.encode(), split, rank, tp, bufs[0].ctypes.data,
                                              C.byref(sizes[0]), bufs[1].ctypes.data, C.byref(sizes[1]),
                                              bufs[2].ctypes.data, C.byref(sizes[2])))
        d, s, o = (b[:sz.value] for b, sz in zip(bufs, sizes))
        return d, s, (o if o.size else None)
