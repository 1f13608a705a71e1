"""Oracle wrapper -- TEST INFRASTRUCTURE ONLY.

ctypes bindings over ``oracle/build/libpox_oracle.so`` (the single-threaded C restatement of
ParaOxidizer's CPU decode path in ``oracle/pox_oracle.c``). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import this module; the
product package never does.

Every function names the reference function it mirrors (paths relative to the reference
repository root).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "libpox_oracle.so")
_lib = None

_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def build() -> str:
    """Compile the oracle with its Makefile (gcc, no FMA contraction)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        L.pox_oracle_f32_to_f16.restype = C.c_uint16
        L.pox_oracle_f32_to_f16.argtypes = [C.c_float]
        L.pox_oracle_f16_to_f32.restype = C.c_float
        L.pox_oracle_f16_to_f32.argtypes = [C.c_uint16]
        L.pox_oracle_f32_to_f16_array.argtypes = [_f32p, _u16p, _sz]
        L.pox_oracle_f16_to_f32_array.argtypes = [_u16p, _f32p, _sz]
        L.pox_oracle_quantize_int4_group.restype = _sz
        L.pox_oracle_quantize_int4_group.argtypes = [_f32p, _sz, _sz, _u8p, _u8p]
        L.pox_oracle_dequantize_int4_group.restype = C.c_int
        L.pox_oracle_dequantize_int4_group.argtypes = [_u8p, _sz, _u8p, _sz, _sz, _sz, _f32p, _sz]
        L.pox_oracle_quantize_int8_symmetric.argtypes = [_f32p, _sz, _u8p, _u8p]
        L.pox_oracle_dequantize_int8_symmetric.restype = C.c_int
        L.pox_oracle_dequantize_int8_symmetric.argtypes = [_u8p, _sz, _u8p, _sz, _f32p, _sz]
        L.pox_oracle_dot_x86.restype = C.c_float
        L.pox_oracle_dot_x86.argtypes = [_f32p, _f32p, _sz]
        L.pox_oracle_dot_neon.restype = C.c_float
        L.pox_oracle_dot_neon.argtypes = [_f32p, _f32p, _sz]
        L.pox_oracle_extract_and_zero_outliers.restype = _sz
        L.pox_oracle_extract_and_zero_outliers.argtypes = [_f32p, _sz, C.c_float, _u32p, _u16p]
        L.pox_oracle_outliers_to_bytes.restype = _sz
        L.pox_oracle_outliers_to_bytes.argtypes = [_u32p, _u16p, _sz, _u8p]
        L.pox_oracle_outliers_from_bytes.restype = C.c_long
        L.pox_oracle_outliers_from_bytes.argtypes = [_u8p, _sz, _u32p, _u16p, _sz]
        L.pox_oracle_outliers_apply.argtypes = [_u32p, _u16p, _sz, _f32p, _sz]
        L.pox_oracle_gemv_int4.restype = C.c_int
        L.pox_oracle_gemv_int4.argtypes = [_u8p, _sz, _u8p, _sz, _sz, _sz, _sz, C.c_void_p, C.c_void_p,
                                           _sz, _f32p, _sz, _f32p, _sz, C.c_int]
        L.pox_oracle_gemv_int8.restype = C.c_int
        L.pox_oracle_gemv_int8.argtypes = [_u8p, _sz, _u8p, _sz, _sz, _sz, _f32p, _sz, _f32p, _sz]
        L.pox_oracle_quantize_int8_rows.argtypes = [_f32p, _sz, _sz, _u8p, _u8p]
        L.pox_oracle_dequantize_int8_rows.restype = C.c_int
        L.pox_oracle_dequantize_int8_rows.argtypes = [_u8p, _sz, _sz, _u8p, _sz, _f32p]
        L.pox_oracle_gemv_int8_rows.restype = C.c_int
        L.pox_oracle_gemv_int8_rows.argtypes = [_u8p, _sz, _sz, _u8p, _sz, _f32p, _f32p]
        L.pox_oracle_gemv_f16.argtypes = [_u16p, _sz, _sz, _f32p, _f32p]
        L.pox_oracle_rms_norm.argtypes = [_f32p, _sz, C.c_void_p, C.c_float]
        L.pox_oracle_rope.argtypes = [_f32p, _sz, _f32p, _sz, _sz, _sz, C.c_float]
        L.pox_oracle_attention.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _f32p]
        L.pox_oracle_swiglu.argtypes = [_f32p, _f32p, _f32p, _sz]
        L.pox_oracle_argmax.restype = C.c_uint32
        L.pox_oracle_argmax.argtypes = [_f32p, _sz]
        L.pox_oracle_forward_token.restype = C.c_int
        L.pox_oracle_forward_token.argtypes = [C.c_void_p, C.c_uint32, _sz, _f32p]
        _lib = L
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# --- binary16 (half 2.7.1 f16::from_f32 / to_f32) -------------------------------------------
def f32_to_f16_bits(a) -> np.ndarray:
    a = _c(a, np.float32).ravel()
    out = np.empty(a.size, np.uint16)
    lib().pox_oracle_f32_to_f16_array(a, out, a.size)
    return out


def f16_bits_to_f32(a) -> np.ndarray:
    a = _c(a, np.uint16).ravel()
    out = np.empty(a.size, np.float32)
    lib().pox_oracle_f16_to_f32_array(a, out, a.size)
    return out


# --- crates/paraoxidizer-quant/src/kernels.rs ------------------------------------------------
def quantize_int4_group(weights, group_size: int):
    """kernels.rs:26-82 -> (packed bytes, scale bytes)."""
    w = _c(weights, np.float32).ravel()
    n = w.size
    ng = (n + group_size - 1) // group_size
    packed = np.zeros((n + ng) // 2 + 1, np.uint8)
    scales = np.zeros(ng * 4, np.uint8)
    np_ = lib().pox_oracle_quantize_int4_group(w, n, group_size, packed, scales)
    return packed[:np_].copy(), scales


def dequantize_int4_group(packed, scales, group_size: int, numel: int) -> np.ndarray:
    """kernels.rs:85-128."""
    p = _c(packed, np.uint8)
    s = _c(scales, np.uint8)
    out = np.zeros(max(numel, 1), np.float32)
    rc = lib().pox_oracle_dequantize_int4_group(p, p.size, s, s.size, group_size, numel, out, out.size)
    if rc != 0:
        raise ValueError("dequantize_int4_group: Err")
    return out[:numel]


def quantize_int8_symmetric(weights):
    """kernels.rs:131-154 -> (q bytes, 4-byte f32 scale)."""
    w = _c(weights, np.float32).ravel()
    q = np.zeros(max(w.size, 1), np.uint8)
    s = np.zeros(4, np.uint8)
    lib().pox_oracle_quantize_int8_symmetric(w, w.size, q, s)
    return q[: w.size].copy(), s


def dequantize_int8_symmetric(q, scales) -> np.ndarray:
    """kernels.rs:157-173."""
    q = _c(q, np.uint8)
    s = _c(scales, np.uint8)
    out = np.zeros(max(q.size, 1), np.float32)
    if lib().pox_oracle_dequantize_int8_symmetric(q, q.size, s, s.size, out, out.size) != 0:
        raise ValueError("dequantize_int8_symmetric: Err")
    return out[: q.size]


def quantize_int8_rows(weights, rows: int, cols: int):
    """Per-output-channel INT8 (the extension: the reference's rules per row, f16 row scales)
    -> (q bytes, rows x 2 bytes of f16 scales)."""
    w = _c(weights, np.float32).ravel()
    q = np.zeros(max(w.size, 1), np.uint8)
    s = np.zeros(max(2 * rows, 1), np.uint8)
    lib().pox_oracle_quantize_int8_rows(w, rows, cols, q, s)
    return q[: w.size].copy(), s[: 2 * rows].copy()


def dequantize_int8_rows(q, scales, rows: int, cols: int) -> np.ndarray:
    q = _c(q, np.uint8)
    s = _c(scales, np.uint8)
    out = np.zeros(max(rows * cols, 1), np.float32)
    if lib().pox_oracle_dequantize_int8_rows(q, rows, cols, s, s.size, out) != 0:
        raise ValueError("dequantize_int8_rows: scales too short")
    return out[: rows * cols]


def gemv_int8_rows(q, scales, rows: int, cols: int, x) -> np.ndarray:
    """gemv_int8's arithmetic (kernels.rs:229-255) with the row's own f16 scale."""
    q = _c(q, np.uint8)
    s = _c(scales, np.uint8)
    x = _c(x, np.float32)
    y = np.zeros(rows, np.float32)
    if lib().pox_oracle_gemv_int8_rows(q, rows, cols, s, s.size, x, y) != 0:
        raise ValueError("gemv_int8_rows: scales too short")
    return y


def dot_product_simd(a, b, neon: bool = False) -> float:
    """kernels.rs:259-317 (x86 order by default, aarch64 order with neon=True)."""
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    n = min(a.size, b.size)
    f = lib().pox_oracle_dot_neon if neon else lib().pox_oracle_dot_x86
    return float(f(a, b, n))


# --- crates/paraoxidizer-quant/src/outlier.rs -------------------------------------------------
SIGMA = {"disabled": None, "conservative": 4.5, "automatic": 3.5, "aggressive": 2.8}


def sigma_for_policy(name: str):
    """outlier.rs:17-34: unknown names map to Automatic."""
    n = name.lower()
    if n == "none":
        n = "disabled"
    return SIGMA.get(n, 3.5)


def extract_and_zero_outliers(weights: np.ndarray, policy: str = "automatic"):
    """outlier.rs:57-85. Zeroes `weights` (float32, modified in place) and returns
    (indices u32, values f16-bits) or None."""
    sig = sigma_for_policy(policy)
    if sig is None or weights.size == 0:
        return None
    assert weights.dtype == np.float32 and weights.flags.c_contiguous
    flat = weights.reshape(-1)
    idx = np.zeros(flat.size, np.uint32)
    val = np.zeros(flat.size, np.uint16)
    cnt = lib().pox_oracle_extract_and_zero_outliers(flat, flat.size, sig, idx, val)
    if cnt == 0:
        return None
    return idx[:cnt].copy(), val[:cnt].copy()


def outliers_to_bytes(idx, val) -> np.ndarray:
    """outlier.rs:99-110."""
    idx = _c(idx, np.uint32)
    val = _c(val, np.uint16)
    out = np.zeros(4 + 6 * idx.size, np.uint8)
    lib().pox_oracle_outliers_to_bytes(idx, val, idx.size, out)
    return out


def outliers_from_bytes(b):
    """outlier.rs:112-127 -> (idx, val); raises on a truncated table (the reference's Err)."""
    b = _c(b, np.uint8)
    cap = max((b.size - 4) // 6, 0) + 1
    idx = np.zeros(cap, np.uint32)
    val = np.zeros(cap, np.uint16)
    n = lib().pox_oracle_outliers_from_bytes(b, b.size, idx, val, cap)
    if n < 0:
        raise ValueError("outlier table truncated")
    return idx[:n].copy(), val[:n].copy()


def outliers_apply(idx, val, deq: np.ndarray) -> None:
    """outlier.rs:88-95 apply_to (in place)."""
    idx = _c(idx, np.uint32)
    val = _c(val, np.uint16)
    lib().pox_oracle_outliers_apply(idx, val, idx.size, deq, deq.size)


# --- GEMV ---------------------------------------------------------------------------------
def gemv_int4(packed, scales, group_size, rows, cols, outliers, x, neon=False) -> np.ndarray:
    """kernels.rs:177-226. `outliers` is None or (idx, val)."""
    p = _c(packed, np.uint8)
    s = _c(scales, np.uint8)
    x = _c(x, np.float32).ravel()
    y = np.zeros(max(rows, 1), np.float32)
    if outliers is not None and len(outliers[0]):
        oi = _c(outliers[0], np.uint32)
        ov = _c(outliers[1], np.uint16)
        oip, ovp, oc = oi.ctypes.data, ov.ctypes.data, oi.size
    else:
        oi = ov = None
        oip = ovp = None
        oc = 0
    rc = lib().pox_oracle_gemv_int4(p, p.size, s, s.size, group_size, rows, cols, oip, ovp, oc, x, x.size,
                                    y, y.size, 1 if neon else 0)
    if rc != 0:
        raise ValueError("gemv_int4: Err")
    return y[:rows]


def gemv_int8(q, scales, rows, cols, x) -> np.ndarray:
    """kernels.rs:229-255."""
    q = _c(q, np.uint8)
    s = _c(scales, np.uint8)
    x = _c(x, np.float32).ravel()
    y = np.zeros(max(rows, 1), np.float32)
    if lib().pox_oracle_gemv_int8(q, q.size, s, s.size, rows, cols, x, x.size, y, y.size) != 0:
        raise ValueError("gemv_int8: Err")
    return y[:rows]


def gemv_f16(w_bits, rows, cols, x) -> np.ndarray:
    """engine.rs:235-250 F16 projection."""
    w = _c(w_bits, np.uint16).ravel()
    x = _c(x, np.float32).ravel()
    y = np.zeros(rows, np.float32)
    lib().pox_oracle_gemv_f16(w, rows, cols, x, y)
    return y


# --- engine pieces ------------------------------------------------------------------------
def rms_norm(x, w_bits=None, eps=1e-5) -> np.ndarray:
    """engine.rs:294-350."""
    x = _c(x, np.float32).copy()
    wb = None if w_bits is None else _c(w_bits, np.uint16)
    lib().pox_oracle_rms_norm(x, x.size, None if wb is None else wb.ctypes.data, eps)
    return x


def rope(q, k, nq, nkv, head_dim, pos, theta):
    """engine.rs:353-408 (interleaved pairs)."""
    q = _c(q, np.float32).copy()
    k = _c(k, np.float32).copy()
    lib().pox_oracle_rope(q, nq, k, nkv, head_dim, pos, theta)
    return q, k


def attention(q, k_cache, v_cache, nq, nkv, head_dim, pos) -> np.ndarray:
    """engine.rs:580-641; caches [pos+1][nkv][head_dim] f32."""
    q = _c(q, np.float32).ravel()
    kc = _c(k_cache, np.float32).ravel()
    vc = _c(v_cache, np.float32).ravel()
    out = np.zeros(nq * head_dim, np.float32)
    lib().pox_oracle_attention(q, kc, vc, nq, nkv, head_dim, pos, out)
    return out


def swiglu(g, u) -> np.ndarray:
    g = _c(g, np.float32)
    u = _c(u, np.float32)
    out = np.zeros_like(g)
    lib().pox_oracle_swiglu(g, u, out, g.size)
    return out


def argmax(logits) -> int:
    """sampler.rs:55-65."""
    l = _c(logits, np.float32)
    return int(lib().pox_oracle_argmax(l, l.size))


# --- forward_token ------------------------------------------------------------------------
class _I4(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("packed_len", C.c_size_t), ("scales", C.c_void_p),
                ("scale_len", C.c_size_t), ("out_idx", C.c_void_p), ("out_val", C.c_void_p),
                ("out_count", C.c_size_t), ("rows", C.c_size_t), ("cols", C.c_size_t),
                ("group_size", C.c_size_t)]


class _Model(C.Structure):
    _fields_ = [("hidden", C.c_size_t), ("inter", C.c_size_t), ("layers", C.c_size_t),
                ("n_heads", C.c_size_t), ("n_kv_heads", C.c_size_t), ("vocab", C.c_size_t),
                ("max_seq", C.c_size_t), ("rms_eps", C.c_float), ("rope_theta", C.c_float),
                ("kv_f16", C.c_int), ("embed", C.c_void_p), ("lm_head", C.c_void_p),
                ("final_norm", C.c_void_p), ("attn_norm", C.c_void_p), ("mlp_norm", C.c_void_p),
                ("proj", C.c_void_p), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p)]


class OracleModel:
    """engine.rs:411-716 forward_token over an in-memory Llama model (INT4 projections with
    optional outlier tables, F16 embedding / lm_head / norms) and the reference's contiguous
    f32 KvCache (engine.rs:10-84); kv_f16 rounds K/V to f16 on store."""

    PROJ = ("q", "k", "v", "o", "gate", "up", "down")

    def __init__(self, cfg: dict, weights: dict, max_seq: int, kv_f16: bool = False):
        self.cfg = cfg
        self._keep = []
        L = cfg["layers"]
        H = cfg["hidden"]
        hd = H // cfg["n_heads"]
        kvd = cfg["n_kv_heads"] * hd
        self.k_cache = np.zeros(L * max_seq * kvd, np.float32)
        self.v_cache = np.zeros(L * max_seq * kvd, np.float32)
        projs = (_I4 * (L * 7))()
        for l in range(L):
            for j, name in enumerate(self.PROJ):
                t = weights["layers"][l][name]
                p = _c(t["packed"], np.uint8)
                s = _c(t["scales"], np.uint8)
                self._keep += [p, s]
                e = projs[l * 7 + j]
                e.packed, e.packed_len = p.ctypes.data, p.size
                e.scales, e.scale_len = s.ctypes.data, s.size
                e.rows, e.cols, e.group_size = t["rows"], t["cols"], t["group_size"]
                if t.get("outliers") is not None:
                    oi = _c(t["outliers"][0], np.uint32)
                    ov = _c(t["outliers"][1], np.uint16)
                    self._keep += [oi, ov]
                    e.out_idx, e.out_val, e.out_count = oi.ctypes.data, ov.ctypes.data, oi.size
        an = (C.c_void_p * L)()
        mn = (C.c_void_p * L)()
        for l in range(L):
            a = _c(weights["layers"][l]["attn_norm"], np.uint16)
            b = _c(weights["layers"][l]["mlp_norm"], np.uint16)
            self._keep += [a, b]
            an[l], mn[l] = a.ctypes.data, b.ctypes.data
        emb = _c(weights["embed"], np.uint16)
        head = _c(weights["lm_head"], np.uint16)
        fn = _c(weights["final_norm"], np.uint16)
        self._keep += [emb, head, fn, projs, an, mn]
        m = _Model()
        m.hidden, m.inter, m.layers = H, cfg["inter"], L
        m.n_heads, m.n_kv_heads, m.vocab, m.max_seq = cfg["n_heads"], cfg["n_kv_heads"], cfg["vocab"], max_seq
        m.rms_eps = np.float32(cfg.get("rms_eps", 1e-5))
        m.rope_theta = np.float32(cfg.get("rope_theta", 500000.0))
        m.kv_f16 = 1 if kv_f16 else 0
        m.embed, m.lm_head, m.final_norm = emb.ctypes.data, head.ctypes.data, fn.ctypes.data
        m.attn_norm, m.mlp_norm = C.cast(an, C.c_void_p), C.cast(mn, C.c_void_p)
        m.proj = C.cast(projs, C.c_void_p)
        m.k_cache, m.v_cache = self.k_cache.ctypes.data, self.v_cache.ctypes.data
        self._m = m

    def forward_token(self, token: int, pos: int) -> np.ndarray:
        logits = np.zeros(self.cfg["vocab"], np.float32)
        if lib().pox_oracle_forward_token(C.byref(self._m), token, pos, logits) != 0:
            raise ValueError("forward_token: Err")
        return logits
