"""Quantize-time tools producing the .pox tensor layout (vectorised numpy, bit-exact).

These are the quantizers the reference runs before decoding (`pox quantize`,
crates/paraoxidizer-cli/src/commands.rs:559-641); the CUDA backend consumes their output. They
reproduce the reference's f32 arithmetic exactly:
  * quantize_int4_group      crates/paraoxidizer-quant/src/kernels.rs:26-82
  * quantize_int8_symmetric  kernels.rs:131-154
  * extract_and_zero_outliers / to_bytes   crates/paraoxidizer-quant/src/outlier.rs:57-110
Rust semantics kept: f32::round is round-half-away-from-zero; `clamp(..) as u8/i8` maps NaN to
0; min/max loops skip NaN and keep the first of equal values; `iter().sum()` over f32 is a
sequential left fold (numpy's add.accumulate, not its pairwise sum); f16::from_f32 is IEEE
round-to-nearest-even (numpy's float16 cast).
"""
from __future__ import annotations

import numpy as np

SIGMA = {"disabled": None, "conservative": 4.5, "automatic": 3.5, "aggressive": 2.8}


def policy_sigma(name: str):
    """OutlierPolicy::from_str_name + sigma_threshold (outlier.rs:17-34)."""
    n = name.lower()
    if n in ("disabled", "none"):
        return None
    return SIGMA.get(n, 3.5)


def _round_half_away(v: np.ndarray) -> np.ndarray:
    r = np.trunc(v)
    f = v - r  # exact in f32
    return r + np.where(np.abs(f) >= np.float32(0.5), np.sign(v), np.float32(0)).astype(np.float32)


def _round_clamp_cast(v: np.ndarray, lo: float, hi: float) -> np.ndarray:
    r = _round_half_away(v)
    r = np.where(np.isnan(r), np.float32(0), r)
    return np.clip(r, lo, hi)


def _f16_bits(a: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore", invalid="ignore"):
        return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def _first_extreme(g: np.ndarray, ext: np.ndarray) -> np.ndarray:
    """For rows whose extreme is zero, take the sign of the first zero (the Rust loop keeps the
    first of -0.0 / +0.0, which compare equal)."""
    zero = ext == 0
    if not np.any(zero):
        return ext
    rows = np.nonzero(zero)[0]
    sub = g[rows]
    first = np.argmax(sub == 0, axis=1)
    vals = sub[np.arange(rows.size), first]
    out = ext.copy()
    out[rows] = vals
    return out


def quantize_int4_group(weights: np.ndarray, group_size: int):
    """kernels.rs:26-82 -> (packed u8, scale bytes u8). Groups run over the flattened tensor;
    every group starts a fresh byte and a group of odd length pads its last high nibble with 0."""
    w = np.ascontiguousarray(weights, np.float32).reshape(-1)
    n = w.size
    gs = int(group_size)
    ng = (n + gs - 1) // gs
    full = n // gs
    packed_parts, scale_parts = [], []

    def do(gw: np.ndarray):
        # gw: [groups, len]
        finite_lo = np.where(np.isnan(gw), np.float32(np.inf), gw)
        finite_hi = np.where(np.isnan(gw), np.float32(-np.inf), gw)
        mn = _first_extreme(gw, finite_lo.min(axis=1))
        mx = _first_extreme(gw, finite_hi.max(axis=1))
        with np.errstate(invalid="ignore", over="ignore"):
            degenerate = np.abs(mx - mn) < np.float32(1e-8)
            mx = np.where(degenerate, mn + np.float32(1e-4), mx).astype(np.float32)
            scale = ((mx - mn) / np.float32(15.0)).astype(np.float32)
            v = ((gw - mn[:, None]) / scale[:, None]).astype(np.float32)
        q = _round_clamp_cast(v, 0.0, 15.0).astype(np.uint8)
        if q.shape[1] % 2:
            q = np.concatenate([q, np.zeros((q.shape[0], 1), np.uint8)], axis=1)
        packed = (q[:, 0::2] & 0x0F) | ((q[:, 1::2] & 0x0F) << 4)
        sc = np.empty((gw.shape[0], 2), np.uint16)
        sc[:, 0] = _f16_bits(scale)
        sc[:, 1] = _f16_bits(mn)
        packed_parts.append(packed.reshape(-1))
        scale_parts.append(sc.reshape(-1).view(np.uint8))

    chunk = max(1, (1 << 22) // max(gs, 1))
    for g0 in range(0, full, chunk):
        g1 = min(full, g0 + chunk)
        do(w[g0 * gs:g1 * gs].reshape(g1 - g0, gs))
    if ng > full:
        do(w[full * gs:].reshape(1, -1))
    packed = np.concatenate(packed_parts) if packed_parts else np.zeros(0, np.uint8)
    scales = np.concatenate(scale_parts) if scale_parts else np.zeros(0, np.uint8)
    return packed.astype(np.uint8), scales.astype(np.uint8)


def quantize_int8_symmetric(weights: np.ndarray):
    """kernels.rs:131-154 -> (q u8 [as i8 bits], 4-byte f32 scale)."""
    w = np.ascontiguousarray(weights, np.float32).reshape(-1)
    a = np.abs(w)
    a = np.where(np.isnan(a), np.float32(0), a)  # NaN never wins `abs > max_abs`
    max_abs = np.float32(a.max()) if a.size else np.float32(0)
    if max_abs < np.float32(1e-8):
        max_abs = np.float32(1e-4)
    scale = np.float32(max_abs / np.float32(127.0))
    with np.errstate(invalid="ignore"):
        q = _round_clamp_cast((w / scale).astype(np.float32), -127.0, 127.0).astype(np.int8)
    return q.view(np.uint8), np.array([scale], np.float32).view(np.uint8)


def quantize_int8_rows(weights: np.ndarray, rows: int, cols: int):
    """Per-output-channel INT8 (an extension; the reference's .pox INT8 is per tensor,
    kernels.rs:131-154): per row max_abs (floor 1e-4 below 1e-8), scale = max_abs / 127 stored as f16
    (round to nearest even), q = round(w / s) half away from zero, clamped to +-127, with s the f16
    scale read back. -> (q u8 [i8 bits], rows x 2 bytes of f16 scales)."""
    w = np.ascontiguousarray(weights, np.float32).reshape(rows, cols)
    a = np.abs(w)
    a = np.where(np.isnan(a), np.float32(0), a)
    max_abs = a.max(axis=1).astype(np.float32) if cols else np.zeros(rows, np.float32)
    max_abs = np.where(max_abs < np.float32(1e-8), np.float32(1e-4), max_abs).astype(np.float32)
    sh = (max_abs / np.float32(127.0)).astype(np.float32).astype(np.float16)
    s = sh.astype(np.float32)[:, None]
    with np.errstate(invalid="ignore", divide="ignore"):
        q = _round_clamp_cast((w / s).astype(np.float32), -127.0, 127.0).astype(np.int8)
    return q.reshape(-1).view(np.uint8), sh.view(np.uint8).reshape(-1)


def extract_and_zero_outliers(weights: np.ndarray, policy: str = "automatic"):
    """outlier.rs:57-85. `weights` (f32, contiguous) is zeroed in place at the outliers.
    Returns (indices u32, f16 value bits) or None."""
    sig = policy_sigma(policy)
    if sig is None or weights.size == 0:
        return None
    flat = weights.reshape(-1)
    assert flat.dtype == np.float32
    n = np.float32(flat.size)
    total = np.add.accumulate(flat, dtype=np.float32)[-1]
    mean = np.float32(total / n)
    d = (flat - mean).astype(np.float32)
    var_sum = np.add.accumulate(d * d, dtype=np.float32)[-1]
    std = np.float32(np.sqrt(np.float32(var_sum / n)))
    thr = np.float32(np.float32(sig) * std)
    hit = np.abs(d) > thr
    idx = np.nonzero(hit)[0].astype(np.uint32)
    if idx.size == 0:
        return None
    vals = _f16_bits(flat[idx])
    flat[idx] = np.float32(0.0)
    return idx, vals


def outliers_to_bytes(idx: np.ndarray, vals: np.ndarray) -> np.ndarray:
    """outlier.rs:99-110: count u32 | indices u32[count] | values f16[count], little endian."""
    idx = np.ascontiguousarray(idx, np.uint32)
    vals = np.ascontiguousarray(vals, np.uint16)
    return np.concatenate([np.array([idx.size], "<u4").view(np.uint8), idx.astype("<u4").view(np.uint8),
                           vals.astype("<u2").view(np.uint8)])


def quantize_int4_tensor(w: np.ndarray, group_size: int = 128, outlier_policy: str = "disabled"):
    """The per-tensor pipeline of `pox quantize` (commands.rs:559-629): extract outliers (on a
    copy), then INT4-quantize the remainder. Returns (packed, scales, outlier bytes or None)."""
    w = np.array(w, np.float32, copy=True).reshape(-1)
    tab = extract_and_zero_outliers(w, outlier_policy)
    packed, scales = quantize_int4_group(w, group_size)
    return packed, scales, None if tab is None else outliers_to_bytes(*tab)
