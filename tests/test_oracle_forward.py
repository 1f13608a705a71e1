"""The oracle's forward_token (engine.rs:411-716) against a float64 numpy restatement of the same
decode step over the same dequantized weights (CPU). The weights come from the oracle's
dequantization (bit-exact, pinned separately); everything after it is recomputed here in float64:
embedding, per layer RMSNorm -> q/k/v -> interleaved RoPE -> GQA attention over the cache -> o
projection + residual -> RMSNorm -> SwiGLU MLP + residual, then the final RMSNorm and the lm_head.
This pins how the oracle composes the step, which the GPU decode tests use as their reference."""
import numpy as np

from oracle import oracle as O
from paraoxidizer_b200.synth import make_llama, oracle_weights

CFG = {"hidden": 256, "inter": 512, "layers": 2, "n_heads": 8, "n_kv_heads": 2, "vocab": 300,
       "rms_eps": 1e-5, "rope_theta": 500000.0}


def f16(bits):
    return np.asarray(bits, np.uint16).view(np.float16).astype(np.float64)


def dequant(t):
    d = O.dequantize_int4_group(t["packed"], t["scales"], t["group_size"], t["rows"] * t["cols"])
    if t.get("outliers") is not None:
        O.outliers_apply(t["outliers"][0], t["outliers"][1], d)
    return d.astype(np.float64).reshape(t["rows"], t["cols"])


def rms(x, w_bits, eps):
    return x / np.sqrt(np.mean(x * x) + eps) * f16(w_bits)


def rope(v, n, hd, pos, theta):
    i = np.arange(hd // 2)
    freq = np.float32(1.0) / np.power(np.float32(theta), (2 * i).astype(np.float32) / np.float32(hd))
    ang = (np.float32(pos) * freq.astype(np.float32)).astype(np.float64)
    c, s = np.cos(ang), np.sin(ang)
    v = v.reshape(n, hd // 2, 2)
    out = np.empty_like(v)
    out[..., 0] = v[..., 0] * c - v[..., 1] * s
    out[..., 1] = v[..., 0] * s + v[..., 1] * c
    return out.ravel()


def test_forward_token_matches_float64_restatement():
    w = oracle_weights(make_llama(CFG, seed=5, outlier_policy="aggressive", norm_jitter=0.1))
    H, nq, nkv, V = CFG["hidden"], CFG["n_heads"], CFG["n_kv_heads"], CFG["vocab"]
    hd, G, eps, theta = H // nq, nq // nkv, CFG["rms_eps"], CFG["rope_theta"]
    Ws = [{k: dequant(lay[k]) for k in ("q", "k", "v", "o", "gate", "up", "down")} for lay in w["layers"]]
    emb = f16(w["embed"]).reshape(V, H)
    head = f16(w["lm_head"]).reshape(V, H)
    om = O.OracleModel(CFG, w, max_seq=16)
    tokens = [3, 141, 59, 26, 5, 35, 89, 79, 32, 38, 46, 264]
    kc = [np.zeros((len(tokens), nkv, hd)) for _ in Ws]
    vc = [np.zeros((len(tokens), nkv, hd)) for _ in Ws]
    worst = 0.0
    for pos, tok in enumerate(tokens):
        got = om.forward_token(tok, pos)
        x = emb[tok].copy()
        for l, W in enumerate(Ws):
            h = rms(x, w["layers"][l]["attn_norm"], eps)
            q = rope(W["q"] @ h, nq, hd, pos, theta)
            kc[l][pos] = rope(W["k"] @ h, nkv, hd, pos, theta).reshape(nkv, hd)
            vc[l][pos] = (W["v"] @ h).reshape(nkv, hd)
            att = np.zeros(nq * hd)
            for hq in range(nq):
                s = kc[l][:pos + 1, hq // G] @ q[hq * hd:(hq + 1) * hd] / np.sqrt(hd)
                p = np.exp(s - s.max())
                att[hq * hd:(hq + 1) * hd] = (p / p.sum()) @ vc[l][:pos + 1, hq // G]
            x = x + W["o"] @ att
            h = rms(x, w["layers"][l]["mlp_norm"], eps)
            g, u = W["gate"] @ h, W["up"] @ h
            x = x + W["down"] @ (g / (1 + np.exp(-g)) * u)
        ref = head @ rms(x, w["final_norm"], eps)
        worst = max(worst, float(np.max(np.abs(got - ref)) / np.max(np.abs(ref))))
        assert int(np.argmax(got)) == int(np.argmax(ref)), pos
    assert worst <= 1e-4, worst  # measured: 7e-7
