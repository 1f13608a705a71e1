"""The oracle's forward_token (restating crates/paraoxidizer-runtime/src/engine.rs:411-716) equals the
composition of the oracle's separately restated steps, in the reference's order: embedding row
(engine.rs:420-524), per layer RMSNorm (:294-350), q/k/v projections, interleaved RoPE (:353-408),
KvCache store (:38-50), GQA attention over 0..=pos (:580-641), o projection + residual
(:644-648), RMSNorm, gate/up, SwiGLU (:671-677), down + residual (:682-684); final RMSNorm and the
F16 lm_head (:696-707). CPU only."""
import numpy as np

from oracle import oracle as O
from paraoxidizer_b200.synth import make_llama, oracle_weights

CFG = {"hidden": 256, "inter": 512, "layers": 2, "n_heads": 8, "n_kv_heads": 2, "vocab": 300, "rms_eps": 1e-5,
       "rope_theta": 500000.0}


def compose(cfg, w, tokens):
    H, I, V = cfg["hidden"], cfg["inter"], cfg["vocab"]
    nq, nkv = cfg["n_heads"], cfg["n_kv_heads"]
    hd = H // nq
    L = cfg["layers"]
    kc = [np.zeros((len(tokens), nkv * hd), np.float32) for _ in range(L)]
    vc = [np.zeros((len(tokens), nkv * hd), np.float32) for _ in range(L)]
    out = []
    for pos, tok in enumerate(tokens):
        x = O.f16_bits_to_f32(w["embed"].reshape(V, H)[tok % V]).astype(np.float32)
        for l, lay in enumerate(w["layers"]):
            P = lambda name, v: O.gemv_int4(lay[name]["packed"], lay[name]["scales"], 128, lay[name]["rows"],
                                            lay[name]["cols"], lay[name]["outliers"], v)
            nx = O.rms_norm(x, lay["attn_norm"], cfg["rms_eps"])
            q, k, v = P("q", nx), P("k", nx), P("v", nx)
            q, k = O.rope(q, k, nq, nkv, hd, pos, cfg["rope_theta"])
            kc[l][pos], vc[l][pos] = k, v
            att = O.attention(q, kc[l].reshape(-1), vc[l].reshape(-1), nq, nkv, hd, pos)
            x = x + P("o", att)
            nx = O.rms_norm(x, lay["mlp_norm"], cfg["rms_eps"])
            x = x + P("down", O.swiglu(P("gate", nx), P("up", nx)))
        x = O.rms_norm(x, w["final_norm"], cfg["rms_eps"])
        lg = O.gemv_f16(w["lm_head"], V, H, x)
        out.append(np.where(np.isfinite(lg), lg, 0).astype(np.float32))
    return out


def test_forward_token_is_the_composition_of_its_steps():
    w = oracle_weights(make_llama(CFG, seed=4, outlier_policy="automatic", norm_jitter=0.1))
    tokens = [5, 299, 17, 42, 1000, 3]  # 1000 wraps to 1000 % vocab (engine.rs:422)
    model = O.OracleModel(CFG, w, max_seq=len(tokens))
    ref = compose(CFG, w, tokens)
    for pos, tok in enumerate(tokens):
        got = model.forward_token(tok, pos)
        assert np.array_equal(got.view(np.uint32), ref[pos].view(np.uint32)), pos
