"""Model fixtures shared by the GPU parity tests and the smoke entry point.

The tiny fp32 model is BASELINE config 0: vocab 512, hidden 256, 2 layers,
4 query / 2 KV heads (head_dim 64), SwiGLU 688, weights ~N(0, 0.02) drawn
from numpy's default_rng(0) in the order embed, per layer wq wk wv wo wg wu wd,
then lm_head; norm weights are 1.
"""
from __future__ import annotations

import numpy as np

# Near-tie threshold for bf16 models (logits stored in bf16, 0.03125 apart in
# [4, 8)): 4 bf16 ulps there.
NEAR_TIE_BF16 = 0.125


def tiny_weights(cfg, seed: int = 0) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    H, d = cfg.hidden, cfg.head_dim
    w: dict[str, np.ndarray] = {}
    w["embed"] = rng.normal(0, 0.02, (cfg.vocab, H)).astype(np.float32)
    shapes = {"wq": (cfg.n_q_heads * d, H), "wk": (cfg.n_kv_heads * d, H), "wv": (cfg.n_kv_heads * d, H),
              "wo": (H, cfg.n_q_heads * d), "wg": (cfg.inter, H), "wu": (cfg.inter, H), "wd": (H, cfg.inter)}
    for l in range(cfg.layers):
        for name, shp in shapes.items():
            w[f"layers.{l}.{name}"] = rng.normal(0, 0.02, shp).astype(np.float32)
        w[f"layers.{l}.attn_norm"] = np.ones(H, np.float32)
        w[f"layers.{l}.mlp_norm"] = np.ones(H, np.float32)
    w["lm_head"] = rng.normal(0, 0.02, (cfg.vocab, H)).astype(np.float32)
    w["final_norm"] = np.ones(H, np.float32)
    return w


def tiny_oracle_model(cfg, w):
    import oracle

    om = oracle.OracleModel(cfg, act_bf16=False)
    om.m.embed = om._hold(w["embed"])
    om.m.lm_head = om.linear(0, cfg.vocab, cfg.hidden, w=w["lm_head"])
    om.m.final_norm = om.set_vec(w["final_norm"])
    for l in range(cfg.layers):
        Ly = om.layers[l]
        Ly.attn_norm = om.set_vec(w[f"layers.{l}.attn_norm"])
        Ly.mlp_norm = om.set_vec(w[f"layers.{l}.mlp_norm"])
        for name in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            a = w[f"layers.{l}.{name}"]
            setattr(Ly, name, om.linear(0, a.shape[0], a.shape[1], w=a))
    return om


def tiny_prompt(cfg, seed: int = 0, length: int = 16) -> np.ndarray:
    rng = np.random.default_rng(seed + 1)
    return rng.integers(0, cfg.vocab, length).astype(np.uint32)


def load_tiny_into_engine(model, w):
    # dict order sets every layer's "wg" before its "wu" (the fused gate/up pack needs both)
    for name, arr in w.items():
        model.set_weight(name, arr)


def walk_greedy(sess, prompt, ref, gaps, near_tie):
    """Compares the engine with the oracle's greedy sequence `ref` at every
    position; returns the positions where a near-tie flipped the token."""
    flips = []
    start = 0
    while start < len(ref):
        pre = np.concatenate([prompt, ref[:start].astype(np.uint32)])
        got = sess.generate(pre, len(ref) - start)
        for j, (a, b) in enumerate(zip(got.tolist(), ref[start:].tolist())):
            i = start + j
            if a != b:
                assert gaps[i] < near_tie, (f"position {i}: engine {a} != oracle {b} with oracle gap "
                                            f"{gaps[i]:.4g} >= {near_tie}")
                flips.append(i)
                start = i + 1
                break
        else:
            start = len(ref)
    return flips
