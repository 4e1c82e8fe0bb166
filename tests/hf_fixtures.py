"""Writes small Hugging Face Llama checkpoints (config.json + safetensors) for
the loader tests, and the matching CPU-oracle model.

The safetensors format is written directly: an 8-byte little-endian header
length, a JSON header {name: {dtype, shape, data_offsets}}, then the raw
little-endian payload. Weights are N(0, 0.02) (BASELINE's random-init recipe),
stored as BF16, F16 or F32; norm weights are 1 + N(0, 0.1).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

TINY_HF = dict(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
               num_key_value_heads=2, intermediate_size=768, rms_norm_eps=1e-5, rope_theta=10000.0,
               max_position_embeddings=256, tie_word_embeddings=False)


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def stored_values(a: np.ndarray, dtype: str) -> np.ndarray:
    """The float32 values a tensor has once stored as `dtype`."""
    if dtype == "BF16":
        return (_bf16_bits(a).astype(np.uint32) << 16).view(np.float32)
    if dtype == "F16":
        return a.astype(np.float16).astype(np.float32)
    return a.astype(np.float32)


def write_safetensors(path: Path, tensors: dict[str, np.ndarray], dtype: str) -> None:
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        if dtype == "BF16":
            b = _bf16_bits(a).tobytes()
        elif dtype == "F16":
            b = a.astype(np.float16).tobytes()
        else:
            b = a.astype(np.float32).tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {"format": "pt"}
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def make_weights(cfg: dict, seed: int = 0) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    H, I, V = cfg["hidden_size"], cfg["intermediate_size"], cfg["vocab_size"]
    nq, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    d = H // nq
    w = {"model.embed_tokens.weight": rng.normal(0, 0.02, (V, H)).astype(np.float32)}
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}."
        w[p + "input_layernorm.weight"] = (1 + rng.normal(0, 0.1, H)).astype(np.float32)
        w[p + "post_attention_layernorm.weight"] = (1 + rng.normal(0, 0.1, H)).astype(np.float32)
        for n, shp in (("self_attn.q_proj", (nq * d, H)), ("self_attn.k_proj", (nkv * d, H)),
                       ("self_attn.v_proj", (nkv * d, H)), ("self_attn.o_proj", (H, nq * d)),
                       ("mlp.gate_proj", (I, H)), ("mlp.up_proj", (I, H)), ("mlp.down_proj", (H, I))):
            w[p + n + ".weight"] = rng.normal(0, 0.02, shp).astype(np.float32)
    w["model.norm.weight"] = (1 + rng.normal(0, 0.1, H)).astype(np.float32)
    if not cfg.get("tie_word_embeddings"):
        w["lm_head.weight"] = rng.normal(0, 0.02, (V, H)).astype(np.float32)
    return w


def write_checkpoint(root: Path, cfg: dict, weights: dict[str, np.ndarray], dtype: str = "BF16",
                     shards: int = 1) -> Path:
    root.mkdir(parents=True, exist_ok=True)
    (root / "config.json").write_text(json.dumps({"architectures": ["LlamaForCausalLM"], "model_type": "llama",
                                                  "torch_dtype": "bfloat16", **cfg}))
    names = list(weights)
    if shards == 1:
        write_safetensors(root / "model.safetensors", weights, dtype)
    else:
        wm = {}
        for i in range(shards):
            part = names[i::shards]
            fn = f"model-{i + 1:05d}-of-{shards:05d}.safetensors"
            write_safetensors(root / fn, {n: weights[n] for n in part}, dtype)
            wm.update({n: fn for n in part})
        (root / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    return root


def oracle_model(cfg: dict, weights: dict[str, np.ndarray], dtype: str, weight_format: int, max_seq: int):
    """The CPU oracle of what am_model_load builds from this checkpoint: the
    stored values, quantized with the oracle's restatement of the loader's
    quantizer (INT4 / INT8) or kept (plain), bf16 activations."""
    import oracle
    from aethermind_b200 import _lib as L
    from aethermind_b200.session import ModelConfig

    H = cfg["hidden_size"]
    tied = cfg.get("tie_word_embeddings", False) or "lm_head.weight" not in weights
    mc = ModelConfig(vocab=cfg["vocab_size"], hidden=H, layers=cfg["num_hidden_layers"],
                     n_q_heads=cfg["num_attention_heads"], n_kv_heads=cfg["num_key_value_heads"],
                     head_dim=H // cfg["num_attention_heads"], inter=cfg["intermediate_size"],
                     rope_theta=cfg["rope_theta"], rms_eps=cfg["rms_norm_eps"], max_seq=max_seq,
                     weight_format=weight_format, tied_embeddings=tied and weight_format != L.WFMT_INT4)
    om = oracle.OracleModel(mc, act_bf16=True)
    v = {n: stored_values(a, dtype) for n, a in weights.items()}
    bf = oracle.bf16_round

    def lin(a):
        n, k = a.shape
        if weight_format == L.WFMT_INT4:
            q, s = oracle.quantize_w4(a)
            return om.linear(2, n, k, q=q, s=s)
        if weight_format == L.WFMT_INT8:
            q, s = oracle.quantize_w8(a)
            return om.linear(1, n, k, q=q, s=s)
        return om.linear(0, n, k, w=bf(a))

    head = v["model.embed_tokens.weight"] if tied else v["lm_head.weight"]
    om.m.lm_head = lin(head)
    om.m.embed = None if (tied and weight_format == L.WFMT_INT8) else om._hold(bf(v["model.embed_tokens.weight"]))
    om.m.final_norm = om.set_vec(bf(v["model.norm.weight"]))
    names = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj", "wo": "self_attn.o_proj",
             "wg": "mlp.gate_proj", "wu": "mlp.up_proj", "wd": "mlp.down_proj"}
    for l in range(mc.layers):
        p = f"model.layers.{l}."
        Ly = om.layers[l]
        Ly.attn_norm = om.set_vec(bf(v[p + "input_layernorm.weight"]))
        Ly.mlp_norm = om.set_vec(bf(v[p + "post_attention_layernorm.weight"]))
        for ours, theirs in names.items():
            setattr(Ly, ours, lin(v[p + theirs + ".weight"]))
    return om
