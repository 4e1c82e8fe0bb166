"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

ctypes front end of:
  * liboracle.so: this project's plain-C restatement of the reference engine's
    Llama hot path (am_oracle.c; citations per function there);
  * _ref/libam_ref_bridge.so: the reference engine's own CPU kernels compiled
    from its sources (RMSNorm, Add, Embedding, SiLU-Mul const-eval, KV layout,
    BFloat16 conversion).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, as the checker / reported CPU baseline. The product
(aethermind_b200) never imports it.

Parity status: RMSNorm/Embedding/Add/SiLU-Mul/KV offsets/bf16 rounding are
pinned to the reference's compiled kernels and its unit-test golden values.
Linear, W8/W4 dequant, RoPE, attention and argmax have neither a reference
kernel nor reference golden vectors: they follow the reference's written
contracts and are "parity unpinned" beyond them.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_BRIDGE = HERE / "_ref" / "libam_ref_bridge.so"

P = C.c_void_p
i64 = C.c_int64


class OrcLinear(C.Structure):
    _fields_ = [("fmt", C.c_int), ("N", i64), ("K", i64), ("group", i64), ("w", P), ("q8", P), ("s8", P),
                ("q4", P), ("s4", P)]


class OrcLayer(C.Structure):
    _fields_ = [("attn_norm", P), ("mlp_norm", P)] + [(n, OrcLinear) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd")]


class OrcModel(C.Structure):
    _fields_ = [("vocab", i64), ("hidden", i64), ("layers", i64), ("nq", i64), ("nkv", i64), ("hd", i64),
                ("inter", i64), ("max_seq", i64), ("eps", C.c_float), ("theta", C.c_double), ("act_bf16", C.c_int),
                ("embed", P), ("lm_head", OrcLinear), ("final_norm", P), ("layer", C.POINTER(OrcLayer))]


_orc = None
_ref = None


def orc() -> C.CDLL:
    global _orc
    if _orc is None:
        if not ORACLE_LIB.exists():
            raise RuntimeError(f"oracle not built: {ORACLE_LIB} (make -C oracle)")
        l = C.CDLL(str(ORACLE_LIB))
        sig = {
            "orc_bf16_round": (C.c_float, [C.c_float]),
            "orc_f32_to_bf16": (C.c_uint16, [C.c_float]),
            "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
            "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
            "orc_hash": (C.c_uint64, [C.c_uint64, C.c_uint64, C.c_uint64]),
            "orc_synth_w4": (None, [C.c_uint64, C.c_uint64, i64, i64, C.c_float, P, P]),
            "orc_synth_w8": (None, [C.c_uint64, C.c_uint64, i64, i64, C.c_float, P, P]),
            "orc_synth_uniform_bf16": (None, [C.c_uint64, C.c_uint64, i64, C.c_float, P]),
            "orc_unpack_w4": (None, [P, i64, i64, P]),
            "orc_pack_w4": (None, [P, i64, i64, P]),
            "orc_linear_f32": (None, [P, P, P, i64, i64, i64, C.c_int]),
            "orc_linear_w8": (None, [P, P, P, P, i64, i64, i64, C.c_int]),
            "orc_linear_w4": (None, [P, P, P, P, i64, i64, i64, i64, C.c_int]),
            "orc_rmsnorm": (None, [P, P, P, i64, i64, C.c_float, C.c_int]),
            "orc_rope": (None, [P, P, i64, i64, i64, C.c_double, C.c_int]),
            "orc_silu_mul": (None, [P, P, P, i64, C.c_int]),
            "orc_add": (None, [P, P, P, i64, C.c_int]),
            "orc_argmax": (i64, [P, i64]),
            "orc_embedding": (C.c_int, [P, i64, P, i64, i64, P]),
            "orc_kv_write": (None, [P, P, P, P, i64, i64, i64, i64, i64]),
            "orc_attention": (None, [P, P, P, P, i64, i64, i64, i64, i64, i64, C.c_int]),
            "orc_generate": (i64, [C.POINTER(OrcModel), P, i64, i64, P, P, P]),
            "orc_last_timing": (None, [C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        }
        for n, (r, a) in sig.items():
            f = getattr(l, n)
            f.restype, f.argtypes = r, a
        _orc = l
    return _orc


def ref_available() -> bool:
    return REF_BRIDGE.exists()


def ref() -> C.CDLL:
    global _ref
    if _ref is None:
        l = C.CDLL(str(REF_BRIDGE))
        sig = {
            "refb_rmsnorm_f32": (C.c_int, [P, P, P, i64, i64, i64, i64, C.c_float, C.c_int]),
            "refb_add": (C.c_int, [P, P, P, i64, C.c_int]),
            "refb_silu_mul": (C.c_int, [P, P, P, i64, C.c_int]),
            "refb_embedding_f32": (C.c_int, [P, i64, C.c_int, P, i64, i64, P]),
            "refb_kv_offset": (C.c_int, [C.c_uint64] * 4 + [C.c_int] + [C.c_uint64] * 4 +
                               [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
            "refb_kv_reserve": (C.c_int, [C.c_uint64, C.c_uint64, C.c_uint64]),
            "refb_bf16_from_f32": (C.c_uint16, [C.c_float]),
        }
        for n, (r, a) in sig.items():
            f = getattr(l, n)
            f.restype, f.argtypes = r, a
        _ref = l
    return _ref


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


# --------------------------------------------------------------- helpers
def bf16_round(x: np.ndarray) -> np.ndarray:
    """Vectorised RNE rounding of float32 to bf16 values (returned as float32)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    r = np.where(nan, (u | 0x00400000) & 0xFFFF0000, r)
    return r.view(np.float32)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def synth_w4(seed, stream, n, k, base):
    q = np.empty((n, k // 2), np.uint8)
    s = np.empty((n, k // 128), np.uint16)
    orc().orc_synth_w4(seed, stream, n, k, base, _p(q), _p(s))
    return q, s


def synth_w8(seed, stream, n, k, base):
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    orc().orc_synth_w8(seed, stream, n, k, base, _p(q), _p(s))
    return q, s


def synth_uniform_bf16(seed, stream, count, amp):
    out = np.empty(count, np.uint16)
    orc().orc_synth_uniform_bf16(seed, stream, count, amp, _p(out))
    return out


def unpack_w4(packed: np.ndarray, n: int, k: int) -> np.ndarray:
    q = np.empty((n, k), np.int8)
    orc().orc_unpack_w4(_p(np.ascontiguousarray(packed)), n, k, _p(q))
    return q


def pack_w4(q: np.ndarray) -> np.ndarray:
    n, k = q.shape
    out = np.empty((n, k // 2), np.uint8)
    orc().orc_pack_w4(_p(np.ascontiguousarray(q, dtype=np.int8)), n, k, _p(out))
    return out


def quantize_w4(w: np.ndarray, group: int = 128):
    """Symmetric absmax INT4 quantization per (row, group of 128) -- the
    recipe of the engine's checkpoint quantizer (amcu_quantize_weight):
    s = fp16(max|w| / 7), q = clip(rint(w / s), -8, 7), all in fp32 with
    correctly rounded division; returns (packed [n][k/2] uint8, s fp16 bits)."""
    w = np.ascontiguousarray(w, np.float32)
    n, k = w.shape
    g = w.reshape(n, k // group, group)
    s16 = (np.abs(g).max(-1) / np.float32(7)).astype(np.float16)
    sc = s16.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(sc > 0, np.rint(g / np.where(sc > 0, sc, np.float32(1))), np.float32(0))
    q = np.clip(q, -8, 7).astype(np.int8).reshape(n, k)
    return pack_w4(q), s16.view(np.uint16)


def quantize_w8(w: np.ndarray):
    """Symmetric absmax INT8 per output row: s = max|w| / 127 (fp32),
    q = clip(rint(w / s), -127, 127); returns (q int8 [n][k], s fp32 [n])."""
    w = np.ascontiguousarray(w, np.float32)
    s = (np.abs(w).max(-1) / np.float32(127)).astype(np.float32)
    sc = s[:, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.where(sc > 0, np.rint(w / np.where(sc > 0, sc, np.float32(1))), np.float32(0))
    return np.clip(q, -127, 127).astype(np.int8), s


def linear_f32(x, w, bf=False):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    y = np.empty((x.shape[0], w.shape[0]), np.float32)
    orc().orc_linear_f32(_p(x), _p(w), _p(y), x.shape[0], w.shape[0], x.shape[1], int(bf))
    return y


def linear_w8(x, q, s, bf=True):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty((x.shape[0], q.shape[0]), np.float32)
    orc().orc_linear_w8(_p(x), _p(np.ascontiguousarray(q)), _p(np.ascontiguousarray(s, np.float32)), _p(y),
                        x.shape[0], q.shape[0], q.shape[1], int(bf))
    return y


def linear_w4(x, packed, s, bf=True, group=128):
    x = np.ascontiguousarray(x, np.float32)
    n, k = packed.shape[0], packed.shape[1] * 2
    y = np.empty((x.shape[0], n), np.float32)
    orc().orc_linear_w4(_p(x), _p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(s, np.uint16)), _p(y),
                        x.shape[0], n, k, group, int(bf))
    return y


def rmsnorm(x, w, eps, bf=False):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    orc().orc_rmsnorm(_p(x), _p(w), _p(y), x.shape[0], x.shape[1], eps, int(bf))
    return y


def rope(x, pos, nheads, d, theta, bf=False):
    x = np.array(x, np.float32, copy=True, order="C")
    pos = np.ascontiguousarray(pos, np.int64)
    orc().orc_rope(_p(x), _p(pos), x.shape[0], nheads, d, theta, int(bf))
    return x


def silu_mul(g, u, bf=False):
    g = np.ascontiguousarray(g, np.float32); u = np.ascontiguousarray(u, np.float32)
    y = np.empty_like(g)
    orc().orc_silu_mul(_p(g), _p(u), _p(y), g.size, int(bf))
    return y


def argmax(v) -> int:
    v = np.ascontiguousarray(v, np.float32)
    return int(orc().orc_argmax(_p(v), v.size))


def attention(q, kplane, vplane, pos, nq, nkv, d, bf=False):
    """q [M, nq*d]; planes [nkv, cap, d] float32."""
    q = np.ascontiguousarray(q, np.float32)
    kp = np.ascontiguousarray(kplane, np.float32); vp = np.ascontiguousarray(vplane, np.float32)
    out = np.empty_like(q)
    orc().orc_attention(_p(q), _p(kp), _p(vp), _p(out), q.shape[0], pos, nq, nkv, kp.shape[1], d, int(bf))
    return out


# --------------------------------------------------------------- model
class OracleModel:
    """Holds numpy weights for the full-model oracle (keeps them alive)."""

    def __init__(self, cfg, act_bf16: bool):
        self.cfg = cfg
        self.keep: list[np.ndarray] = []
        self.layers = (OrcLayer * cfg.layers)()
        self.m = OrcModel()
        m = self.m
        m.vocab, m.hidden, m.layers = cfg.vocab, cfg.hidden, cfg.layers
        m.nq, m.nkv, m.hd, m.inter = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, cfg.inter
        m.max_seq, m.eps, m.theta, m.act_bf16 = cfg.max_seq, cfg.rms_eps, cfg.rope_theta, int(act_bf16)
        m.layer = self.layers

    def _hold(self, a):
        a = np.ascontiguousarray(a)
        self.keep.append(a)
        return a.ctypes.data

    def linear(self, fmt, n, k, w=None, q=None, s=None):
        L = OrcLinear()
        L.fmt, L.N, L.K, L.group = fmt, n, k, 128
        if fmt == 0:
            L.w = self._hold(np.asarray(w, np.float32))
        elif fmt == 1:
            L.q8, L.s8 = self._hold(q), self._hold(np.asarray(s, np.float32))
        else:
            L.q4, L.s4 = self._hold(q), self._hold(s)
        return L

    def set_vec(self, a):
        return self._hold(np.asarray(a, np.float32))

    def generate(self, prompt, max_new):
        p = np.ascontiguousarray(prompt, np.int64)
        out = np.zeros(max_new, np.int64)
        gaps = np.zeros(max_new, np.float32)
        n = orc().orc_generate(C.byref(self.m), _p(p), p.size, max_new, _p(out), None, _p(gaps))
        return out[:n], gaps[:n]

    @staticmethod
    def last_timing() -> tuple[float, float]:
        """(prefill seconds, decode seconds) of the last generate call."""
        a, b = C.c_double(), C.c_double()
        orc().orc_last_timing(C.byref(a), C.byref(b))
        return a.value, b.value


# same float32 arithmetic as the engine's constants (0.02f / 4.6098f, 0.02f / 73.61f)
W4_BASE = float(np.float32(0.02) / np.float32(4.6098))
W8_BASE = float(np.float32(0.02) / np.float32(73.61))
EMBED_AMP = 0.0692820


def synthetic_oracle_model(cfg, seed: int, layers: int | None = None) -> OracleModel:
    """The engine's seeded synthetic model (am_model_init_synthetic), regenerated
    on the CPU with the same integer-hash generators (bit-identical weights)."""
    from aethermind_b200 import _lib as L  # constants only; no compute

    om = OracleModel(cfg, act_bf16=True)
    H, d = cfg.hidden, cfg.head_dim
    fmt = 2 if cfg.weight_format == L.WFMT_INT4 else 1
    gen = (lambda st, n, k: synth_w4(seed, st, n, k, W4_BASE)) if fmt == 2 else \
        (lambda st, n, k: synth_w8(seed, st, n, k, W8_BASE))
    if cfg.tied_embeddings:
        q, s = gen(1, cfg.vocab, H)
        om.m.lm_head = om.linear(fmt, cfg.vocab, H, q=q, s=s)
        om.m.embed = None
    else:
        e = bf16_bits_to_f32(synth_uniform_bf16(seed, 1, cfg.vocab * H, EMBED_AMP)).reshape(cfg.vocab, H)
        om.m.embed = om._hold(e)
        q, s = gen(2, cfg.vocab, H)
        om.m.lm_head = om.linear(fmt, cfg.vocab, H, q=q, s=s)
    ones = np.ones(H, np.float32)
    om.m.final_norm = om.set_vec(ones)
    shapes = {"wq": (cfg.n_q_heads * d, H), "wk": (cfg.n_kv_heads * d, H), "wv": (cfg.n_kv_heads * d, H),
              "wo": (H, cfg.n_q_heads * d), "wg": (cfg.inter, H), "wu": (cfg.inter, H), "wd": (H, cfg.inter)}
    nl = cfg.layers if layers is None else layers
    for l in range(nl):
        Ly = om.layers[l]
        Ly.attn_norm = om.set_vec(ones)
        Ly.mlp_norm = om.set_vec(ones)
        for t, name in enumerate(("wq", "wk", "wv", "wo", "wg", "wu", "wd")):
            n, k = shapes[name]
            q, s = gen(16 + l * 8 + t, n, k)
            setattr(Ly, name, om.linear(fmt, n, k, q=q, s=s))
    return om
