"""Generates tests/golden/ref_kernels.npz from the reference engine's own CPU
kernels (compiled from its sources into oracle/_ref by oracle/Makefile).

Run here, where the reference sources exist:
    make -C oracle && python tests/golden/make_golden.py
The fixtures travel with the repo; the GPU box never needs the reference.
Every array is produced by a reference entry point through
oracle/ref_bridge.cpp (no arithmetic of this project's own):
  rmsnorm_*   LaunchRmsNorm (AVX2 path) and RmsNormKernel_CPU_FP32_Scalar
  silu_*      the SiluMul constant evaluator (fp32 and bf16)
  add_bf16_*  LaunchAdd on bf16
  emb_*       EmbeddingKernel on fp32
  kv_*        KVCacheLayout::Offset / BytesPerPlane via KVCacheManager::Init
  bf16_*      BFloat16(float) conversion
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402


def p(a):
    return a.ctypes.data


def main() -> None:
    R = oracle.ref()
    rng = np.random.default_rng(123456789)
    out: dict[str, np.ndarray] = {}

    # RMSNorm: the unit-test golden row and seeded random rows.
    x = np.array([[1, 2, 3, 4]], np.float32)
    y = np.zeros_like(x)
    assert R.refb_rmsnorm_f32(p(x), p(np.ones(4, np.float32)), p(y), 1, 4, 4, 4, 1e-5, 0) == 0
    out["rmsnorm_unit_in"], out["rmsnorm_unit_out"] = x, y
    for name, (rows, hidden) in {"small": (8, 256), "h4096": (4, 4096)}.items():
        x = rng.normal(0, 1, (rows, hidden)).astype(np.float32)
        w = rng.uniform(0.5, 1.5, hidden).astype(np.float32)
        y_avx = np.zeros_like(x)
        y_sc = np.zeros_like(x)
        assert R.refb_rmsnorm_f32(p(x), p(w), p(y_avx), rows, hidden, hidden, hidden, 1e-5, 0) == 0
        assert R.refb_rmsnorm_f32(p(x), p(w), p(y_sc), rows, hidden, hidden, hidden, 1e-5, 1) == 0
        out[f"rmsnorm_{name}_x"], out[f"rmsnorm_{name}_w"] = x, w
        out[f"rmsnorm_{name}_avx2"], out[f"rmsnorm_{name}_scalar"] = y_avx, y_sc

    # SiLU-Mul const evaluator, fp32 and bf16 (bf16 passed as raw bits).
    g = np.concatenate([rng.normal(0, 3, 4093), [0.0, -0.0, 88.0, -88.0, 20.0, -20.0, 1e-30]]).astype(np.float32)
    u = rng.normal(0, 1, g.size).astype(np.float32)
    yf = np.zeros_like(g)
    assert R.refb_silu_mul(p(g), p(u), p(yf), g.size, 0) == 0
    gb, ub = oracle.f32_to_bf16_bits(g), oracle.f32_to_bf16_bits(u)
    yb = np.zeros_like(gb)
    assert R.refb_silu_mul(p(gb), p(ub), p(yb), g.size, 1) == 0
    out.update(silu_g=g, silu_u=u, silu_f32=yf, silu_g_bf16=gb, silu_u_bf16=ub, silu_bf16=yb)

    # Residual add in bf16.
    a = oracle.f32_to_bf16_bits(rng.normal(0, 2, 4096).astype(np.float32))
    b = oracle.f32_to_bf16_bits(rng.normal(0, 2, 4096).astype(np.float32))
    c = np.zeros_like(a)
    assert R.refb_add(p(a), p(b), p(c), a.size, 1) == 0
    out.update(add_bf16_a=a, add_bf16_b=b, add_bf16_out=c)

    # Embedding rows (int64 ids) and the out-of-range status.
    table = rng.normal(0, 0.02, (64, 32)).astype(np.float32)
    ids = np.array([0, 63, 7, 7, 31], np.int64)
    emb = np.zeros((ids.size, 32), np.float32)
    assert R.refb_embedding_f32(p(ids), ids.size, 1, p(table), 64, 32, p(emb)) == 0
    bad = np.array([1, 64], np.int64)
    emb_bad = np.zeros((2, 32), np.float32)
    out.update(emb_table=table, emb_ids=ids, emb_out=emb,
               emb_bad_status=np.array([R.refb_embedding_f32(p(bad), 2, 1, p(table), 64, 32, p(emb_bad))], np.int32))

    # KV layout offsets: (layers, heads, max_tokens, head_dim, dtype, l, h, pos, dim) -> (offset, bytes/plane)
    import ctypes as C
    cases = [(2, 2, 4, 8, 0, 1, 1, 3, 5), (32, 8, 4096, 128, 1, 31, 7, 4095, 127), (16, 8, 2048, 64, 1, 3, 2, 100, 9),
             (2, 2, 128, 64, 0, 0, 1, 17, 63), (80, 8, 4096, 128, 1, 79, 0, 2047, 1)]
    rows = []
    for cs in cases:
        off, bpp = C.c_uint64(), C.c_uint64()
        st = R.refb_kv_offset(*cs, C.byref(off), C.byref(bpp))
        rows.append(list(cs) + [st, off.value, bpp.value])
    oob = (2, 2, 4, 8, 0, 0, 0, 4, 0)  # pos == max_tokens -> OutOfRange
    off, bpp = C.c_uint64(), C.c_uint64()
    rows.append(list(oob) + [R.refb_kv_offset(*oob, C.byref(off), C.byref(bpp)), 0, 0])
    out["kv_cases"] = np.array(rows, np.uint64)
    res = [(16, 10, 6), (16, 10, 7), (16, 0, 0), (16, 16, 0), (4096, 512, 256)]
    out["kv_reserve"] = np.array([[m, pl, mn, R.refb_kv_reserve(m, pl, mn)] for m, pl, mn in res], np.int64)

    # BFloat16 conversion (RNE) of edge values and random floats.
    f = np.concatenate([np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 3.0e38, 1e-40, np.inf, -np.inf],
                                 np.float32), rng.normal(0, 100, 1000).astype(np.float32)])
    out["bf16_in"] = f
    out["bf16_out"] = np.array([R.refb_bf16_from_f32(float(v)) for v in f], np.uint16)

    dst = Path(__file__).with_name("ref_kernels.npz")
    np.savez_compressed(dst, **out)
    print("wrote", dst, sum(v.nbytes for v in out.values()), "bytes")


if __name__ == "__main__":
    main()
