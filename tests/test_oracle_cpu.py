"""The CPU oracle pinned against the reference engine (CPU only).

Pins: the reference unit tests' golden values, and fixtures produced by the
reference's own compiled kernels (tests/golden/ref_kernels.npz, made by
tests/golden/make_golden.py). Restated ops without a reference kernel are
checked against straightforward float64 numpy restatements of the same
contracts.
"""
import numpy as np
import pytest

GOLD = None


@pytest.fixture(scope="module")
def gold():
    from pathlib import Path
    return np.load(Path(__file__).parent / "golden" / "ref_kernels.npz")


@pytest.fixture(scope="module")
def orc(oracle_lib):
    return oracle_lib


def test_rmsnorm_reference_unit_golden(orc, gold):
    # tests/unit/backend/cpu/kernels/test_cpu_rmsnorm_kernel.cpp:65-89 of the reference
    expect = np.array([0.365148, 0.730297, 1.095445, 1.460593], np.float32)
    np.testing.assert_allclose(gold["rmsnorm_unit_out"][0], expect, atol=1e-5)
    y = orc.rmsnorm(np.array([[1, 2, 3, 4]], np.float32), np.ones(4, np.float32), 1e-5)
    np.testing.assert_allclose(y[0], expect, atol=1e-5)


@pytest.mark.parametrize("name", ["small", "h4096"])
def test_rmsnorm_restatement_matches_reference_kernels(orc, gold, name):
    x, w = gold[f"rmsnorm_{name}_x"], gold[f"rmsnorm_{name}_w"]
    y = orc.rmsnorm(x, w, 1e-5)
    np.testing.assert_allclose(y, gold[f"rmsnorm_{name}_scalar"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(y, gold[f"rmsnorm_{name}_avx2"], rtol=1e-5, atol=1e-6)


def test_silu_mul_matches_reference_const_evaluator(orc, gold):
    y = orc.silu_mul(gold["silu_g"], gold["silu_u"])
    np.testing.assert_allclose(y, gold["silu_f32"], rtol=1e-6, atol=1e-30)
    gb = orc.bf16_bits_to_f32(gold["silu_g_bf16"])
    ub = orc.bf16_bits_to_f32(gold["silu_u_bf16"])
    yb = orc.silu_mul(gb, ub, bf=True)
    np.testing.assert_array_equal(orc.f32_to_bf16_bits(yb), gold["silu_bf16"])


def test_add_bf16_matches_reference(orc, gold):
    a, b = orc.bf16_bits_to_f32(gold["add_bf16_a"]), orc.bf16_bits_to_f32(gold["add_bf16_b"])
    y = np.empty_like(a)
    import ctypes as C
    orc.orc().orc_add(a.ctypes.data, b.ctypes.data, y.ctypes.data, a.size, 1)
    np.testing.assert_array_equal(orc.f32_to_bf16_bits(y), gold["add_bf16_out"])


def test_embedding_matches_reference(orc, gold):
    import ctypes as C
    t, ids = gold["emb_table"], gold["emb_ids"]
    out = np.zeros((ids.size, t.shape[1]), np.float32)
    assert orc.orc().orc_embedding(ids.ctypes.data, ids.size, t.ctypes.data, t.shape[0], t.shape[1],
                                   out.ctypes.data) == 0
    np.testing.assert_array_equal(out, gold["emb_out"])
    bad = np.array([1, 64], np.int64)
    assert orc.orc().orc_embedding(bad.ctypes.data, 2, t.ctypes.data, 64, 32, out.ctypes.data) == int(
        gold["emb_bad_status"][0])


def test_bf16_conversion_matches_reference(orc, gold):
    f = gold["bf16_in"]
    np.testing.assert_array_equal(orc.f32_to_bf16_bits(f), gold["bf16_out"])
    np.testing.assert_array_equal(np.array([orc.orc().orc_f32_to_bf16(float(v)) for v in f], np.uint16),
                                  gold["bf16_out"])


def test_f16_conversion_is_ieee_rne(orc):
    rng = np.random.default_rng(3)
    v = np.concatenate([rng.normal(0, 1, 2000), rng.uniform(-70000, 70000, 200), rng.normal(0, 1e-5, 200),
                        [0.0, 65504.0, 65519.0, 65520.0, 6.1e-5, 5.96e-8, 2.98e-8]]).astype(np.float32)
    got = np.array([orc.orc().orc_f32_to_f16(float(x)) for x in v], np.uint16)
    np.testing.assert_array_equal(got, v.astype(np.float16).view(np.uint16))
    back = np.array([orc.orc().orc_f16_to_f32(int(h)) for h in got], np.float32)
    np.testing.assert_array_equal(back, got.view(np.float16).astype(np.float32))


def test_w4_pack_unpack_exhaustive(orc):
    # all 16 values in both nibble positions
    q = np.array([[a, b] for a in range(-8, 8) for b in range(-8, 8)], np.int8).reshape(16, 32)
    packed = orc.pack_w4(q)
    lo, hi = int(q[0, 0]) & 15, int(q[0, 1]) & 15
    assert int(packed[0, 0]) == lo | (hi << 4)
    np.testing.assert_array_equal(orc.unpack_w4(packed, 16, 32), q)


def test_synth_is_deterministic_and_in_range(orc):
    q, s = orc.synth_w4(7, 3, 32, 256, orc.W4_BASE)
    q2, s2 = orc.synth_w4(7, 3, 32, 256, orc.W4_BASE)
    np.testing.assert_array_equal(q, q2)
    np.testing.assert_array_equal(s, s2)
    vals = orc.unpack_w4(q, 32, 256)
    assert vals.min() == -8 and vals.max() == 7
    sf = s.view(np.float16).astype(np.float32)
    assert np.all(sf > 0.74 * orc.W4_BASE) and np.all(sf < 1.26 * orc.W4_BASE)
    q8, s8 = orc.synth_w8(7, 3, 16, 128, orc.W8_BASE)
    assert q8.min() >= -127 and q8.max() <= 127
    e = orc.bf16_bits_to_f32(orc.synth_uniform_bf16(7, 1, 10000, orc.EMBED_AMP))
    assert abs(e.std() - 0.02) < 0.002


def _dense_w4(q4, s4, n, k):
    q = orc_mod().unpack_w4(q4, n, k).astype(np.float64)
    s = s4.view(np.float16).astype(np.float64)
    return q * np.repeat(s, 128, axis=1)


def orc_mod():
    import oracle
    return oracle


@pytest.mark.parametrize("m", [1, 3, 8])
def test_linear_w4_w8_match_dense_dequant(orc, m):
    n, k = 48, 512
    rng = np.random.default_rng(m)
    x = orc.bf16_round(rng.normal(0, 1, (m, k)).astype(np.float32))
    q4, s4 = orc.synth_w4(1, 5, n, k, orc.W4_BASE)
    ref = x.astype(np.float64) @ _dense_w4(q4, s4, n, k).T
    np.testing.assert_allclose(orc.linear_w4(x, q4, s4, bf=False), ref, rtol=1e-4, atol=1e-5)
    q8, s8 = orc.synth_w8(1, 5, n, k, orc.W8_BASE)
    ref8 = x.astype(np.float64) @ (q8.astype(np.float64) * s8[:, None].astype(np.float64)).T
    np.testing.assert_allclose(orc.linear_w8(x, q8, s8, bf=False), ref8, rtol=1e-4, atol=1e-6)


def test_rope_matches_float64_formula(orc):
    d, nh, theta = 128, 4, 500000.0
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (3, nh * d)).astype(np.float32)
    pos = np.array([0, 17, 4095])
    y = orc.rope(x, pos, nh, d, theta)
    half = d // 2
    inv = 1.0 / theta ** (2.0 * np.arange(half) / d)
    for r in range(3):
        c, s = np.cos(pos[r] * inv).astype(np.float32), np.sin(pos[r] * inv).astype(np.float32)
        xv = x[r].reshape(nh, d)
        exp = np.concatenate([xv[:, :half] * c - xv[:, half:] * s, xv[:, half:] * c + xv[:, :half] * s], axis=1)
        np.testing.assert_allclose(y[r].reshape(nh, d), exp, rtol=1e-6, atol=1e-6)
    assert np.array_equal(y[0], x[0])  # position 0 is the identity


def test_attention_matches_float64_softmax(orc):
    nq, nkv, d, cap, M, pos = 8, 2, 64, 40, 3, 20
    rng = np.random.default_rng(1)
    q = rng.normal(0, 1, (M, nq * d)).astype(np.float32)
    kp = rng.normal(0, 1, (nkv, cap, d)).astype(np.float32)
    vp = rng.normal(0, 1, (nkv, cap, d)).astype(np.float32)
    out = orc.attention(q, kp, vp, pos, nq, nkv, d)
    for m in range(M):
        L = pos + m + 1
        for h in range(nq):
            kv = h // (nq // nkv)
            sc = (kp[kv, :L].astype(np.float64) @ q[m, h * d:(h + 1) * d].astype(np.float64)) / np.sqrt(d)
            p = np.exp(sc - sc.max())
            p /= p.sum()
            np.testing.assert_allclose(out[m, h * d:(h + 1) * d], p @ vp[kv, :L], rtol=1e-5, atol=1e-6)


def test_argmax_ties_lowest_index(orc):
    v = np.array([1.0, 3.0, 2.0, 3.0], np.float32)
    assert orc.argmax(v) == 1
    assert orc.argmax(np.full(100, -1.0, np.float32)) == 0


def test_tiny_model_oracle_runs(orc):
    from aethermind_b200.session import TINY_F32
    from tests.model_fixtures import tiny_oracle_model, tiny_prompt, tiny_weights

    w = tiny_weights(TINY_F32)
    om = tiny_oracle_model(TINY_F32, w)
    toks, gaps = om.generate(tiny_prompt(TINY_F32), 32)
    assert toks.shape == (32,) and toks.min() >= 0 and toks.max() < 512
    toks2, _ = om.generate(tiny_prompt(TINY_F32), 32)
    np.testing.assert_array_equal(toks, toks2)
