"""Per-op parity of the CUDA kernels (through the C ABI) against the CPU oracle.

Tolerances: integer/byte work (synthetic weights, packing, argmax indices,
KV addressing) is bit-exact; bf16 outputs are compared with rtol 1e-2 (the
north-star bf16 tolerance) and fp32 outputs with rtol 1e-4 (plus a small atol
for values near zero).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

BF_RTOL, BF_ATOL = 1e-2, 1e-2
F32_RTOL = 1e-4


@pytest.fixture(scope="module")
def ops(built_lib):
    from aethermind_b200 import ops as O
    return O


@pytest.fixture(scope="module")
def orc(oracle_lib):
    return oracle_lib


@pytest.fixture(scope="module")
def gold():
    from pathlib import Path
    return np.load(Path(__file__).parent / "golden" / "ref_kernels.npz")


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bf16_dev(a_f32):
    return torch.from_numpy(np.ascontiguousarray(a_f32, np.float32)).cuda().to(torch.bfloat16)


def to_np(t):
    return t.float().cpu().numpy() if t.dtype == torch.bfloat16 else t.cpu().numpy()


# ------------------------------------------------------------- weights
def test_synth_bit_exact_vs_oracle(ops, orc):
    q, s = ops.synth_w4(11, 9, 64, 512, orc.W4_BASE)
    rq, rs = orc.synth_w4(11, 9, 64, 512, orc.W4_BASE)
    np.testing.assert_array_equal(q.cpu().numpy(), rq)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), rs)
    q8, s8 = ops.synth_w8(11, 9, 32, 256, orc.W8_BASE)
    rq8, rs8 = orc.synth_w8(11, 9, 32, 256, orc.W8_BASE)
    np.testing.assert_array_equal(q8.cpu().numpy(), rq8)
    np.testing.assert_array_equal(s8.cpu().numpy(), rs8)
    e = ops.synth_uniform_bf16(11, 1, 4096, orc.EMBED_AMP)
    np.testing.assert_array_equal(e.cpu().view(torch.int16).numpy().view(np.uint16),
                                  orc.synth_uniform_bf16(11, 1, 4096, orc.EMBED_AMP))


@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("k", [1024, 384, 1792])
def test_prepack_roundtrip_bit_exact(ops, fmt, k):
    from aethermind_b200 import _lib as L
    n = 96
    if fmt == "int4":
        q, s = ops.synth_w4(3, 1, n, k, 0.01)
        pw = ops.prepack(L.WFMT_INT4, q, s, n, k)
    else:
        q, s = ops.synth_w8(3, 1, n, k, 0.01)
        pw = ops.prepack(L.WFMT_INT8, q, s, n, k)
    q2, s2 = ops.unpack(pw)
    assert torch.equal(q2.view(torch.uint8).flatten(), q.view(torch.uint8).flatten())
    assert torch.equal(s2.flatten().view(torch.uint8), s.flatten().view(torch.uint8))


@pytest.mark.parametrize("fmt", ["int4", "int8"])
def test_prepack_rows_builds_fused_weight(ops, fmt):
    """Packing row ranges one by one into a fused weight gives the same bytes
    as packing the concatenated canonical matrix (the q/k/v fusion)."""
    import ctypes as C
    from aethermind_b200 import _lib as L
    k, parts = 1792, [64, 32, 32]
    f = L.WFMT_INT4 if fmt == "int4" else L.WFMT_INT8
    syn = ops.synth_w4 if fmt == "int4" else ops.synth_w8
    qs, ss = zip(*[syn(7, i, n, k, 0.01) for i, n in enumerate(parts)])
    n_total = sum(parts)
    whole = ops.prepack(f, torch.cat(qs), torch.cat(ss), n_total, k)
    fused = ops.prepack(f, torch.cat(qs), torch.cat(ss), n_total, k)
    fused.data.zero_()
    if fused.scales is not None:
        fused.scales.zero_()
    row0 = 0
    for q, s, n in zip(qs, ss, parts):
        code = L.lib().amcu_prepack_weight_rows(f, L.BF16, n, k, 128, n_total, row0, q.data_ptr(), s.data_ptr(),
                                                fused.data.data_ptr(), ops._p(fused.scales),
                                                torch.cuda.current_stream().cuda_stream)
        L.check(code, "amcu_prepack_weight_rows")
        row0 += n
    torch.cuda.synchronize()
    assert torch.equal(fused.data, whole.data)
    assert fused.scales is None or torch.equal(fused.scales, whole.scales)
    bad = L.lib().amcu_prepack_weight_rows(f, L.BF16, 32, k, 128, n_total, 8, qs[1].data_ptr(), ss[1].data_ptr(),
                                           fused.data.data_ptr(), ops._p(fused.scales), None)
    assert bad == 3 and b"16-row" in L.lib().amcu_last_error()


# ------------------------------------------------------------- rmsnorm
def test_rmsnorm_f32_matches_reference_kernels(ops, gold):
    for name in ("small", "h4096"):
        x, w = gold[f"rmsnorm_{name}_x"], gold[f"rmsnorm_{name}_w"]
        y = ops.rmsnorm(dev(x), dev(w), 1e-5)
        np.testing.assert_allclose(to_np(y), gold[f"rmsnorm_{name}_scalar"], rtol=F32_RTOL, atol=1e-6)
    y = ops.rmsnorm(dev(np.array([[1, 2, 3, 4]], np.float32)), dev(np.ones(4, np.float32)), 1e-5)
    np.testing.assert_allclose(to_np(y)[0], [0.365148, 0.730297, 1.095445, 1.460593], atol=1e-5)


@pytest.mark.parametrize("m", [1, 8, 64, 512])
def test_rmsnorm_bf16_fused_residual(ops, orc, m):
    rng = np.random.default_rng(m)
    x = orc.bf16_round(rng.normal(0, 1, (m, 4096)).astype(np.float32))
    r = orc.bf16_round(rng.normal(0, 1, (m, 4096)).astype(np.float32))
    w = orc.bf16_round(rng.uniform(0.5, 1.5, 4096).astype(np.float32))
    y, h = ops.rmsnorm(bf16_dev(x), bf16_dev(w), 1e-5, residual=bf16_dev(r))
    h_ref = orc.bf16_round(x + r)
    np.testing.assert_array_equal(to_np(h), h_ref)
    np.testing.assert_allclose(to_np(y), orc.rmsnorm(h_ref, w, 1e-5, bf=True), rtol=BF_RTOL, atol=BF_ATOL)


@pytest.mark.parametrize("hidden", [2048, 8192, 4100, 16384])
@pytest.mark.parametrize("with_res", [False, True])
def test_rmsnorm_bf16_widths(ops, orc, hidden, with_res):
    """bf16 rows that take the 16-byte-vector kernel (hidden % 8 == 0 and at
    most 8192) and rows that keep the scalar one (4100, 16384)."""
    m = 3
    rng = np.random.default_rng(hidden)
    x = orc.bf16_round(rng.normal(0, 2, (m, hidden)).astype(np.float32))
    w = orc.bf16_round(rng.uniform(0.5, 1.5, hidden).astype(np.float32))
    if with_res:
        r = orc.bf16_round(rng.normal(0, 1, (m, hidden)).astype(np.float32))
        y, h = ops.rmsnorm(bf16_dev(x), bf16_dev(w), 1e-5, residual=bf16_dev(r))
        x = orc.bf16_round(x + r)
        np.testing.assert_array_equal(to_np(h), x)
    else:
        y = ops.rmsnorm(bf16_dev(x), bf16_dev(w), 1e-5)
    np.testing.assert_allclose(to_np(y), orc.rmsnorm(x, w, 1e-5, bf=True), rtol=BF_RTOL, atol=BF_ATOL)


def test_rmsnorm_empty_rows_is_ok(ops):
    x = torch.empty(0, 64, device="cuda", dtype=torch.float32)
    y = ops.rmsnorm(x, torch.ones(64, device="cuda"), 1e-5)
    assert y.shape == (0, 64)


# ------------------------------------------------------------- linear
def _w(ops, orc, fmt, n, k, seed=5):
    from aethermind_b200 import _lib as L
    if fmt == "int4":
        q, s = ops.synth_w4(seed, 2, n, k, orc.W4_BASE)
        return ops.prepack(L.WFMT_INT4, q, s, n, k), (q.cpu().numpy(), s.cpu().numpy().view(np.uint16))
    q, s = ops.synth_w8(seed, 2, n, k, orc.W8_BASE)
    return ops.prepack(L.WFMT_INT8, q, s, n, k), (q.cpu().numpy(), s.cpu().numpy())


def _oracle_linear(orc, fmt, x, host):
    return orc.linear_w4(x, *host) if fmt == "int4" else orc.linear_w8(x, *host)


@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("m", [1, 8])
@pytest.mark.parametrize("n", [4096, 14336])
def test_gemv_matches_oracle(ops, orc, fmt, m, n):
    k = 4096
    pw, host = _w(ops, orc, fmt, n, k)
    x = orc.bf16_round(np.random.default_rng(m).normal(0, 1, (m, k)).astype(np.float32))
    entry = "amcu_gemv_w4g128" if fmt == "int4" else "amcu_gemv_w8"
    y = ops.linear(bf16_dev(x), pw, entry=entry)
    np.testing.assert_allclose(to_np(y), _oracle_linear(orc, fmt, x, host), rtol=BF_RTOL, atol=BF_ATOL)


@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("m", [1, 5])
def test_gemv_fused_rmsnorm_matches_oracle(ops, orc, fmt, m):
    """norm_weight: RMSNorm of x fused into the GEMV's staging == RMSNorm
    (bf16 output) then the GEMV."""
    n, k = 64, 4096
    pw, host = _w(ops, orc, fmt, n, k, seed=21)
    rng = np.random.default_rng(m + 40)
    x = orc.bf16_round(rng.normal(0, 3, (m, k)).astype(np.float32))
    w = orc.bf16_round(rng.uniform(0.5, 1.5, k).astype(np.float32))
    y = ops.linear(bf16_dev(x), pw, norm_weight=bf16_dev(w))
    h = orc.rmsnorm(x, w, 1e-5, bf=True)
    np.testing.assert_allclose(to_np(y), _oracle_linear(orc, fmt, h, host), rtol=BF_RTOL, atol=BF_ATOL)


@pytest.mark.parametrize("scale", [1e3, 3e5])
def test_gemv_w4_large_activations(ops, orc, scale):
    """Rows beyond fp16's range take the staging's power-of-two guard: one row
    scaled up, one normal row, both against the oracle."""
    n, k = 64, 1024
    pw, host = _w(ops, orc, "int4", n, k, seed=22)
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, (2, k)).astype(np.float32)
    x[0] *= scale
    x = orc.bf16_round(x)
    y = to_np(ops.linear(bf16_dev(x), pw))
    ref = _oracle_linear(orc, "int4", x, host)
    np.testing.assert_allclose(y, ref, rtol=BF_RTOL, atol=BF_ATOL * scale)
    assert np.isfinite(y).all()


@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("m", [1, 3])
@pytest.mark.parametrize("k", [384, 1792, 14336])
def test_gemv_stream_geometries(ops, orc, fmt, m, k):
    """K values with stages of 3 (384), 14 (1792) and 16 (14336) pair records."""
    n = 48
    pw, host = _w(ops, orc, fmt, n, k, seed=k)
    x = orc.bf16_round(np.random.default_rng(k + m).normal(0, 1, (m, k)).astype(np.float32))
    y = ops.linear(bf16_dev(x), pw)
    np.testing.assert_allclose(to_np(y), _oracle_linear(orc, fmt, x, host), rtol=BF_RTOL, atol=BF_ATOL)


@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("m", [64, 512])
def test_prefill_gemm_matches_torch_fp32(ops, orc, fmt, m):
    """Large-m GEMM against a torch fp32 matmul of the unpacked weights."""
    n, k = 4096, 4096
    pw, host = _w(ops, orc, fmt, n, k)
    x = orc.bf16_round(np.random.default_rng(m).normal(0, 1, (m, k)).astype(np.float32))
    entry = "amcu_gemm_w4g128_prefill" if fmt == "int4" else "amcu_gemm_w8_prefill"
    y = ops.linear(bf16_dev(x), pw, entry=entry)
    if fmt == "int4":
        q = torch.from_numpy(orc.unpack_w4(host[0], n, k)).cuda().float()
        s = torch.from_numpy(host[1].view(np.float16)).cuda().float().repeat_interleave(128, dim=1)
        wd = q * s
    else:
        wd = torch.from_numpy(host[0]).cuda().float() * torch.from_numpy(host[1]).cuda()[:, None]
    ref = dev(x) @ wd.T
    torch.testing.assert_close(y.float(), ref, rtol=BF_RTOL, atol=5e-2)


@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("m", [64, 512])
def test_prefill_gemm_n14336_matches_oracle(ops, orc, fmt, m):
    """The op sweep's N = 14336 (K = 4096) through the tensor-core GEMM at
    m = 64 and 512, against the CPU oracle's Linear."""
    n, k = 14336, 4096
    pw, host = _w(ops, orc, fmt, n, k, seed=31)
    x = orc.bf16_round(np.random.default_rng(m + 7).normal(0, 1, (m, k)).astype(np.float32))
    entry = "amcu_gemm_w4g128_prefill" if fmt == "int4" else "amcu_gemm_w8_prefill"
    y = ops.linear(bf16_dev(x), pw, entry=entry)
    np.testing.assert_allclose(to_np(y), _oracle_linear(orc, fmt, x, host), rtol=BF_RTOL, atol=BF_ATOL)


def _one_hot_expected(fmt, host, n, cols):
    """bf16(q[n, k] * s) for the columns k in `cols`: rows [len(cols), n]."""
    from oracle import bf16_round, unpack_w4
    if fmt == "int4":
        q = unpack_w4(host[0], n, len(host[0][0]) * 2).astype(np.float32)
        s = host[1].view(np.float16).astype(np.float32)
        return bf16_round(np.stack([q[:, c] * s[:, c // 128] for c in cols]) + np.float32(0))  # -0 -> +0
    q = host[0].astype(np.float32)
    return bf16_round(np.stack([q[:, c] * host[1] for c in cols]) + np.float32(0))


@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("entry_kind,m", [("gemv", 1), ("gemv", 8), ("gemm", 64), ("gemm", 512)])
def test_in_kernel_dequant_bit_exact(ops, orc, fmt, entry_kind, m):
    """One-hot activation rows pick single weight columns: the output must be
    bf16(q[n, k] * s[n, group]) (INT4) or bf16(q[n, k] * s[n]) (INT8) bit for
    bit, which pins the kernels' nibble/byte unpacking, the group and scale
    indexing and the offset removal (no rounding happens before the final
    bf16 store: q * s is exact in fp32 for INT4, one fp32 rounding for INT8,
    as in the reference's dequant). Every column of K is covered."""
    n, k = 256, 1024
    pw, host = _w(ops, orc, fmt, n, k, seed=41)
    entry = {("gemv", "int4"): "amcu_gemv_w4g128", ("gemv", "int8"): "amcu_gemv_w8",
             ("gemm", "int4"): "amcu_gemm_w4g128_prefill", ("gemm", "int8"): "amcu_gemm_w8_prefill"}[
        (entry_kind, fmt)]
    order = np.random.default_rng(m).permutation(k)
    for c0 in range(0, k, m):
        cols = order[c0:c0 + m]
        x = np.zeros((len(cols), k), np.float32)
        x[np.arange(len(cols)), cols] = 1.0
        y = ops.linear(bf16_dev(x), pw, entry=entry)
        got = y.cpu().view(torch.int16).numpy().view(np.uint16)
        want = orc.f32_to_bf16_bits(_one_hot_expected(fmt, host, n, cols))
        np.testing.assert_array_equal(got, want, err_msg=f"columns {cols[:8]}...")


@pytest.mark.parametrize("fmt", ["int4", "int8"])
def test_prefill_gemm_epilogues_ragged_tiles(ops, orc, fmt):
    """Tensor-core GEMM with m and n that do not fill the 128 x 128 tiles:
    residual add (in place) and the gate/up SiLU-Mul epilogue against the
    oracle on every row."""
    from aethermind_b200 import _lib as L
    m, k, n, inter = 200, 1024, 2064, 520
    rng = np.random.default_rng(12)
    x = orc.bf16_round(rng.normal(0, 1, (m, k)).astype(np.float32))
    res = orc.bf16_round(rng.normal(0, 1, (m, n)).astype(np.float32))
    pw, host = _w(ops, orc, fmt, n, k, seed=13)
    xr = bf16_dev(res)
    y = ops.linear(bf16_dev(x), pw, epilogue=L.EPI_RESIDUAL_ADD, residual=xr, out=xr)
    ref = orc.bf16_round(res + _oracle_linear(orc, fmt, x, host))
    np.testing.assert_allclose(to_np(y), ref, rtol=BF_RTOL, atol=5e-2)
    syn = ops.synth_w4 if fmt == "int4" else ops.synth_w8
    base = orc.W4_BASE if fmt == "int4" else orc.W8_BASE
    f = L.WFMT_INT4 if fmt == "int4" else L.WFMT_INT8
    gq, gs = syn(14, 1, inter, k, base)
    uq, us = syn(14, 2, inter, k, base)
    gu = ops.prepack_gate_up(f, gq, gs, uq, us, inter, k)
    hs = (lambda s: s.cpu().numpy().view(np.uint16)) if fmt == "int4" else (lambda s: s.cpu().numpy())
    g = _oracle_linear(orc, fmt, x, (gq.cpu().numpy(), hs(gs)))
    u = _oracle_linear(orc, fmt, x, (uq.cpu().numpy(), hs(us)))
    a = ops.linear(bf16_dev(x), gu, epilogue=L.EPI_SILU_MUL)
    ref = orc.silu_mul(orc.bf16_round(g), orc.bf16_round(u), bf=True)
    np.testing.assert_allclose(to_np(a), ref, rtol=BF_RTOL, atol=5e-2)


@pytest.mark.parametrize("fmt", ["int4", "int8"])
def test_linear_residual_and_silu_epilogues(ops, orc, fmt):
    from aethermind_b200 import _lib as L
    m, k, inter, n = 4, 4096, 1024, 2048
    rng = np.random.default_rng(2)
    x = orc.bf16_round(rng.normal(0, 1, (m, k)).astype(np.float32))
    res = orc.bf16_round(rng.normal(0, 1, (m, n)).astype(np.float32))
    pw, host = _w(ops, orc, fmt, n, k)
    xr = bf16_dev(res)
    y = ops.linear(bf16_dev(x), pw, epilogue=L.EPI_RESIDUAL_ADD, residual=xr, out=xr)  # in place
    ref = orc.bf16_round(res + _oracle_linear(orc, fmt, x, host))
    np.testing.assert_allclose(to_np(y), ref, rtol=BF_RTOL, atol=BF_ATOL)
    # gate/up interleaved + SiLU-Mul
    if fmt == "int4":
        gq, gs = ops.synth_w4(8, 1, inter, k, orc.W4_BASE)
        uq, us = ops.synth_w4(8, 2, inter, k, orc.W4_BASE)
        gu = ops.prepack_gate_up(L.WFMT_INT4, gq, gs, uq, us, inter, k)
        g = orc.linear_w4(x, gq.cpu().numpy(), gs.cpu().numpy().view(np.uint16))
        u = orc.linear_w4(x, uq.cpu().numpy(), us.cpu().numpy().view(np.uint16))
    else:
        gq, gs = ops.synth_w8(8, 1, inter, k, orc.W8_BASE)
        uq, us = ops.synth_w8(8, 2, inter, k, orc.W8_BASE)
        gu = ops.prepack_gate_up(L.WFMT_INT8, gq, gs, uq, us, inter, k)
        g = orc.linear_w8(x, gq.cpu().numpy(), gs.cpu().numpy())
        u = orc.linear_w8(x, uq.cpu().numpy(), us.cpu().numpy())
    y = ops.linear(bf16_dev(x), gu, epilogue=L.EPI_SILU_MUL)
    np.testing.assert_allclose(to_np(y), orc.silu_mul(g, u, bf=True), rtol=BF_RTOL, atol=BF_ATOL)
    # the same weights through the prefill GEMM path (m = 64)
    x64 = orc.bf16_round(rng.normal(0, 1, (64, k)).astype(np.float32))
    y64 = ops.linear(bf16_dev(x64), gu, epilogue=L.EPI_SILU_MUL)
    g64 = _oracle_linear(orc, fmt, x64, (gq.cpu().numpy(), gs.cpu().numpy().view(np.uint16) if fmt == "int4" else gs.cpu().numpy()))
    u64 = _oracle_linear(orc, fmt, x64, (uq.cpu().numpy(), us.cpu().numpy().view(np.uint16) if fmt == "int4" else us.cpu().numpy()))
    np.testing.assert_allclose(to_np(y64), orc.silu_mul(g64, u64, bf=True), rtol=BF_RTOL, atol=BF_ATOL)


def test_plain_f32_linear(ops, orc):
    from aethermind_b200 import _lib as L
    rng = np.random.default_rng(4)
    x = rng.normal(0, 1, (16, 256)).astype(np.float32)
    w = rng.normal(0, 0.02, (688, 256)).astype(np.float32)
    pw = ops.PackedWeight(L.WFMT_PLAIN, 688, 256, L.F32, 128, dev(w), None)
    y = ops.linear(dev(x), pw)
    np.testing.assert_allclose(to_np(y), orc.linear_f32(x, w), rtol=F32_RTOL, atol=1e-6)


# ------------------------------------------------------------- rope / kv / attention
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_rope_kv_write_matches_oracle(ops, orc, dtype):
    nq, nkv, d, theta, M, cap = 32, 8, 128, 500000.0, 5, 64
    rng = np.random.default_rng(0)
    q = rng.normal(0, 1, (M, nq * d)).astype(np.float32)
    k = rng.normal(0, 1, (M, nkv * d)).astype(np.float32)
    v = rng.normal(0, 1, (M, nkv * d)).astype(np.float32)
    bf = dtype == "bf16"
    if bf:
        q, k, v = orc.bf16_round(q), orc.bf16_round(k), orc.bf16_round(v)
    mk = bf16_dev if bf else dev
    qd, kd, vd = mk(q), mk(k), mk(v)
    tdt = torch.bfloat16 if bf else torch.float32
    kc = torch.zeros(1, nkv, cap, d, dtype=tdt, device="cuda")
    vc = torch.zeros_like(kc)
    seq_pos = torch.tensor([40], dtype=torch.int32, device="cuda")
    ops.rope_kv_write(qd, kd, vd, kc, vc, seq_pos, M, nq, nkv, d, theta)
    pos = 40 + np.arange(M)
    qr = orc.rope(q, pos, nq, d, theta, bf=bf)
    kr = orc.rope(k, pos, nkv, d, theta, bf=bf)
    np.testing.assert_array_equal(to_np(qd), qr)
    kcn = to_np(kc)
    for i in range(M):
        np.testing.assert_array_equal(kcn[0, :, 40 + i, :], kr[i].reshape(nkv, d))
        np.testing.assert_array_equal(to_np(vc)[0, :, 40 + i, :], v[i].reshape(nkv, d))
    assert not kcn[0, :, :40].any()  # nothing written outside [pos, pos + M)


def test_rope_out_of_capacity_sets_status(ops):
    q = torch.zeros(1, 4 * 64, device="cuda")
    kv = torch.zeros(1, 2 * 64, device="cuda")
    kc = torch.zeros(1, 2, 8, 64, device="cuda")
    vc = torch.zeros_like(kc)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.rope_kv_write(q, kv, kv, kc, vc, torch.tensor([8], dtype=torch.int32, device="cuda"), 1, 4, 2, 64, 1e4,
                      status=st)
    assert int(st.item()) == 11 and not kc.any()


@pytest.mark.parametrize("L", [512, 2048, 8192])
def test_attention_decode_matches_oracle(ops, orc, L):
    nq, nkv, d = 32, 8, 128
    rng = np.random.default_rng(L)
    q = orc.bf16_round(rng.normal(0, 1, (1, nq * d)).astype(np.float32))
    kp = orc.bf16_round(rng.normal(0, 1, (nkv, L, d)).astype(np.float32))
    vp = orc.bf16_round(rng.normal(0, 1, (nkv, L, d)).astype(np.float32))
    kc, vc = bf16_dev(kp)[None], bf16_dev(vp)[None]
    seq_pos = torch.tensor([L - 1], dtype=torch.int32, device="cuda")
    out = ops.attention(bf16_dev(q), kc, vc, seq_pos, 1, nq, nkv, d, max_context=L)
    ref = orc.attention(q, kp, vp, L - 1, nq, nkv, d, bf=True)
    np.testing.assert_allclose(to_np(out), ref, rtol=BF_RTOL, atol=BF_ATOL)


def test_attention_decode_batch_slots(ops, orc):
    nq, nkv, d, cap = 8, 2, 64, 96
    rng = np.random.default_rng(9)
    B = 3
    q = orc.bf16_round(rng.normal(0, 1, (B, nq * d)).astype(np.float32))
    kp = orc.bf16_round(rng.normal(0, 1, (B, nkv, cap, d)).astype(np.float32))
    vp = orc.bf16_round(rng.normal(0, 1, (B, nkv, cap, d)).astype(np.float32))
    pos = np.array([5, 60, 95], np.int32)
    out = ops.attention(bf16_dev(q), bf16_dev(kp), bf16_dev(vp), dev(pos), 1, nq, nkv, d, max_context=cap)
    for b in range(B):
        ref = orc.attention(q[b:b + 1], kp[b], vp[b], int(pos[b]), nq, nkv, d, bf=True)
        np.testing.assert_allclose(to_np(out)[b:b + 1], ref, rtol=BF_RTOL, atol=BF_ATOL)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_attention_prefill_causal(ops, orc, dtype):
    nq, nkv, d, M, p0, cap = 32, 8, 128, 48, 16, 128
    rng = np.random.default_rng(1)
    bf = dtype == "bf16"
    rnd = orc.bf16_round if bf else (lambda a: a)
    q = rnd(rng.normal(0, 1, (M, nq * d)).astype(np.float32))
    kp = rnd(rng.normal(0, 1, (nkv, cap, d)).astype(np.float32))
    vp = rnd(rng.normal(0, 1, (nkv, cap, d)).astype(np.float32))
    mk = bf16_dev if bf else dev
    out = ops.attention(mk(q), mk(kp)[None], mk(vp)[None], torch.tensor([p0], dtype=torch.int32, device="cuda"),
                        M, nq, nkv, d, decode=False)
    ref = orc.attention(q, kp, vp, p0, nq, nkv, d, bf=bf)
    if bf:
        np.testing.assert_allclose(to_np(out), ref, rtol=BF_RTOL, atol=BF_ATOL)
    else:
        np.testing.assert_allclose(to_np(out), ref, rtol=F32_RTOL, atol=1e-5)


@pytest.mark.parametrize("nq,nkv,d,R,B", [(32, 8, 128, 130, 1), (32, 8, 64, 64, 2), (64, 8, 128, 200, 2),
                                         (8, 8, 64, 17, 1)])
def test_attention_prefill_shapes(ops, orc, nq, nkv, d, R, B):
    """Prefill attention (bf16: the tensor-core flash kernel) over ragged row
    counts, head_dim 64 and 128, GQA groups 1/4/8 and two sequences with
    different start positions, against the oracle sequence by sequence."""
    cap = 512
    rng = np.random.default_rng(R + d)
    p0s = [5, 100][:B]
    q = orc.bf16_round(rng.normal(0, 1, (B * R, nq * d)).astype(np.float32))
    kc = orc.bf16_round(rng.normal(0, 1, (B, nkv, cap, d)).astype(np.float32))
    vc = orc.bf16_round(rng.normal(0, 1, (B, nkv, cap, d)).astype(np.float32))
    out = ops.attention(bf16_dev(q), bf16_dev(kc), bf16_dev(vc), torch.tensor(p0s, dtype=torch.int32, device="cuda"),
                        R, nq, nkv, d, decode=False)
    got = to_np(out)
    for b in range(B):
        ref = orc.attention(q[b * R:(b + 1) * R], kc[b], vc[b], p0s[b], nq, nkv, d, bf=True)
        np.testing.assert_allclose(got[b * R:(b + 1) * R], ref, rtol=BF_RTOL, atol=BF_ATOL)


@pytest.mark.parametrize("fmt", ["int4", "int8"])
@pytest.mark.parametrize("m,k", [(8, 14336), (7, 16384), (8, 4096 * 3)])
@pytest.mark.parametrize("residual", [False, True])
def test_gemv_k_split_cluster(ops, orc, fmt, m, k, residual):
    """Activation rows too long to stage whole in one CTA (8 x 14336 bf16)
    take the 2-CTA cluster that splits K (each CTA stages half of every row,
    rank 1 hands its partials to rank 0 through distributed shared memory):
    against the oracle, including the residual epilogue applied by rank 0."""
    from aethermind_b200 import _lib as L
    n = 4096
    pw, host = _w(ops, orc, fmt, n, k, seed=k + m)
    rng = np.random.default_rng(k)
    x = orc.bf16_round(rng.normal(0, 1, (m, k)).astype(np.float32))
    ref = _oracle_linear(orc, fmt, x, host)
    if residual:
        res = orc.bf16_round(rng.normal(0, 1, (m, n)).astype(np.float32))
        xr = bf16_dev(res)
        y = ops.linear(bf16_dev(x), pw, epilogue=L.EPI_RESIDUAL_ADD, residual=xr, out=xr)
        ref = orc.bf16_round(res + ref)
    else:
        y = ops.linear(bf16_dev(x), pw)
    np.testing.assert_allclose(to_np(y), ref, rtol=BF_RTOL, atol=5e-2 if residual else BF_ATOL)
    import ctypes as C
    err = C.c_int32(0)
    assert L.lib().amcu_device_error(C.byref(err), 1) == 0 and err.value == 0  # no wait ran out


# ------------------------------------------------------------- elementwise
@pytest.mark.parametrize("nq,nkv,d", [(32, 8, 128), (32, 8, 64), (16, 8, 128), (8, 8, 64)])
def test_fused_rope_attention_matches_two_step_path(ops, orc, nq, nkv, d):
    """amcu_attn_decode_rope == amcu_rope_kv_write + amcu_attn_decode: same
    appended cache rows (bit-exact) and the same outputs within bf16 rounding;
    ragged positions across sequences, including position 0 and the last
    cache slot."""
    cap, B = 1024, 4
    rng = np.random.default_rng(nq + d)
    pos = np.array([0, 37, 700, cap - 1], np.int32)
    qkv = bf16_dev(rng.normal(0, 1, (B, (nq + 2 * nkv) * d)).astype(np.float32))
    kc = bf16_dev(rng.normal(0, 1, (B, nkv, cap, d)).astype(np.float32))
    vc = bf16_dev(rng.normal(0, 1, (B, nkv, cap, d)).astype(np.float32))
    q, k, v = qkv[:, :nq * d], qkv[:, nq * d:(nq + nkv) * d], qkv[:, (nq + nkv) * d:]
    sp = dev(pos)
    table = torch.empty(cap * d // 2 * 2, dtype=torch.float32, device="cuda")
    from aethermind_b200 import _lib as L
    L.check(L.lib().amcu_rope_table(500000.0, d, cap, table.data_ptr(), torch.cuda.current_stream().cuda_stream),
            "amcu_rope_table")
    kc2, vc2, q2 = kc.clone(), vc.clone(), q.clone()
    fused = ops.attention_rope_decode(q, k, v, kc, vc, sp, nq, nkv, d, 500000.0, cos_sin=table)
    ops.rope_kv_write(q2, k, v, kc2, vc2, sp, 1, nq, nkv, d, 500000.0)
    ref = ops.attention(q2, kc2, vc2, sp, 1, nq, nkv, d, max_context=cap)
    torch.cuda.synchronize()
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    assert torch.equal(q, qkv[:, :nq * d])  # q untouched
    np.testing.assert_allclose(to_np(fused), to_np(ref), rtol=BF_RTOL, atol=BF_ATOL)
    # and against the oracle for one sequence
    b = 2
    qr = to_np(q2)[b:b + 1]
    ro = orc.attention(qr, to_np(kc2)[b], to_np(vc2)[b], int(pos[b]), nq, nkv, d, bf=True)
    np.testing.assert_allclose(to_np(fused)[b:b + 1], ro, rtol=BF_RTOL, atol=BF_ATOL)


def test_fused_rope_attention_out_of_range_sets_status(ops):
    nq, nkv, d, cap = 8, 2, 64, 64
    q = torch.zeros(1, nq * d, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(1, nkv * d, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(1, nkv, cap, d, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.attention_rope_decode(q, kv, kv, kc, vc, torch.tensor([cap], dtype=torch.int32, device="cuda"), nq, nkv, d,
                              10000.0, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 11  # AM_STATUS_OUT_OF_RANGE
    assert torch.count_nonzero(kc).item() == 0


def test_silu_mul_and_add_match_reference_bits(ops, orc, gold):
    g = torch.from_numpy(gold["silu_g_bf16"].view(np.int16)).cuda().view(torch.bfloat16)
    u = torch.from_numpy(gold["silu_u_bf16"].view(np.int16)).cuda().view(torch.bfloat16)
    y = ops.silu_mul(g, u)
    got = y.view(torch.int16).cpu().numpy().view(np.uint16)
    # device expf may differ from the host libm in the last fp32 bit: allow 1 bf16 ulp
    diff = np.abs(got.astype(np.int32) - gold["silu_bf16"].astype(np.int32))
    assert diff.max() <= 1 and (diff == 0).mean() > 0.99
    yf = ops.silu_mul(dev(gold["silu_g"]), dev(gold["silu_u"]))
    np.testing.assert_allclose(to_np(yf), gold["silu_f32"], rtol=1e-5, atol=1e-30)
    a = torch.from_numpy(gold["add_bf16_a"].view(np.int16)).cuda().view(torch.bfloat16)
    b = torch.from_numpy(gold["add_bf16_b"].view(np.int16)).cuda().view(torch.bfloat16)
    c = ops.add(a, b)
    np.testing.assert_array_equal(c.view(torch.int16).cpu().numpy().view(np.uint16), gold["add_bf16_out"])


def test_argmax_ties_and_gap(ops):
    x = torch.zeros(3, 128256, dtype=torch.bfloat16, device="cuda")
    x[0, 7] = 3.0
    x[0, 70000] = 3.0  # tie -> lowest index
    x[1, 128255] = 1.0
    x[2, 5] = 2.0
    x[2, 6] = 1.5
    idx, gap = ops.argmax(x, with_gap=True)
    assert idx.tolist() == [7, 128255, 5]
    assert gap[0].item() == 0.0 and abs(gap[2].item() - 0.5) < 1e-6
    r = torch.randn(4, 50000, device="cuda")
    assert torch.equal(ops.argmax(r), torch.argmax(r, dim=1))


def test_embedding_matches_reference(ops, gold):
    t, ids = gold["emb_table"], gold["emb_ids"]
    out = ops.embedding(dev(ids), dev(t))
    np.testing.assert_array_equal(to_np(out), gold["emb_out"])
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    bad = ops.embedding(dev(np.array([1, 64], np.int64)), dev(t), status=st)
    assert int(st.item()) == int(gold["emb_bad_status"][0])
    assert not bad[1].any()
    ids32 = dev(ids.astype(np.int32))
    np.testing.assert_array_equal(to_np(ops.embedding(ids32, dev(t))), gold["emb_out"])


def test_embedding_int8_rows(ops, orc):
    q, s = orc.synth_w8(4, 1, 64, 128, orc.W8_BASE)
    ids = np.array([3, 0, 63], np.int64)
    out = ops.embedding(dev(ids), dev(q), row_scales=dev(s))
    ref = orc.bf16_round(q[ids].astype(np.float32) * s[ids][:, None])
    np.testing.assert_array_equal(to_np(out), ref)
