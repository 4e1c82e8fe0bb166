"""End-to-end greedy generation through the am_* session ABI vs the CPU oracle.

Greedy token ids must match the oracle except at documented near-ties, where
the oracle's top-1/top-2 logit gap is below the threshold (1e-4 for fp32
models; 0.125, 4 bf16 ulps of a logit in [4, 8), for bf16 models, whose
logits are stored in bf16 as the reference Linear does). The fp32 tiny model
is compared up to its first near-tie; the quantized models at every position
(tests.model_fixtures.walk_greedy restarts the engine on the oracle's prefix
after a near-tie flip).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from tests.model_fixtures import NEAR_TIE_BF16, walk_greedy  # noqa: E402


def _compare(got, ref, gaps, tie):
    for i, (a, b) in enumerate(zip(got, ref)):
        if a != b:
            assert gaps[i] < tie, (f"token {i}: {a} != {b} with oracle gap {gaps[i]:.4g} >= {tie}; "
                                   f"engine {list(got)[:12]} oracle {list(ref)[:12]}")
            return i
    return len(ref)


@pytest.fixture(scope="module")
def sess_mod(built_lib):
    from aethermind_b200 import session
    return session


@pytest.fixture(scope="module")
def rt(sess_mod):
    return sess_mod.Runtime(0)


def test_tiny_f32_model_matches_oracle(sess_mod, rt, oracle_lib):
    from tests.model_fixtures import load_tiny_into_engine, tiny_oracle_model, tiny_prompt, tiny_weights
    cfg = sess_mod.TINY_F32
    w = tiny_weights(cfg)
    m = sess_mod.Model(rt, cfg)
    load_tiny_into_engine(m, w)
    s = sess_mod.Session(m)
    prompt = tiny_prompt(cfg)
    got = s.generate(prompt, 32)
    ref, gaps = tiny_oracle_model(cfg, w).generate(prompt.astype(np.int64), 32)
    n = _compare(got.tolist(), ref.tolist(), gaps, 1e-4)
    assert n >= 16, f"only {n} tokens matched before a near-tie"
    # CUDA graph replay and eager execution produce identical tokens
    s2 = sess_mod.Session(m, use_cuda_graph=False)
    np.testing.assert_array_equal(s2.generate(prompt, 32), got)
    # a second call on the same session reuses the captured graph
    np.testing.assert_array_equal(s.generate(prompt, 32), got)


def _small(cfg_name, sess_mod, layers=2):
    import dataclasses
    base = getattr(sess_mod, cfg_name)
    return dataclasses.replace(base, layers=layers, max_seq=256, max_batch=2)


@pytest.mark.parametrize("cfg_name", ["LLAMA_8B_W4", "LLAMA_1B_W8", "LLAMA_70B_W4"])
def test_quantized_model_matches_oracle(sess_mod, rt, oracle_lib, cfg_name):
    cfg = _small(cfg_name, sess_mod)
    m = sess_mod.Model(rt, cfg)
    m.init_synthetic(seed=0)
    s = sess_mod.Session(m)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, 16).astype(np.uint32)
    got = s.generate(prompt, 8)
    om = oracle_lib.synthetic_oracle_model(cfg, seed=0)
    ref, gaps = om.generate(prompt.astype(np.int64), 8)
    # every position is compared (restarting on the oracle's prefix after a near-tie flip)
    flips = walk_greedy(s, prompt, ref, gaps, NEAR_TIE_BF16)
    assert len(flips) <= 2, f"near-tie flips at {flips}, oracle gaps {gaps.tolist()}"
    # the unfused RoPE + attention steps give the same tokens
    s_unfused = sess_mod.Session(m, fused_attention=False)
    np.testing.assert_array_equal(s_unfused.generate(prompt, 8), got)
    # batch of 2 equals two single runs (per-row math is independent of the batch)
    p2 = np.stack([prompt, np.random.default_rng(6).integers(0, cfg.vocab, 16).astype(np.uint32)])
    gb = s.generate(p2, 8)
    np.testing.assert_array_equal(gb[0], got)
    np.testing.assert_array_equal(gb[1], s.generate(p2[1], 8))


def test_batch8_rows_equal_single_runs(sess_mod, rt):
    """Batch 8 (the decode GEMVs' largest m: the down projection's 8 rows of
    K = 14336 go in two row slices) gives every sequence the tokens it gets
    alone."""
    import dataclasses
    cfg = dataclasses.replace(sess_mod.LLAMA_8B_W4, layers=2, max_seq=128, max_batch=8)
    m = sess_mod.Model(rt, cfg)
    m.init_synthetic(seed=4)
    s = sess_mod.Session(m)
    p8 = np.random.default_rng(13).integers(0, cfg.vocab, (8, 12)).astype(np.uint32)
    got = s.generate(p8, 6)
    for i in range(8):
        np.testing.assert_array_equal(got[i], s.generate(p8[i], 6))


def test_persistent_decode_matches_per_op_plan(sess_mod, rt, oracle_lib):
    """The persistent decode step (one launch for all layers, batch 1, INT4)
    against the oracle and the per-op decode plan: every position compared
    (near-tie flips allowed: its GEMVs sum in another order, so fp32 sums
    round differently); eager and graph replay give the same tokens; batch 2
    takes the per-op plan."""
    import dataclasses
    cfg = dataclasses.replace(sess_mod.LLAMA_8B_W4, layers=3, max_seq=1024, max_batch=2)
    m = sess_mod.Model(rt, cfg)
    m.init_synthetic(seed=1)
    # 300 prompt tokens: the attention phase splits the keys (256 per split)
    prompt = np.random.default_rng(9).integers(0, cfg.vocab, 300).astype(np.uint32)
    s_p = sess_mod.Session(m, persistent_decode=True)
    assert any("DecodeStackPersistent" in l for l in s_p.plan_steps(1, 1, 1))
    assert not any("DecodeStackPersistent" in l for l in s_p.plan_steps(1, 2, 1))
    ref, gaps = oracle_lib.synthetic_oracle_model(cfg, seed=1).generate(prompt.astype(np.int64), 24)
    flips = walk_greedy(s_p, prompt, ref, gaps, NEAR_TIE_BF16)
    assert len(flips) <= 4, f"near-tie flips at {flips}"
    got = s_p.generate(prompt, 24)
    per_op = sess_mod.Session(m).generate(prompt, 24)
    assert _compare(got.tolist(), per_op.tolist(), gaps, NEAR_TIE_BF16) >= 8
    np.testing.assert_array_equal(sess_mod.Session(m, use_cuda_graph=False, persistent_decode=True).generate(prompt, 24),
                                  got)
    # a full 8B-depth stack (32 layers) on a short prompt against the per-op plan
    cfg32 = dataclasses.replace(sess_mod.LLAMA_8B_W4, max_seq=128, max_batch=1)
    m32 = sess_mod.Model(rt, cfg32)
    m32.init_synthetic(seed=0)
    p32 = np.random.default_rng(100).integers(0, cfg32.vocab, 16).astype(np.uint32)
    a = sess_mod.Session(m32, persistent_decode=True).generate(p32, 16)
    b = sess_mod.Session(m32).generate(p32, 16)
    assert _compare(a.tolist(), b.tolist(), np.zeros(16), 1.0) >= 12


def test_plan_resolves_phase_kernels(sess_mod, rt):
    cfg = _small("LLAMA_8B_W4", sess_mod, layers=1)
    m = sess_mod.Model(rt, cfg)
    m.init_synthetic(0)
    s = sess_mod.Session(m)
    dec = s.plan_steps(1, 1, 1)
    pre = s.plan_steps(0, 1, 16)
    assert any("GemvW4G128_CUDA_Decode" in l for l in dec)
    assert any("RoPEAttnDecodeCluster_CUDA_BF16" in l for l in dec)
    # every batch size decodes one row per sequence: the fused kernel applies
    assert any("RoPEAttnDecodeCluster_CUDA_BF16" in l for l in s.plan_steps(1, 2, 1))
    unf = sess_mod.Session(m, fused_attention=False).plan_steps(1, 1, 1)
    assert any("AttnDecodeSplitK" in l for l in unf)
    assert any("GemmW4G128_CUDA_Prefill" in l for l in pre)
    assert any("AttnPrefill" in l for l in pre)
    names = [l.split()[0] for l in dec]
    assert names[0] == "embedding" and names[-1] == "argmax"


def test_session_errors(sess_mod, rt):
    from aethermind_b200._lib import AmError
    cfg = _small("LLAMA_8B_W4", sess_mod, layers=1)
    m = sess_mod.Model(rt, cfg)
    m.init_synthetic(0)
    s = sess_mod.Session(m)
    with pytest.raises(AmError) as e:
        s.generate(np.zeros(250, np.uint32), 10)  # 250 + 10 > max_seq 256
    assert e.value.code == 11
    with pytest.raises(AmError) as e:
        s.generate(np.array([cfg.vocab], np.uint32), 2)
    assert e.value.code == 11
    # the session stays usable after errors
    assert s.generate(np.array([1, 2, 3], np.uint32), 2).shape == (2,)
