"""Checkpoint loading (am_model_load / am_model_load_ex) of Hugging Face Llama
directories, against the CPU oracle.

* The device quantizer (amcu_quantize_weight) gives the same bytes as the
  oracle's restatement of its recipe (symmetric absmax; INT4 per group of 128
  with fp16 scales, INT8 per row with fp32 scales), from BF16, F16 and F32.
* A tiny Llama checkpoint (tests/hf_fixtures.py) loads as INT4, INT8 and
  plain bf16, single-file and sharded, tied and untied, and generates the
  oracle's greedy tokens (every position compared; near-tie flips allowed).
* Malformed directories fail with the reference loader's status codes.
"""
import ctypes as C
import json

import numpy as np
import pytest

from tests.hf_fixtures import TINY_HF, make_weights, oracle_model, stored_values, write_checkpoint
from tests.model_fixtures import NEAR_TIE_BF16, walk_greedy

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rt(built_lib):
    from aethermind_b200 import session
    return session.Runtime(0)


@pytest.mark.parametrize("src", ["BF16", "F16", "F32"])
def test_quantizer_matches_oracle_bytes(built_lib, oracle_lib, src):
    from aethermind_b200 import _lib as L
    rng = np.random.default_rng(3)
    n, k = 48, 512
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    w[3] = 0.0                      # an all-zero row / groups: s = 0, q = 0
    w[5, 7] = 0.5                   # one large value dominating its group
    vals = stored_values(w, src)
    t = torch.from_numpy(vals).cuda()
    t = {"BF16": t.to(torch.bfloat16), "F16": t.to(torch.float16), "F32": t}[src]
    dt = {"BF16": L.BF16, "F16": L.F16, "F32": L.F32}[src]
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    q4 = torch.empty(n, k // 2, dtype=torch.uint8, device="cuda")
    s4 = torch.empty(n, k // 128, dtype=torch.int16, device="cuda")
    L.check(built_lib.amcu_quantize_weight(L.WFMT_INT4, t.data_ptr(), dt, n, k, 128, q4.data_ptr(), s4.data_ptr(),
                                           stream), "quantize int4")
    q8 = torch.empty(n, k, dtype=torch.int8, device="cuda")
    s8 = torch.empty(n, dtype=torch.float32, device="cuda")
    L.check(built_lib.amcu_quantize_weight(L.WFMT_INT8, t.data_ptr(), dt, n, k, 0, q8.data_ptr(), s8.data_ptr(),
                                           stream), "quantize int8")
    torch.cuda.synchronize()
    rq4, rs4 = oracle_lib.quantize_w4(vals)
    np.testing.assert_array_equal(q4.cpu().numpy(), rq4)
    np.testing.assert_array_equal(s4.cpu().numpy().view(np.uint16), rs4)
    rq8, rs8 = oracle_lib.quantize_w8(vals)
    np.testing.assert_array_equal(q8.cpu().numpy(), rq8)
    np.testing.assert_array_equal(s8.cpu().numpy(), rs8)


@pytest.mark.parametrize("fmt_name,dtype,shards,tied", [
    ("INT4", "BF16", 2, False),
    ("INT4", "F16", 1, True),
    ("INT8", "BF16", 1, True),
    ("INT8", "F32", 3, False),
    ("PLAIN", "BF16", 1, False),
])
def test_loaded_checkpoint_generates_oracle_tokens(rt, oracle_lib, tmp_path, fmt_name, dtype, shards, tied):
    from aethermind_b200 import _lib as L
    from aethermind_b200 import session
    fmt = {"INT4": L.WFMT_INT4, "INT8": L.WFMT_INT8, "PLAIN": L.WFMT_PLAIN}[fmt_name]
    cfg = dict(TINY_HF, tie_word_embeddings=tied)
    w = make_weights(cfg, seed=7)
    d = write_checkpoint(tmp_path / "ckpt", cfg, w, dtype=dtype, shards=shards)
    m = session.Model.load(rt, d, weight_format=fmt, max_seq=128)
    s = session.Session(m)
    prompt = np.random.default_rng(11).integers(0, cfg["vocab_size"], 12).astype(np.uint32)
    ref, gaps = oracle_model(cfg, w, dtype, fmt, 128).generate(prompt.astype(np.int64), 16)
    flips = walk_greedy(s, prompt, ref, gaps, NEAR_TIE_BF16)
    assert len(flips) <= 3, f"near-tie flips at {flips}; oracle gaps {np.round(gaps, 4).tolist()}"


def test_default_load_is_int4_and_sharded_equals_single_file(rt, tmp_path):
    """am_model_load (no options): INT4 g128, bf16; the same tensors split
    over shards load to the same model."""
    from aethermind_b200 import _lib as L
    from aethermind_b200 import session
    w = make_weights(TINY_HF, seed=2)
    a = write_checkpoint(tmp_path / "one", TINY_HF, w, shards=1)
    b = write_checkpoint(tmp_path / "four", TINY_HF, w, shards=4)
    err = C.c_void_p()
    h = L.lib().am_model_load(rt.h, str(a).encode(), C.byref(err))
    assert h, L.lib().am_error_message(err).decode() if err.value else "load failed"
    ma = session.Model.__new__(session.Model)
    ma.rt, ma.cfg, ma._c, ma.h = rt, None, None, h
    mb = session.Model.load(rt, b, weight_format=L.WFMT_INT4, max_seq=256)
    prompt = np.arange(1, 9, dtype=np.uint32)
    np.testing.assert_array_equal(session.Session(ma).generate(prompt, 8), session.Session(mb).generate(prompt, 8))


def test_malformed_checkpoints_fail_with_reference_codes(rt, tmp_path):
    from aethermind_b200 import _lib as L
    from aethermind_b200 import session
    with pytest.raises(L.AmError) as e:
        session.Model.load(rt, tmp_path / "nope")
    assert e.value.code == L.NOT_FOUND
    w = make_weights(TINY_HF, seed=1)
    d = write_checkpoint(tmp_path / "missing", TINY_HF, {k: v for k, v in w.items() if "layers.1.mlp.up_proj" not in k})
    with pytest.raises(L.AmError) as e:
        session.Model.load(rt, d)
    assert e.value.code == L.INVALID_ARGUMENT and "layers.1.mlp.up_proj" in str(e.value)
    d = write_checkpoint(tmp_path / "shape", TINY_HF, dict(w, **{"model.norm.weight": np.ones(7, np.float32)}))
    with pytest.raises(L.AmError) as e:
        session.Model.load(rt, d)
    assert e.value.code == L.INVALID_ARGUMENT and "model.norm.weight" in str(e.value)
    d = tmp_path / "badjson"
    d.mkdir()
    (d / "config.json").write_text("{\"vocab_size\": 512,")
    with pytest.raises(L.AmError) as e:
        session.Model.load(rt, d)
    assert e.value.code == L.INVALID_ARGUMENT
    d = write_checkpoint(tmp_path / "scaled", dict(TINY_HF, rope_scaling={"rope_type": "llama3", "factor": 8.0}), w)
    with pytest.raises(L.AmError) as e:
        session.Model.load(rt, d)
    assert e.value.code == L.UNIMPLEMENTED
