"""The C-ABI library loads, exports every declared symbol, and its host logic
(kernel registry, KV layout/session contract, error objects, argument
validation) behaves like the reference's -- all without a GPU."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions() -> list[str]:
    text = (ROOT / "include" / "aethermind_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:amcu|am)_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(built_lib):
    names = declared_functions()
    assert len(names) > 40
    missing = [n for n in names if not hasattr(built_lib, n)]
    assert not missing, missing


def test_python_binding_covers_header(built_lib):
    from aethermind_b200 import _lib
    assert set(declared_functions()) <= set(_lib.exported_symbols())


def test_error_objects(built_lib):
    e = built_lib.am_error_create(11, b"bad token")
    assert built_lib.am_error_code(e) == 11
    assert built_lib.am_error_message(e) == b"bad token"
    built_lib.am_error_destroy(e)
    assert built_lib.amcu_version().startswith(b"aethermind_b200")


def _resolve(lib, op, act, w, fmt, phase):
    buf = C.create_string_buffer(128)
    code = lib.am_debug_resolve_kernel(op, act, w, fmt, phase, buf, 128)
    return code, buf.value.decode()


def test_registry_selection_rules(built_lib):
    from aethermind_b200 import _lib as L
    LINEAR, RMSNORM, ATTN, ARGMAX = 3, 2, 6, 13
    assert built_lib.am_debug_registry_size() >= 20
    # phase-specific kernels win for their phase; kBoth kernels serve both
    assert _resolve(built_lib, LINEAR, L.BF16, L.I4, 3, 1) == (0, "GemvW4G128_CUDA_Decode")
    assert _resolve(built_lib, LINEAR, L.BF16, L.I4, 3, 0) == (0, "GemmW4G128_CUDA_Prefill")
    assert _resolve(built_lib, LINEAR, L.BF16, L.I8, 2, 1) == (0, "GemvW8_CUDA_Decode")
    assert _resolve(built_lib, RMSNORM, L.F32, L.F32, 0, 1) == (0, "RmsNorm_CUDA_F32")
    assert _resolve(built_lib, RMSNORM, L.BF16, L.BF16, 0, 0) == (0, "RmsNorm_CUDA_BF16")
    assert _resolve(built_lib, ATTN, L.BF16, L.BF16, 0, 1)[1] == "AttnDecodeSplitK_CUDA_BF16"
    assert _resolve(built_lib, ATTN, L.BF16, L.BF16, 0, 0)[1] == "AttnPrefill_CUDA_BF16"
    # exact dtype/format match is required
    assert _resolve(built_lib, LINEAR, L.F32, L.I4, 3, 1)[0] == 5  # NOT_FOUND
    assert _resolve(built_lib, ARGMAX, L.BF16, L.BF16, 3, 1)[0] == 5


@pytest.fixture(scope="module")
def gold():
    return np.load(ROOT / "tests" / "golden" / "ref_kernels.npz")


def test_kv_layout_matches_reference(built_lib, gold):
    for row in gold["kv_cases"].astype(np.int64):
        L_, H, T, D, dt, l, h, p, d, st, off, bpp = (int(v) for v in row)
        o, b = C.c_uint64(), C.c_uint64()
        code = built_lib.am_debug_kv_offset(L_, H, T, D, dt, 1, l, h, p, d, 0, C.byref(o), C.byref(b))
        assert code == st
        if st == 0:
            assert (o.value, b.value) == (off, bpp)


def test_kv_slot_axis_extends_layout(built_lib):
    # slot s of layer l starts one slot-plane after slot s-1; slot 0 is the reference layout
    o0, o1, b = C.c_uint64(), C.c_uint64(), C.c_uint64()
    assert built_lib.am_debug_kv_offset(4, 8, 128, 64, 1, 3, 2, 5, 7, 9, 0, C.byref(o0), C.byref(b)) == 0
    assert built_lib.am_debug_kv_offset(4, 8, 128, 64, 1, 3, 2, 5, 7, 9, 1, C.byref(o1), C.byref(b)) == 0
    assert o1.value - o0.value == 8 * 128 * 64 * 2
    assert b.value == 4 * 3 * 8 * 128 * 64 * 2


def test_kv_reservation_contract_matches_reference(built_lib, gold):
    for m, pl, mn, st in gold["kv_reserve"]:
        assert built_lib.am_debug_kv_reserve(int(m), int(pl), int(mn)) == int(st)


def test_argument_validation_without_gpu(built_lib):
    from aethermind_b200 import _lib as L
    a = L.AmcuRmsNormArgs()
    a.rows, a.hidden = 0, 16
    assert built_lib.amcu_rmsnorm(C.byref(a), None) == 0  # empty batch is OK, touches nothing
    a.rows, a.hidden = 4, 0
    assert built_lib.amcu_rmsnorm(C.byref(a), None) == 3
    assert b"hidden" in built_lib.amcu_last_error()
    la = L.AmcuLinearArgs()
    la.m, la.w.n, la.w.k, la.w.format = 1, 16, 100, L.WFMT_INT4
    la.x = la.y = la.w.data = la.w.scales = 256
    la.act_dtype = L.BF16
    la.w.group = 128
    assert built_lib.amcu_linear(C.byref(la), None) == 3  # k % 64 != 0
    # INT4 pair records carry the group scales: 2 x 512 B of nibbles + 32 B of fp16 scales per 16 x 128
    assert built_lib.amcu_packed_weight_bytes(L.WFMT_INT4, L.BF16, 4096, 4096, 128) == 4096 * 2048 + 4096 * 32 * 2
    assert built_lib.amcu_packed_scale_bytes(L.WFMT_INT4, 4096, 4096, 128) == 0
    assert built_lib.amcu_packed_weight_bytes(L.WFMT_INT8, L.BF16, 64, 1792, 128) == 64 * 1792
    assert built_lib.amcu_packed_scale_bytes(L.WFMT_INT8, 64, 1792, 128) == 64 * 4
    err = C.c_void_p()
    assert built_lib.am_model_load(None, b"/nonexistent", C.byref(err)) is None
    assert built_lib.am_error_code(err) == 3  # no runtime
    built_lib.am_error_destroy(err)
