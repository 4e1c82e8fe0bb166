"""amcu_attn_decode_noalloc: decode attention with the library's built-in
scratch instead of a caller workspace.

Called through the C ABI and compared with amcu_attn_decode (the workspace
entry point) on the same inputs, two calls in a row with different sizes, so
that the second call reuses scratch the first one left dirty. The file is
named to be collected last: it must pass alone and after the rest of the
suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _args(L, q, kc, vc, seq_pos, out, n_q, n_kv, d, num_splits=0):
    a = L.AmcuAttentionArgs()
    a.q, a.q_stride = q.data_ptr(), q.stride(0)
    a.k_cache, a.v_cache = kc.data_ptr(), vc.data_ptr()
    a.slot_stride, a.capacity = kc.stride(0), kc.shape[2]
    a.seq_pos = seq_pos.data_ptr()
    a.out, a.out_stride = out.data_ptr(), out.stride(0)
    a.rows, a.rows_per_seq = q.shape[0], 1
    a.n_q_heads, a.n_kv_heads, a.head_dim = n_q, n_kv, d
    a.dtype = L.BF16
    a.num_splits = num_splits
    a.max_context = kc.shape[2]
    a.workspace, a.workspace_size = None, 0
    return a


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


def test_noalloc_matches_workspace_entry(built_lib):
    import torch

    from aethermind_b200 import _lib as L
    from aethermind_b200 import ops

    n_q, n_kv, d, cap = 32, 8, 128, 2048
    for call, (rows, ctx) in enumerate([(1, 1500), (2, 700)]):
        g = torch.Generator(device="cuda").manual_seed(100 + call)
        q = torch.randn(rows, n_q * d, generator=g, device="cuda").to(torch.bfloat16)
        kc = torch.randn(rows, n_kv, cap, d, generator=g, device="cuda").to(torch.bfloat16)
        vc = torch.randn(rows, n_kv, cap, d, generator=g, device="cuda").to(torch.bfloat16)
        seq_pos = torch.tensor([ctx - 1 - 37 * r for r in range(rows)], dtype=torch.int32, device="cuda")
        out = torch.full((rows, n_q * d), float("nan"), dtype=torch.bfloat16, device="cuda")
        a = _args(L, q, kc, vc, seq_pos, out, n_q, n_kv, d)
        code = built_lib.amcu_attn_decode_noalloc(C.byref(a), C.c_void_p(_stream()))
        assert code == 0, built_lib.amcu_last_error()
        ref = ops.attention(q, kc, vc, seq_pos, 1, n_q, n_kv, d, max_context=cap)
        torch.cuda.synchronize()
        assert not torch.isnan(out.float()).any()
        np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), rtol=1e-2, atol=1e-2)


def test_noalloc_rejects_oversize(built_lib):
    import torch

    from aethermind_b200 import _lib as L

    rows, n_q, n_kv, d, cap = 64, 64, 8, 128, 8192
    q = torch.zeros(rows, n_q * d, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(1, n_kv, cap, d, dtype=torch.bfloat16, device="cuda")
    seq_pos = torch.full((rows,), cap - 1, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    a = _args(L, q, kc, kc, seq_pos, out, n_q, n_kv, d, num_splits=64)
    a.slot_stride = 0  # every row reads slot 0: validation only, nothing launches
    need = built_lib.amcu_attention_workspace_bytes(C.byref(a))
    assert need > 4 << 20
    code = built_lib.amcu_attn_decode_noalloc(C.byref(a), C.c_void_p(_stream()))
    assert code == 3  # AM_STATUS_INVALID_ARGUMENT
    assert b"scratch" in built_lib.amcu_last_error()
