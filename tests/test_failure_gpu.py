"""Bounded device waits: a wait that nobody satisfies ends with an error code
instead of a hang, and the session API reports it.

The one-shot all-reduce (tensor-parallel decode) waits for every peer's flag
in its exchange area. Here a single rank of a "world" of 2 runs alone: the
second exchange area is a plain local buffer that no peer ever signals, so the
wait runs out after its limit (1 ms here), the kernel records 0x401 in the
device error word and returns. No second rank runs at all, so no two kernels
wait on each other on one GPU.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ERR_AR_WAIT = 0x401


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _device_error(lib, clear):
    v = C.c_int32(0)
    assert lib.amcu_device_error(C.byref(v), clear) == 0
    return v.value


def _run_unanswered_allreduce(built_lib, n=4096, limit_us=1000):
    from aethermind_b200 import _lib as L
    nbytes = built_lib.amcu_allreduce_area_bytes()
    areas = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    part = torch.ones(n, dtype=torch.bfloat16, device="cuda")
    x = torch.zeros(n, dtype=torch.bfloat16, device="cuda")
    a = L.AmcuAllReduceArgs()
    a.part, a.x, a.n, a.rank, a.world = part.data_ptr(), x.data_ptr(), n, 0, 2
    a.areas[0], a.areas[1] = areas[0].data_ptr(), areas[1].data_ptr()
    a.wait_limit_us = limit_us
    L.check(built_lib.amcu_allreduce_oneshot_add(C.byref(a), C.c_void_p(_stream())), "allreduce")
    torch.cuda.synchronize()
    # the rank's own chunk did reach the "peer" area (the push ran before the wait)
    return areas


def test_allreduce_wait_runs_out_and_records_code(built_lib):
    _device_error(built_lib, 1)
    _run_unanswered_allreduce(built_lib)
    assert _device_error(built_lib, 1) == ERR_AR_WAIT
    assert _device_error(built_lib, 0) == 0  # cleared


def test_allreduce_rejects_bad_arguments(built_lib):
    from aethermind_b200 import _lib as L
    a = L.AmcuAllReduceArgs()
    a.n, a.rank, a.world = 4096, 0, 1
    assert built_lib.amcu_allreduce_oneshot_add(C.byref(a), None) == L.INVALID_ARGUMENT
    a.world, a.n = 2, 65536 + 8
    assert built_lib.amcu_allreduce_oneshot_add(C.byref(a), None) == L.INVALID_ARGUMENT


def test_session_reports_timed_out_wait(built_lib):
    """A wait that ran out before a generate call finishes is reported by that
    call as DEADLINE_EXCEEDED (the error word is read at the call's final
    synchronisation, like a sticky CUDA error), then cleared: the next call
    succeeds."""
    import dataclasses

    from aethermind_b200 import _lib as L
    from aethermind_b200 import session
    cfg = dataclasses.replace(session.LLAMA_8B_W4, layers=1, max_seq=64, max_batch=1)
    rt = session.Runtime(0)
    m = session.Model(rt, cfg)
    m.init_synthetic(0)
    s = session.Session(m)
    prompt = np.array([1, 2, 3, 4], np.uint32)
    ok = s.generate(prompt, 4)
    _device_error(built_lib, 1)
    _run_unanswered_allreduce(built_lib)
    with pytest.raises(L.AmError) as e:
        s.generate(prompt, 4)
    assert e.value.code == L.DEADLINE_EXCEEDED
    assert "0x401" in str(e.value)
    assert _device_error(built_lib, 0) == 0
    np.testing.assert_array_equal(s.generate(prompt, 4), ok)
