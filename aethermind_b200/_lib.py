"""ctypes binding of the C ABI declared in include/aethermind_b200.h.

Loading fails loudly when the compiled library is missing: there is no
Python or CPU fallback for any op.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("AMCU_LIB") or Path(__file__).resolve().parent / "lib" / "libaethermind_b200.so")

# amcu_dtype
F32, BF16, F16, I8, I4, I32, I64, U32 = range(8)
# amcu_weight_format
WFMT_PLAIN, WFMT_INT8, WFMT_INT4 = 0, 2, 3
# amcu_epilogue
EPI_STORE, EPI_RESIDUAL_ADD, EPI_SILU_MUL = 0, 1, 2

STATUS_NAMES = [
    "OK", "CANCELLED", "UNKNOWN", "INVALID_ARGUMENT", "DEADLINE_EXCEEDED", "NOT_FOUND", "ALREADY_EXISTS",
    "PERMISSION_DENIED", "RESOURCE_EXHAUSTED", "FAILED_PRECONDITION", "ABORTED", "OUT_OF_RANGE",
    "UNIMPLEMENTED", "INTERNAL", "UNAVAILABLE", "DATA_LOSS", "OVERFLOW", "UNAUTHENTICATED",
]
OK, INVALID_ARGUMENT, DEADLINE_EXCEEDED, NOT_FOUND, FAILED_PRECONDITION, OUT_OF_RANGE, UNIMPLEMENTED = \
    0, 3, 4, 5, 9, 11, 12


class AmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        self.code = code
        name = STATUS_NAMES[code] if 0 <= code < len(STATUS_NAMES) else str(code)
        super().__init__(f"{name}: {msg}")


class AmcuWeight(C.Structure):
    _fields_ = [("format", C.c_int32), ("dtype", C.c_int32), ("n", C.c_int64), ("k", C.c_int64),
                ("group", C.c_int64), ("data", C.c_void_p), ("scales", C.c_void_p),
                ("gate_up_interleaved", C.c_int32)]


class AmcuRmsNormArgs(C.Structure):
    _fields_ = [("input", C.c_void_p), ("weight", C.c_void_p), ("output", C.c_void_p),
                ("residual", C.c_void_p), ("residual_out", C.c_void_p), ("rows", C.c_int64),
                ("hidden", C.c_int64), ("input_row_stride", C.c_int64), ("output_row_stride", C.c_int64),
                ("eps", C.c_float), ("dtype", C.c_int32)]


class AmcuL2Prefetch(C.Structure):
    _fields_ = [("ptr", C.c_void_p * 4), ("bytes", C.c_uint64 * 4)]


class AmcuLinearArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("w", AmcuWeight), ("y", C.c_void_p), ("residual", C.c_void_p),
                ("m", C.c_int64), ("x_stride", C.c_int64), ("y_stride", C.c_int64),
                ("act_dtype", C.c_int32), ("epilogue", C.c_int32), ("workspace", C.c_void_p),
                ("workspace_size", C.c_size_t), ("norm_weight", C.c_void_p), ("norm_eps", C.c_float),
                ("l2_next", AmcuL2Prefetch), ("peer_reduce", C.c_void_p)]


class AmcuRopeKvArgs(C.Structure):
    _fields_ = [("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("q_stride", C.c_int64),
                ("k_stride", C.c_int64), ("v_stride", C.c_int64), ("k_cache", C.c_void_p),
                ("v_cache", C.c_void_p), ("slot_stride", C.c_int64), ("capacity", C.c_int64),
                ("seq_pos", C.c_void_p), ("rows", C.c_int64), ("rows_per_seq", C.c_int64),
                ("n_q_heads", C.c_int64), ("n_kv_heads", C.c_int64), ("head_dim", C.c_int64),
                ("theta", C.c_double), ("dtype", C.c_int32), ("status", C.c_void_p), ("cos_sin", C.c_void_p)]


class AmcuAttentionArgs(C.Structure):
    _fields_ = [("q", C.c_void_p), ("q_stride", C.c_int64), ("k_cache", C.c_void_p), ("v_cache", C.c_void_p),
                ("slot_stride", C.c_int64), ("capacity", C.c_int64), ("seq_pos", C.c_void_p),
                ("out", C.c_void_p), ("out_stride", C.c_int64), ("rows", C.c_int64),
                ("rows_per_seq", C.c_int64), ("n_q_heads", C.c_int64), ("n_kv_heads", C.c_int64),
                ("head_dim", C.c_int64), ("dtype", C.c_int32), ("num_splits", C.c_int32),
                ("max_context", C.c_int64), ("workspace", C.c_void_p), ("workspace_size", C.c_size_t)]


class AmcuEmbeddingArgs(C.Structure):
    _fields_ = [("ids", C.c_void_p), ("id_dtype", C.c_int32), ("count", C.c_int64), ("table", C.c_void_p),
                ("row_scales", C.c_void_p), ("vocab", C.c_int64), ("hidden", C.c_int64), ("out", C.c_void_p),
                ("dtype", C.c_int32), ("status", C.c_void_p)]


class AmConfig(C.Structure):
    _fields_ = [("device_id", C.c_int32), ("tp_rank", C.c_int32), ("tp_size", C.c_int32),
                ("nccl_unique_id", C.c_void_p)]


class AmModelConfig(C.Structure):
    _fields_ = [("vocab", C.c_int64), ("hidden", C.c_int64), ("layers", C.c_int64), ("n_q_heads", C.c_int64),
                ("n_kv_heads", C.c_int64), ("head_dim", C.c_int64), ("inter", C.c_int64),
                ("rms_eps", C.c_float), ("rope_theta", C.c_double), ("tied_embeddings", C.c_int32),
                ("act_dtype", C.c_int32), ("weight_format", C.c_int32), ("group_size", C.c_int64),
                ("max_seq", C.c_int64), ("max_batch", C.c_int64)]


class AmLoadOptions(C.Structure):
    _fields_ = [("weight_format", C.c_int32), ("act_dtype", C.c_int32), ("max_seq", C.c_int64),
                ("max_batch", C.c_int64)]


class AmSessionConfig(C.Structure):
    _fields_ = [("max_new_tokens", C.c_int64), ("use_cuda_graph", C.c_int32), ("unfused_attention", C.c_int32),
                ("persistent_decode", C.c_int32)]


class AmcuAllReduceArgs(C.Structure):
    _fields_ = [("part", C.c_void_p), ("x", C.c_void_p), ("n", C.c_int64), ("rank", C.c_int32),
                ("world", C.c_int32), ("areas", C.c_void_p * 8), ("wait_limit_us", C.c_uint64)]


P = C.c_void_p
_SIGS = {
    "amcu_last_error": (C.c_char_p, []),
    "amcu_version": (C.c_char_p, []),
    "amcu_device_error": (C.c_int, [C.POINTER(C.c_int32), C.c_int32]),
    "am_error_create": (P, [C.c_int, C.c_char_p]),
    "am_error_destroy": (None, [P]),
    "am_error_code": (C.c_int, [P]),
    "am_error_message": (C.c_char_p, [P]),
    "amcu_packed_weight_bytes": (C.c_int64, [C.c_int32, C.c_int32, C.c_int64, C.c_int64, C.c_int64]),
    "amcu_packed_scale_bytes": (C.c_int64, [C.c_int32, C.c_int64, C.c_int64, C.c_int64]),
    "amcu_prepack_weight_rows": (C.c_int, [C.c_int32, C.c_int32, C.c_int64, C.c_int64, C.c_int64, C.c_int64,
                                           C.c_int64, P, P, P, P, P]),
    "amcu_prepack_weight": (C.c_int, [C.c_int32, C.c_int32, C.c_int64, C.c_int64, C.c_int64, P, P, P, P, P]),
    "amcu_unpack_weight": (C.c_int, [C.c_int32, C.c_int32, C.c_int64, C.c_int64, C.c_int64, P, P, P, P, P]),
    "amcu_prepack_gate_up": (C.c_int, [C.c_int32, C.c_int32, C.c_int64, C.c_int64, C.c_int64, P, P, P, P, P, P, P]),
    "amcu_synth_w4": (C.c_int, [C.c_uint64, C.c_uint64, C.c_int64, C.c_int64, C.c_float, P, P, P]),
    "amcu_synth_w8": (C.c_int, [C.c_uint64, C.c_uint64, C.c_int64, C.c_int64, C.c_float, P, P, P]),
    "amcu_synth_uniform_bf16": (C.c_int, [C.c_uint64, C.c_uint64, C.c_int64, C.c_float, P, P]),
    "amcu_rmsnorm": (C.c_int, [C.POINTER(AmcuRmsNormArgs), P]),
    "amcu_linear": (C.c_int, [C.POINTER(AmcuLinearArgs), P]),
    "amcu_linear_workspace_bytes": (C.c_size_t, [C.POINTER(AmcuLinearArgs)]),
    "amcu_gemv_w8": (C.c_int, [C.POINTER(AmcuLinearArgs), P]),
    "amcu_gemv_w4g128": (C.c_int, [C.POINTER(AmcuLinearArgs), P]),
    "amcu_gemm_w8_prefill": (C.c_int, [C.POINTER(AmcuLinearArgs), P]),
    "amcu_gemm_w4g128_prefill": (C.c_int, [C.POINTER(AmcuLinearArgs), P]),
    "amcu_rope_kv_write": (C.c_int, [C.POINTER(AmcuRopeKvArgs), P]),
    "amcu_rope_table": (C.c_int, [C.c_double, C.c_int64, C.c_int64, P, P]),
    "amcu_attention_workspace_bytes": (C.c_size_t, [C.POINTER(AmcuAttentionArgs)]),
    "amcu_attn_decode": (C.c_int, [C.POINTER(AmcuAttentionArgs), P]),
    "amcu_attn_prefill": (C.c_int, [C.POINTER(AmcuAttentionArgs), P]),
    "amcu_attn_decode_noalloc": (C.c_int, [C.POINTER(AmcuAttentionArgs), P]),
    "amcu_attn_decode_rope": (C.c_int, [C.POINTER(AmcuRopeKvArgs), C.POINTER(AmcuAttentionArgs), P]),
    "amcu_decode_stack": (C.c_int, [P, P]),
    "amcu_decode_stack_workspace_bytes": (C.c_size_t, [P]),
    "amcu_silu_mul": (C.c_int, [P, P, P, C.c_int64, C.c_int32, P]),
    "amcu_add": (C.c_int, [P, P, P, C.c_int64, C.c_int32, P]),
    "amcu_argmax": (C.c_int, [P, C.c_int64, C.c_int64, C.c_int64, C.c_int32, P, P, P]),
    "amcu_argmax_workspace_bytes": (C.c_size_t, [C.c_int64]),
    "amcu_argmax_ws": (C.c_int, [P, C.c_int64, C.c_int64, C.c_int64, C.c_int32, P, P, P, C.c_size_t, P]),
    "amcu_embedding": (C.c_int, [C.POINTER(AmcuEmbeddingArgs), P]),
    "amcu_allreduce_area_bytes": (C.c_size_t, []),
    "amcu_allreduce_oneshot_add": (C.c_int, [C.POINTER(AmcuAllReduceArgs), P]),
    "am_runtime_create": (P, [C.POINTER(AmConfig)]),
    "am_runtime_destroy": (None, [P]),
    "am_nccl_get_unique_id": (C.c_int, [P]),
    "am_runtime_peer_handle": (C.c_int, [P, P]),
    "am_runtime_open_peers": (C.c_int, [P, P]),
    "am_last_error": (C.c_char_p, []),
    "am_model_load": (P, [P, C.c_char_p, C.POINTER(P)]),
    "am_model_load_ex": (P, [P, C.c_char_p, C.POINTER(AmLoadOptions), C.POINTER(P)]),
    "amcu_quantize_weight": (C.c_int, [C.c_int32, P, C.c_int32, C.c_int64, C.c_int64, C.c_int64, P, P, P]),
    "amcu_convert": (C.c_int, [P, C.c_int32, P, C.c_int32, C.c_int64, P]),
    "am_model_create": (P, [P, C.POINTER(AmModelConfig), C.POINTER(P)]),
    "am_model_init_synthetic": (C.c_int, [P, C.c_uint64]),
    "am_model_set_weight": (C.c_int, [P, C.c_char_p, P, P]),
    "am_model_unload": (None, [P]),
    "am_session_create": (P, [P, C.POINTER(AmSessionConfig)]),
    "am_session_destroy": (None, [P]),
    "am_session_generate": (C.c_int, [P, P, C.c_size_t, P, C.c_size_t, C.POINTER(C.c_size_t), C.POINTER(P)]),
    "am_session_generate_batch": (C.c_int, [P, P, C.c_size_t, C.c_size_t, P, C.c_size_t, C.POINTER(C.c_size_t),
                                            C.POINTER(P)]),
    "am_session_last_timing": (C.c_int, [P, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(C.c_int64)]),
    "am_session_last_gaps": (C.c_int, [P, P, C.c_size_t]),
    "am_debug_registry_size": (C.c_int64, []),
    "am_debug_plan_steps": (C.c_int, [P, C.c_int32, C.c_int64, C.c_int64, C.c_char_p, C.c_size_t]),
    "am_debug_resolve_kernel": (C.c_int, [C.c_int32] * 5 + [C.c_char_p, C.c_size_t]),
    "am_debug_kv_offset": (C.c_int, [C.c_uint64] * 4 + [C.c_int32] + [C.c_uint64] * 6 +
                           [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "am_debug_kv_reserve": (C.c_int, [C.c_uint64] * 3),
    "am_debug_tp_shard": (C.c_int, [C.c_char_p, C.c_int64, C.c_int64, C.c_int32, C.c_int32, C.POINTER(C.c_int64)]),
}

_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"aethermind_b200 CUDA library not built ({LIB_PATH}); run `python -m aethermind_b200.build`")
        l = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            f = getattr(l, name)
            f.restype = res
            f.argtypes = args
        _lib = l
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGS)


def check(code: int, what: str = "") -> None:
    if code != OK:
        msg = lib().amcu_last_error().decode()
        if not msg:
            msg = lib().am_last_error().decode()
        raise AmError(code, f"{what}: {msg}" if what else msg)
