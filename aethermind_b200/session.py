"""Python front end of the am_* session ABI (runtime -> model -> session -> generate).

Mirrors the reference product spec's C API (docs/products/aethermind_prd.md:
296-320): host token ids in, host token ids out.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from ._lib import AmError, lib


@dataclass
class ModelConfig:
    vocab: int
    hidden: int
    layers: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    inter: int
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    tied_embeddings: bool = False
    act_dtype: int = L.BF16
    weight_format: int = L.WFMT_INT4
    group_size: int = 128
    max_seq: int = 2048
    max_batch: int = 1

    def to_c(self) -> L.AmModelConfig:
        c = L.AmModelConfig()
        for f in ("vocab", "hidden", "layers", "n_q_heads", "n_kv_heads", "head_dim", "inter", "rms_eps",
                  "rope_theta", "act_dtype", "weight_format", "group_size", "max_seq", "max_batch"):
            setattr(c, f, getattr(self, f))
        c.tied_embeddings = int(self.tied_embeddings)
        return c


# The BASELINE configurations (shapes; synthetic random-init weights).
TINY_F32 = ModelConfig(vocab=512, hidden=256, layers=2, n_q_heads=4, n_kv_heads=2, head_dim=64, inter=688,
                       rms_eps=1e-5, rope_theta=10000.0, act_dtype=L.F32, weight_format=L.WFMT_PLAIN, max_seq=128)
LLAMA_1B_W8 = ModelConfig(vocab=128256, hidden=2048, layers=16, n_q_heads=32, n_kv_heads=8, head_dim=64,
                          inter=8192, rope_theta=500000.0, tied_embeddings=True, weight_format=L.WFMT_INT8,
                          max_seq=2048)
LLAMA_8B_W4 = ModelConfig(vocab=128256, hidden=4096, layers=32, n_q_heads=32, n_kv_heads=8, head_dim=128,
                          inter=14336, rope_theta=500000.0, weight_format=L.WFMT_INT4, max_seq=4096)
LLAMA_70B_W4 = ModelConfig(vocab=128256, hidden=8192, layers=80, n_q_heads=64, n_kv_heads=8, head_dim=128,
                           inter=28672, rope_theta=500000.0, weight_format=L.WFMT_INT4, max_seq=4096)


def _err(msg: str = "") -> AmError:
    return AmError(13, f"{msg}: {lib().am_last_error().decode()}")


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    L.check(lib().am_nccl_get_unique_id(buf), "am_nccl_get_unique_id")
    return buf.raw


class Runtime:
    def __init__(self, device_id: int = 0, tp_rank: int = 0, tp_size: int = 1, nccl_id: bytes | None = None):
        cfg = L.AmConfig()
        cfg.device_id, cfg.tp_rank, cfg.tp_size = device_id, tp_rank, tp_size
        self._id = C.create_string_buffer(nccl_id, 128) if nccl_id else None
        cfg.nccl_unique_id = C.cast(self._id, C.c_void_p) if self._id is not None else None
        h = lib().am_runtime_create(C.byref(cfg))
        if not h:
            raise _err("am_runtime_create")
        self.h = h
        self.tp_rank, self.tp_size = tp_rank, tp_size

    def peer_handle(self) -> bytes:
        """This rank's 64-byte CUDA IPC handle of its all-reduce exchange area."""
        buf = C.create_string_buffer(64)
        L.check(lib().am_runtime_peer_handle(self.h, buf), "am_runtime_peer_handle")
        return buf.raw

    def open_peers(self, handles: list[bytes]) -> None:
        """Opens every rank's exchange area (handles in rank order): decode steps
        of sessions created afterwards all-reduce over peer memory."""
        blob = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        L.check(lib().am_runtime_open_peers(self.h, blob), "am_runtime_open_peers")

    def close(self):
        if getattr(self, "h", None):
            lib().am_runtime_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: module globals already cleared
            pass


class Model:
    def __init__(self, rt: Runtime, cfg: ModelConfig):
        self.rt, self.cfg = rt, cfg
        self._c = cfg.to_c()
        err = C.c_void_p()
        h = lib().am_model_create(rt.h, C.byref(self._c), C.byref(err))
        if not h:
            code = lib().am_error_code(err) if err.value else 13
            msg = lib().am_error_message(err).decode() if err.value else ""
            if err.value:
                lib().am_error_destroy(err)
            raise AmError(code, f"am_model_create: {msg}")
        self.h = h

    @classmethod
    def load(cls, rt: Runtime, path: str, weight_format: int = L.WFMT_INT4, act_dtype: int = L.BF16,
             max_seq: int = 0, max_batch: int = 0) -> "Model":
        """A model from a Hugging Face Llama checkpoint directory (config.json +
        safetensors), quantized on the device at load time (am_model_load_ex)."""
        o = L.AmLoadOptions()
        o.weight_format, o.act_dtype, o.max_seq, o.max_batch = weight_format, act_dtype, max_seq, max_batch
        err = C.c_void_p()
        h = lib().am_model_load_ex(rt.h, str(path).encode(), C.byref(o), C.byref(err))
        if not h:
            code = lib().am_error_code(err) if err.value else 13
            msg = lib().am_error_message(err).decode() if err.value else ""
            if err.value:
                lib().am_error_destroy(err)
            raise AmError(code, f"am_model_load: {msg}")
        self = cls.__new__(cls)
        self.rt, self.cfg, self._c, self.h = rt, None, None, h
        return self

    def init_synthetic(self, seed: int = 0) -> None:
        L.check(lib().am_model_init_synthetic(self.h, seed), "am_model_init_synthetic")

    def set_weight(self, name: str, data: np.ndarray, scales: np.ndarray | None = None) -> None:
        data = np.ascontiguousarray(data)
        sp = None
        if scales is not None:
            scales = np.ascontiguousarray(scales)
            sp = scales.ctypes.data
        L.check(lib().am_model_set_weight(self.h, name.encode(), data.ctypes.data, sp), f"set_weight({name})")

    def close(self):
        if getattr(self, "h", None):
            lib().am_model_unload(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: module globals already cleared
            pass


class Session:
    def __init__(self, model: Model, max_new_tokens: int = 0, use_cuda_graph: bool = True,
                 fused_attention: bool = True, persistent_decode: bool = False):
        self.model = model
        c = L.AmSessionConfig()
        c.max_new_tokens, c.use_cuda_graph = max_new_tokens, int(use_cuda_graph)
        c.unfused_attention = 0 if fused_attention else 1
        c.persistent_decode = 1 if persistent_decode else 0
        h = lib().am_session_create(model.h, C.byref(c))
        if not h:
            raise _err("am_session_create")
        self.h = h

    def generate(self, prompt, max_new: int) -> np.ndarray:
        """Greedy generation. prompt: 1-D (one sequence) or 2-D [batch, len] token ids."""
        p = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        batch = 1 if p.ndim == 1 else p.shape[0]
        plen = p.shape[-1]
        out = np.zeros((batch, max_new), dtype=np.uint32)
        n = C.c_size_t(0)
        err = C.c_void_p()
        code = lib().am_session_generate_batch(self.h, p.ctypes.data, batch, plen, out.ctypes.data, max_new,
                                               C.byref(n), C.byref(err))
        if code != 0:
            msg = lib().am_error_message(err).decode() if err.value else ""
            if err.value:
                lib().am_error_destroy(err)
            raise AmError(code, f"am_session_generate: {msg}")
        out = out[:, : n.value]
        return out[0] if p.ndim == 1 else out

    def timing(self) -> tuple[float, float, int]:
        pf, dc, st = C.c_double(), C.c_double(), C.c_int64()
        L.check(lib().am_session_last_timing(self.h, C.byref(pf), C.byref(dc), C.byref(st)))
        return pf.value, dc.value, st.value

    def gaps(self, count: int) -> np.ndarray:
        g = np.zeros(count, dtype=np.float32)
        L.check(lib().am_session_last_gaps(self.h, g.ctypes.data, count))
        return g

    def plan_steps(self, phase: int, batch: int, rows_per_seq: int) -> list[str]:
        buf = C.create_string_buffer(1 << 20)
        L.check(lib().am_debug_plan_steps(self.h, phase, batch, rows_per_seq, buf, len(buf)))
        return [l for l in buf.value.decode().splitlines() if l]

    def close(self):
        if getattr(self, "h", None):
            lib().am_session_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except TypeError:  # interpreter shutdown: module globals already cleared
            pass
