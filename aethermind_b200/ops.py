"""Torch-tensor front end of the amcu_* kernel launchers.

Every function here calls the CUDA C ABI on the current torch stream; tensors
must already be on a CUDA device. These are the host-side mirror of the
reference's SDK launchers (LaunchRmsNorm / LaunchAdd style: plain pointers,
shapes, strides and a status code, include/aethermind/backend/cpu/kernels/
rmsnorm/cpu_rmsnorm_kernel.h:13-53), used by the tests and by users who drive
single ops; the engine itself calls the same entry points from C++.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib as L
from ._lib import check, lib

_DT = {torch.float32: L.F32, torch.bfloat16: L.BF16, torch.int32: L.I32, torch.int64: L.I64}


def _dt(t: torch.Tensor) -> int:
    return _DT[t.dtype]


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("aethermind_b200 ops take CUDA tensors")


# ------------------------------------------------------------------ weights
@dataclass
class PackedWeight:
    """A weight in the device (tile16x64) format plus its AmcuWeight descriptor."""

    fmt: int
    n: int
    k: int
    dtype: int = L.BF16
    group: int = 128
    data: torch.Tensor | None = None
    scales: torch.Tensor | None = None
    gate_up: bool = False
    desc: L.AmcuWeight = field(default_factory=L.AmcuWeight)

    def __post_init__(self):
        self.desc.format = self.fmt
        self.desc.dtype = self.dtype
        self.desc.n = self.n
        self.desc.k = self.k
        self.desc.group = self.group
        self.desc.data = _p(self.data)
        self.desc.scales = _p(self.scales)
        self.desc.gate_up_interleaved = int(self.gate_up)


def _alloc_packed(fmt: int, dtype: int, n: int, k: int, group: int, device) -> tuple[torch.Tensor, torch.Tensor | None]:
    wb = lib().amcu_packed_weight_bytes(fmt, dtype, n, k, group)
    sb = lib().amcu_packed_scale_bytes(fmt, n, k, group)
    q = torch.empty(wb, dtype=torch.uint8, device=device)
    s = torch.empty(max(sb, 1), dtype=torch.uint8, device=device) if sb > 0 else None
    return q, s


def prepack(fmt: int, q: torch.Tensor, s: torch.Tensor | None, n: int, k: int, group: int = 128,
            dtype: int = L.BF16) -> PackedWeight:
    """Canonical (device) weight -> device format (amcu_prepack_weight)."""
    _require_cuda(q, s)
    qp, sp = _alloc_packed(fmt, dtype, n, k, group, q.device)
    check(lib().amcu_prepack_weight(fmt, dtype, n, k, group, _p(q), _p(s), _p(qp), _p(sp), _stream()),
          "amcu_prepack_weight")
    return PackedWeight(fmt, n, k, dtype, group, qp, sp)


def prepack_gate_up(fmt: int, gq, gs, uq, us, inter: int, k: int, group: int = 128,
                    dtype: int = L.BF16) -> PackedWeight:
    _require_cuda(gq, uq)
    qp, sp = _alloc_packed(fmt, dtype, 2 * inter, k, group, gq.device)
    check(lib().amcu_prepack_gate_up(fmt, dtype, inter, k, group, _p(gq), _p(gs), _p(uq), _p(us), _p(qp), _p(sp),
                                     _stream()), "amcu_prepack_gate_up")
    return PackedWeight(fmt, 2 * inter, k, dtype, group, qp, sp, gate_up=True)


def unpack(pw: PackedWeight) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Device format -> canonical bytes (amcu_unpack_weight)."""
    dev = pw.data.device
    if pw.fmt == L.WFMT_INT4:
        q = torch.empty(pw.n, pw.k // 2, dtype=torch.uint8, device=dev)
        s = torch.empty(pw.n, pw.k // pw.group, dtype=torch.float16, device=dev)
    elif pw.fmt == L.WFMT_INT8:
        q = torch.empty(pw.n, pw.k, dtype=torch.int8, device=dev)
        s = torch.empty(pw.n, dtype=torch.float32, device=dev)
    else:
        q = torch.empty(pw.n, pw.k, dtype=torch.float32 if pw.dtype == L.F32 else torch.bfloat16, device=dev)
        s = None
    check(lib().amcu_unpack_weight(pw.fmt, pw.dtype, pw.n, pw.k, pw.group, _p(pw.data), _p(pw.scales), _p(q),
                                   _p(s), _stream()), "amcu_unpack_weight")
    return q, s


def synth_w4(seed: int, stream_id: int, n: int, k: int, base: float, device="cuda"):
    q = torch.empty(n, k // 2, dtype=torch.uint8, device=device)
    s = torch.empty(n, k // 128, dtype=torch.float16, device=device)
    check(lib().amcu_synth_w4(seed, stream_id, n, k, base, _p(q), _p(s), _stream()), "amcu_synth_w4")
    return q, s


def synth_w8(seed: int, stream_id: int, n: int, k: int, base: float, device="cuda"):
    q = torch.empty(n, k, dtype=torch.int8, device=device)
    s = torch.empty(n, dtype=torch.float32, device=device)
    check(lib().amcu_synth_w8(seed, stream_id, n, k, base, _p(q), _p(s), _stream()), "amcu_synth_w8")
    return q, s


def synth_uniform_bf16(seed: int, stream_id: int, count: int, amplitude: float, device="cuda"):
    out = torch.empty(count, dtype=torch.bfloat16, device=device)
    check(lib().amcu_synth_uniform_bf16(seed, stream_id, count, amplitude, _p(out), _stream()),
          "amcu_synth_uniform_bf16")
    return out


# ------------------------------------------------------------------ ops
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-5, residual: torch.Tensor | None = None,
            out: torch.Tensor | None = None, residual_out: torch.Tensor | None = None):
    """RMSNorm over the last axis; with `residual`, h = x + residual first.

    Returns y, or (y, h) when a residual is given."""
    _require_cuda(x, w, residual)
    rows, hidden = (x.shape[0], x.shape[1]) if x.dim() == 2 else (1, x.shape[0])
    y = out if out is not None else torch.empty(rows, hidden, dtype=x.dtype, device=x.device)
    a = L.AmcuRmsNormArgs()
    a.input, a.weight, a.output = _p(x), _p(w), _p(y)
    a.rows, a.hidden = rows, hidden
    a.input_row_stride = x.stride(0) if x.dim() == 2 else hidden
    a.output_row_stride = y.stride(0)
    a.eps = eps
    a.dtype = _dt(x)
    h = None
    if residual is not None:
        h = residual_out if residual_out is not None else torch.empty_like(y)
        a.residual, a.residual_out = _p(residual), _p(h)
    check(lib().amcu_rmsnorm(C.byref(a), _stream()), "amcu_rmsnorm")
    return y if residual is None else (y, h)


def _linear_args(x: torch.Tensor, pw: PackedWeight, epilogue: int, residual, out):
    m = x.shape[0]
    n_out = pw.n // 2 if epilogue == L.EPI_SILU_MUL else pw.n
    y = out if out is not None else torch.empty(m, n_out, dtype=x.dtype, device=x.device)
    a = L.AmcuLinearArgs()
    a.x, a.w, a.y = _p(x), pw.desc, _p(y)
    a.residual = _p(residual)
    a.m = m
    a.x_stride = x.stride(0)
    a.y_stride = y.stride(0)
    a.act_dtype = _dt(x)
    a.epilogue = epilogue
    ws_bytes = lib().amcu_linear_workspace_bytes(C.byref(a))
    ws = None
    if ws_bytes:
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        a.workspace, a.workspace_size = _p(ws), ws_bytes
    return a, y, ws


def linear(x: torch.Tensor, pw: PackedWeight, epilogue: int = L.EPI_STORE, residual: torch.Tensor | None = None,
           out: torch.Tensor | None = None, entry: str = "amcu_linear", norm_weight: torch.Tensor | None = None,
           norm_eps: float = 1e-5) -> torch.Tensor:
    """y = x @ W^T with the chosen epilogue, through `entry` (amcu_linear by
    default); with norm_weight, x is RMS-normalized first (fused, decode GEMV)."""
    _require_cuda(x, residual, norm_weight)
    a, y, ws = _linear_args(x, pw, epilogue, residual, out)
    if norm_weight is not None:
        a.norm_weight, a.norm_eps = _p(norm_weight), norm_eps
    check(getattr(lib(), entry)(C.byref(a), _stream()), entry)
    del ws
    return y


def rope_kv_write(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                  seq_pos: torch.Tensor, rows_per_seq: int, n_q: int, n_kv: int, head_dim: int, theta: float,
                  status: torch.Tensor | None = None) -> None:
    """Rotates q in place; writes rotated k and v into cache[slot, kv_head, pos]."""
    _require_cuda(q, k, v, k_cache, v_cache, seq_pos)
    a = L.AmcuRopeKvArgs()
    a.q, a.k, a.v = _p(q), _p(k), _p(v)
    a.q_stride, a.k_stride, a.v_stride = q.stride(0), k.stride(0), v.stride(0)
    a.k_cache, a.v_cache = _p(k_cache), _p(v_cache)
    a.slot_stride = k_cache.stride(0)
    a.capacity = k_cache.shape[2]
    a.seq_pos = _p(seq_pos)
    a.rows, a.rows_per_seq = q.shape[0], rows_per_seq
    a.n_q_heads, a.n_kv_heads, a.head_dim = n_q, n_kv, head_dim
    a.theta = theta
    a.dtype = _dt(q)
    a.status = _p(status)
    check(lib().amcu_rope_kv_write(C.byref(a), _stream()), "amcu_rope_kv_write")


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, seq_pos: torch.Tensor,
              rows_per_seq: int, n_q: int, n_kv: int, head_dim: int, max_context: int | None = None,
              num_splits: int = 0, decode: bool | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal GQA attention over cache [slots, n_kv, capacity, head_dim]."""
    _require_cuda(q, k_cache, v_cache, seq_pos)
    rows = q.shape[0]
    o = out if out is not None else torch.empty(rows, n_q * head_dim, dtype=q.dtype, device=q.device)
    a = L.AmcuAttentionArgs()
    a.q, a.q_stride = _p(q), q.stride(0)
    a.k_cache, a.v_cache = _p(k_cache), _p(v_cache)
    a.slot_stride, a.capacity = k_cache.stride(0), k_cache.shape[2]
    a.seq_pos = _p(seq_pos)
    a.out, a.out_stride = _p(o), o.stride(0)
    a.rows, a.rows_per_seq = rows, rows_per_seq
    a.n_q_heads, a.n_kv_heads, a.head_dim = n_q, n_kv, head_dim
    a.dtype = _dt(q)
    a.num_splits = num_splits
    a.max_context = max_context if max_context is not None else k_cache.shape[2]
    if decode is None:
        decode = rows_per_seq == 1
    ws = None
    if decode:
        nb = lib().amcu_attention_workspace_bytes(C.byref(a))
        if nb:
            ws = torch.empty(nb, dtype=torch.uint8, device=q.device)
            a.workspace, a.workspace_size = _p(ws), nb
        check(lib().amcu_attn_decode(C.byref(a), _stream()), "amcu_attn_decode")
    else:
        check(lib().amcu_attn_prefill(C.byref(a), _stream()), "amcu_attn_prefill")
    del ws
    return o


def attention_rope_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, k_cache: torch.Tensor,
                          v_cache: torch.Tensor, seq_pos: torch.Tensor, n_q: int, n_kv: int, head_dim: int,
                          theta: float, cos_sin: torch.Tensor | None = None, status: torch.Tensor | None = None,
                          out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused decode step (amcu_attn_decode_rope): RoPE, KV-cache append and
    attention for one row per sequence. q is not modified."""
    _require_cuda(q, k, v, k_cache, v_cache, seq_pos)
    o = out if out is not None else torch.empty(q.shape[0], n_q * head_dim, dtype=q.dtype, device=q.device)
    r, a = _rope_attn_args(q, k, v, k_cache, v_cache, seq_pos, n_q, n_kv, head_dim, theta, cos_sin, status, o)
    check(lib().amcu_attn_decode_rope(C.byref(r), C.byref(a), _stream()), "amcu_attn_decode_rope")
    return o


def _rope_attn_args(q, k, v, k_cache, v_cache, seq_pos, n_q, n_kv, head_dim, theta, cos_sin, status, o):
    rows = q.shape[0]
    r = L.AmcuRopeKvArgs()
    r.q, r.k, r.v = _p(q), _p(k), _p(v)
    r.q_stride, r.k_stride, r.v_stride = q.stride(0), k.stride(0), v.stride(0)
    r.k_cache, r.v_cache = _p(k_cache), _p(v_cache)
    r.slot_stride, r.capacity = k_cache.stride(0), k_cache.shape[2]
    r.seq_pos = _p(seq_pos)
    r.rows, r.rows_per_seq = rows, 1
    r.n_q_heads, r.n_kv_heads, r.head_dim = n_q, n_kv, head_dim
    r.theta = theta
    r.dtype = _dt(q)
    r.status = _p(status)
    r.cos_sin = _p(cos_sin)
    a = L.AmcuAttentionArgs()
    a.q, a.q_stride = _p(q), q.stride(0)
    a.k_cache, a.v_cache = _p(k_cache), _p(v_cache)
    a.slot_stride, a.capacity = k_cache.stride(0), k_cache.shape[2]
    a.seq_pos = _p(seq_pos)
    a.out, a.out_stride = _p(o), o.stride(0)
    a.rows, a.rows_per_seq = rows, 1
    a.n_q_heads, a.n_kv_heads, a.head_dim = n_q, n_kv, head_dim
    a.dtype = _dt(q)
    a.max_context = k_cache.shape[2]
    return r, a


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _require_cuda(gate, up)
    y = out if out is not None else torch.empty_like(gate)
    check(lib().amcu_silu_mul(_p(gate), _p(up), _p(y), gate.numel(), _dt(gate), _stream()), "amcu_silu_mul")
    return y


def add(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _require_cuda(a, b)
    y = out if out is not None else torch.empty_like(a)
    check(lib().amcu_add(_p(a), _p(b), _p(y), a.numel(), _dt(a), _stream()), "amcu_add")
    return y


def argmax(logits: torch.Tensor, with_gap: bool = False):
    _require_cuda(logits)
    rows, vocab = logits.shape
    idx = torch.empty(rows, dtype=torch.int64, device=logits.device)
    gap = torch.empty(rows, dtype=torch.float32, device=logits.device) if with_gap else None
    check(lib().amcu_argmax(_p(logits), rows, vocab, logits.stride(0), _dt(logits), _p(idx), _p(gap), _stream()),
          "amcu_argmax")
    return (idx, gap) if with_gap else idx


def embedding(ids: torch.Tensor, table: torch.Tensor, row_scales: torch.Tensor | None = None,
              out_dtype: torch.dtype | None = None, status: torch.Tensor | None = None) -> torch.Tensor:
    _require_cuda(ids, table, row_scales)
    vocab, hidden = table.shape
    dt = out_dtype or (torch.bfloat16 if row_scales is not None else table.dtype)
    out = torch.empty(ids.numel(), hidden, dtype=dt, device=ids.device)
    a = L.AmcuEmbeddingArgs()
    a.ids = _p(ids)
    a.id_dtype = {torch.int32: L.I32, torch.int64: L.I64}.get(ids.dtype, L.U32)
    a.count = ids.numel()
    a.table, a.row_scales = _p(table), _p(row_scales)
    a.vocab, a.hidden = vocab, hidden
    a.out, a.dtype = _p(out), _DT[dt]
    a.status = _p(status)
    check(lib().amcu_embedding(C.byref(a), _stream()), "amcu_embedding")
    return out
