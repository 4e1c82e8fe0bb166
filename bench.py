"""Benchmark of the Llama decode/prefill hot path on B200.

Workload (N=1): the Llama-3-8B-shaped model with INT4 group-128 weight-only
quantization and bf16 activations/KV, synthetic seeded
random-init weights, batch 1, a 512-token prompt of uniform token ids and
256 greedy decode tokens, static KV capacity 4096. One "step" is one full
greedy generation (prefill 512 + 256 decode tokens) through the engine.

  value  decode tok/s = decoded tokens / device decode time (CUDA events in
         the engine around the replayed decode graphs; prompt ids are already
         staged on the device before that region).
  e2e    generated tok/s of the public am_session_generate call, host token
         ids in and out, pinned H2D/D2H inside the timed region.
  roofline  the dominant kernel, the W4 GEMV, timed alone with CUDA events on
         the 8B shapes, weights rotated over >L2 buffers (cold HBM).
  cpu_baseline  the CPU oracle's greedy decode of the same synthetic model on
         the host cores (bounded sample, see "sample").

With --gpus N > 1 (torchrun), the model is tensor-parallel over N GPUs
(one NCCL all-reduce per attention and per MLP block); total work is fixed
("strong" scaling) and timing is the max over ranks.
--impl reference times the reference-side CPU implementation (the oracle
restatement; the reference engine itself cannot run a Llama forward) on the
same config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROMPT = 512
NEW = 256
SEED = 0
METRIC = "decode tok/s bs=1 (8B W4 g128, 512-token prompt, 256 greedy tokens)"
WORKLOAD = "llama3-8b-shape W4 g128 bs=1: prefill 512 + 256 greedy decode"


E2E_DEFINITION = ("generated tokens per second of one whole greedy generation (512-token prompt in, 256 tokens "
                  "out, host buffers): prefill + decode + copies, wall clock of the call")


def bench_config(world: int, nccl_allreduce: bool, layers: int) -> dict:
    """The workload description both arms print (same keys, same values)."""
    return {"workload": WORKLOAD, "global_batch": 1, "seq_len": PROMPT + NEW, "parallelism": f"tp{world}",
            "allreduce": "none" if world == 1 else ("nccl" if nccl_allreduce else
                                                    ("peer memory inside the o/down GEMV epilogue" if world == 2 else
                                                     "one-shot peer-memory kernel after the o/down GEMV")
                                                    + " (decode), nccl (prefill)"),
            "l2": "weights (3.9 GB) exceed L2; no flush needed", "layers": layers}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    def __init__(self, index: int = 0):
        self.index = index
        self.rows: list[list[str]] = []
        self._stop = threading.Event()
        self._t = None

    def start(self):
        def run():
            q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            while not self._stop.is_set():
                try:
                    out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                         timeout=5).stdout.strip()
                    if out:
                        self.rows.append([c.strip() for c in out.split(",")])
                except Exception:
                    pass
                self._stop.wait(0.2)
        self._t = threading.Thread(target=run, daemon=True)
        self._t.start()

    def stop(self) -> dict:
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


# (n, k) of the 8B decode GEMVs (q/k/v fused, o, gate/up interleaved, down, lm_head)
GEMV_SHAPES_8B = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (2 * 14336, 4096), "down": (4096, 14336),
                  "lm_head": (128256, 4096),
                  # the 70B-shaped model's (hidden 8192, 64 / 8 heads, intermediate 28672)
                  "70b_qkv": (10240, 8192), "70b_o": (8192, 8192), "70b_gate_up": (2 * 28672, 8192),
                  "70b_down": (8192, 28672)}


def gemv_roofline(hbm_peak: float, ncopy: int | None = None, reps: int | None = None, m: int = 1,
                  shape: str = "gate_up") -> dict:
    """Times one W4 GEMV of the 8B decode step (GEMV_SHAPES_8B; the bench's
    roofline line uses gate/up, N = 2 x 14336, K = 4096) alone for m
    activation rows, rotating over enough weight copies that every launch
    reads HBM."""
    import ctypes as C

    import torch

    from aethermind_b200 import _lib as L
    from aethermind_b200 import ops

    n, k = GEMV_SHAPES_8B[shape]
    q, s = ops.synth_w4(SEED, 99, n, k, 0.004)
    copies = []
    per = n * k // 2 + n * (k // 128) * 2
    ncopy = ncopy or max(2, int(512e6 // per) + 1)  # > 4 x L2
    for _ in range(ncopy):
        copies.append(ops.prepack(L.WFMT_INT4, q, s, n, k))
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    y = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    args = []
    for pw in copies:
        a, _, _ = ops._linear_args(x, pw, L.EPI_STORE, None, y)
        args.append(a)
    lib = L.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for a in args[:4]:
        L.check(lib.amcu_gemv_w4g128(C.byref(a), stream), "amcu_gemv_w4g128")  # a failed launch is not timed
    torch.cuda.synchronize()
    reps = reps or 20 * ncopy
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(reps):
        lib.amcu_gemv_w4g128(C.byref(args[i % ncopy]), stream)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    alg = n * k // 2 + n * (k // 128) * 2 + m * (k * 2 + n * 2)
    gbs = alg / (us * 1e-6) / 1e9
    del copies
    torch.cuda.empty_cache()
    return {"kernel": f"gemv_tc_kernel<INT4> (8B {shape}, n={n} k={k}, m={m})", "bound": "hbm",
            "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s", "frac": round(gbs / hbm_peak, 3),
            # dram__bytes_read.sum + dram__bytes_write.sum of one launch of this kernel and shape,
            # from the ncu capture summarised in profiles/gemv_w4_gate_up_8b.md
            "traffic": GEMV_GATE_UP_TRAFFIC if (shape, m) == ("gate_up", 1) else None, "alg_bytes_per_launch": alg, "us_per_launch": round(us, 2)}


GEMV_GATE_UP_TRAFFIC = 60764416


def gemm_prefill_timing(tc_peak: float, reps: int = 20) -> dict:
    """Times the tcgen05 prefill GEMM of the 8B gate/up projection, m = 512
    prompt rows (n = 2 x 14336, k = 4096, INT4 g128, SiLU-Mul epilogue)."""
    import ctypes as C

    import torch

    from aethermind_b200 import _lib as L
    from aethermind_b200 import ops

    m, inter, k = PROMPT, 14336, 4096
    gq, gs = ops.synth_w4(SEED, 98, inter, k, 0.004)
    uq, us_ = ops.synth_w4(SEED, 99, inter, k, 0.004)
    pw = ops.prepack_gate_up(L.WFMT_INT4, gq, gs, uq, us_, inter, k)
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    y = torch.empty(m, inter, device="cuda", dtype=torch.bfloat16)
    a, _, ws = ops._linear_args(x, pw, L.EPI_SILU_MUL, None, y)  # ws: the tail split-K workspace, kept alive
    lib = L.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(3):
        L.check(lib.amcu_gemm_w4g128_prefill(C.byref(a), stream), "amcu_gemm_w4g128_prefill")
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        lib.amcu_gemm_w4g128_prefill(C.byref(a), stream)
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / reps
    del ws
    tflops = 2.0 * m * 2 * inter * k / (us * 1e-6) / 1e12
    return {"kernel": "gemm_w4_swap_kernel<SILU_MUL> (8B gate_up, m=512 n=28672 k=4096)", "bound": "tensor",
            "achieved": round(tflops, 1), "peak": tc_peak, "unit": "TFLOP/s", "frac": round(tflops / tc_peak, 3),
            "us_per_launch": round(us, 2)}


def op_bench(args) -> None:
    """Single-kernel timing for the profiles (one GPU): --op gemv_gate_up | gemm_gate_up."""
    import torch
    torch.cuda.set_device(0)
    hbm_peak, tc_peak, _ = _peaks()
    if args.op.startswith("gemv_") and args.op[5:] in GEMV_SHAPES_8B:
        r = gemv_roofline(hbm_peak, ncopy=args.copies, reps=args.reps, m=args.m, shape=args.op[5:])
    elif args.op == "gemm_gate_up":
        r = gemm_prefill_timing(tc_peak, reps=args.reps or 20)
    else:
        raise SystemExit(f"unknown --op {args.op}")
    print(json.dumps({"op": args.op, **r}), flush=True)


def decode_bytes_per_token(cfg, ctx: float, batch: int = 1) -> float:
    """HBM bytes of one decode step: every linear weight and its scales once
    (lm_head included; a tied lm_head counted once, as INT8 rows) plus each
    sequence's KV cache up to ctx."""
    from aethermind_b200 import _lib as L
    H, I, d = cfg.hidden, cfg.inter, cfg.head_dim
    qkv = (cfg.n_q_heads + 2 * cfg.n_kv_heads) * d
    per_layer = H * qkv + cfg.n_q_heads * d * H + 2 * I * H + I * H
    rows = cfg.layers * (qkv + H + 2 * I + H) + cfg.vocab
    params = cfg.layers * per_layer + cfg.vocab * H
    if cfg.weight_format == L.WFMT_INT8:
        w = params + rows * 4
    else:
        w = params / 2 + params / 128 * 2
    kv = cfg.layers * 2 * cfg.n_kv_heads * d * 2 * ctx * batch
    return w + kv


def timed_generate(sess, prompt, new: int, dist) -> tuple[float, float]:
    """One generate call; (prefill ms, decode ms) on the device, max over ranks."""
    import torch
    sess.generate(prompt, new)
    p, d, _ = sess.timing()
    if dist:
        t = torch.tensor([p, d], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        p, d = t.tolist()
    return p, d


def extra_configs(sess, model_cfg, rt, world: int, dist, hbm_peak: float, tc_peak: float) -> dict:
    """The other BASELINE workloads, one timed generate each after a short
    warm-up: the 8B model at batch 8, the 1B W8 model (one GPU: replicas
    only) and the 70B W4 model (tensor parallel over all ranks)."""
    import dataclasses

    import numpy as np

    from aethermind_b200 import session
    out = {}
    rng = np.random.default_rng(SEED + 1)
    # 8B W4, batch 8, 512-token prompts, 256 tokens
    p8 = rng.integers(0, model_cfg.vocab, (8, PROMPT)).astype(np.uint32)
    sess.generate(p8, 4)
    pre, dec = timed_generate(sess, p8, NEW, dist)
    bpt = decode_bytes_per_token(model_cfg, PROMPT + NEW / 2, 8) / world
    out["8b_w4_bs8"] = {"decode_tok_s": round(8 * (NEW - 1) / (dec / 1e3), 1),
                        "prefill_tok_s": round(8 * PROMPT / (pre / 1e3), 1),
                        "decode_hbm_frac_per_gpu": round(bpt * (NEW - 1) / (dec / 1e3) / 1e9 / hbm_peak, 3)}
    # 1B W8 (tied embeddings), 128-token prompt, 128 tokens, one GPU
    if world == 1:
        c1 = dataclasses.replace(session.LLAMA_1B_W8, max_seq=2048)
        m1 = session.Model(rt, c1)
        m1.init_synthetic(SEED)
        s1 = session.Session(m1)
        pr = rng.integers(0, c1.vocab, 128).astype(np.uint32)
        s1.generate(pr, 4)
        pre, dec = timed_generate(s1, pr, 128, None)
        bpt = decode_bytes_per_token(c1, 128 + 64)
        out["1b_w8"] = {"decode_tok_s": round(127 / (dec / 1e3), 1), "prefill_tok_s": round(128 / (pre / 1e3), 1),
                        "decode_hbm_frac": round(bpt * 127 / (dec / 1e3) / 1e9 / hbm_peak, 3)}
        del s1, m1
    # 70B W4, 2048-token prompt, 256 tokens, TP over all ranks
    c7 = dataclasses.replace(session.LLAMA_70B_W4, max_seq=4096)
    m7 = session.Model(rt, c7)
    m7.init_synthetic(SEED)
    s7 = session.Session(m7)
    pr = rng.integers(0, c7.vocab, 2048).astype(np.uint32)
    s7.generate(pr[:64], 4)
    pre, dec = timed_generate(s7, pr, NEW, dist)
    bpt = decode_bytes_per_token(c7, 2048 + NEW / 2) / world
    out["70b_w4"] = {"decode_tok_s": round((NEW - 1) / (dec / 1e3), 2), "prefill_tok_s": round(2048 / (pre / 1e3), 1),
                     "decode_hbm_frac_per_gpu": round(bpt * (NEW - 1) / (dec / 1e3) / 1e9 / hbm_peak, 3),
                     "tp": world}
    del s7, m7
    return out


def cpu_oracle_model(cfg):
    import oracle
    return oracle.synthetic_oracle_model(cfg, SEED)


def cpu_oracle_decode(om, cfg, prompt_len: int, new: int) -> dict:
    """Greedy decode of the synthetic model by the CPU oracle; returns tok/s of
    the decode phase (all host threads via OpenMP)."""
    import numpy as np

    prompt = np.random.default_rng(SEED).integers(0, cfg.vocab, prompt_len).astype(np.int64)
    om.generate(prompt, 1 + new)
    t_prefill, t_decode = om.last_timing()
    return {"tok_s": new / max(t_decode, 1e-9), "prefill_s": t_prefill, "cores": os.cpu_count()}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from aethermind_b200.session import LLAMA_8B_W4
    import dataclasses
    cfg = dataclasses.replace(LLAMA_8B_W4, max_seq=PROMPT + NEW)
    om = cpu_oracle_model(cfg)
    steps = []
    for _ in range(args.warmup + args.steps):
        steps.append(cpu_oracle_decode(om, cfg, 8, 2))
    timed = steps[args.warmup:]
    v = statistics.mean(s["tok_s"] for s in timed)
    # whole-call rate of the full workload, extrapolated from the sample's
    # per-token prefill and decode times (the CPU needs minutes for one real call)
    pre_tok_s = statistics.mean(s["prefill_s"] for s in timed) / 8
    dec_tok_s = statistics.mean(2 / s["tok_s"] for s in timed) / 2
    e2e = NEW / (PROMPT * pre_tok_s + (NEW - 1) * dec_tok_s)
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * 2 / v, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded integer-hash INT4 weights, uniform token ids)",
            # the GPU arm's config (the timed CPU work is a bounded sample of it, see cpu_baseline.sample)
            "config": bench_config(args.gpus, False, cfg.layers),
            "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": "per step: 8-token prompt prefill + 2 greedy decode tokens of the full 32-layer "
                                       "8B W4 model; decode tok/s (CPU restatement in oracle/am_oracle.c, OpenMP)"},
            "e2e": {"value": round(e2e, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "e2e_definition": E2E_DEFINITION + "; CPU: extrapolated from the sample's per-token prefill "
                              f"({pre_tok_s:.3f} s) and decode ({dec_tok_s:.3f} s) times"}
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="aethermind_b200")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-roofline", action="store_true")
    ap.add_argument("--layers", type=int, default=None, help="debug: fewer layers (invalidates the number)")
    ap.add_argument("--no-extra", action="store_true", help="skip the other BASELINE workloads (bs=8, 1B W8, 70B W4)")
    ap.add_argument("--decode", default="per-op", choices=["per-op", "persistent"],
                    help="decode plan: one kernel per op, or the persistent all-layers kernel (batch 1)")
    ap.add_argument("--nccl-allreduce", action="store_true", help="TP: NCCL for every all-reduce (no peer-memory one-shot)")
    ap.add_argument("--op", default=None,
                    help="time one kernel instead: gemv_<shape> (qkv, o, gate_up, down, lm_head, 70b_qkv, 70b_o, "
                         "70b_gate_up, 70b_down) | gemm_gate_up")
    ap.add_argument("--copies", type=int, default=None, help="--op gemv_*: weight copies rotated")
    ap.add_argument("--m", type=int, default=1, help="--op gemv_*: activation rows")
    ap.add_argument("--reps", type=int, default=None, help="--op: timed launches")
    args = ap.parse_args()
    if args.op:
        op_bench(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    import dataclasses

    import numpy as np
    import torch

    from aethermind_b200 import session

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    nccl_id = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        obj = [session.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nccl_id = obj[0]

    cfg = dataclasses.replace(session.LLAMA_8B_W4, max_seq=4096, max_batch=8)
    if args.layers:
        cfg = dataclasses.replace(cfg, layers=args.layers)
    rt = session.Runtime(local, rank, world, nccl_id)
    peer_error = None
    if world > 1 and not args.nccl_allreduce:
        # decode all-reduces over peer memory: share the ranks' CUDA IPC handles
        # (every rank must agree: any failure keeps all ranks on NCCL)
        try:
            mine = rt.peer_handle()
        except Exception as e:  # pragma: no cover - depends on the box
            mine, peer_error = None, f"peer_handle: {e}"
        handles = [None] * world
        dist.all_gather_object(handles, mine)
        if all(h is not None for h in handles):
            try:
                rt.open_peers(handles)
                ok = 1
            except Exception as e:  # pragma: no cover
                ok, peer_error = 0, f"open_peers: {e}"
            flags = [None] * world
            dist.all_gather_object(flags, ok)
            if not all(flags):
                raise SystemExit(f"rank {rank}: peer all-reduce setup failed on a rank ({peer_error}); "
                                 "rerun with --nccl-allreduce")
        else:
            args.nccl_allreduce = True
    model = session.Model(rt, cfg)
    model.init_synthetic(SEED)
    sess = session.Session(model, persistent_decode=args.decode == "persistent")
    prompt = np.random.default_rng(SEED).integers(0, cfg.vocab, PROMPT).astype(np.uint32)

    for _ in range(args.warmup):
        sess.generate(prompt, NEW)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    dec_ms, pre_ms, wall = [], [], []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        toks = sess.generate(prompt, NEW)
        wall.append(time.perf_counter() - t0)
        p, d, n = sess.timing()
        pre_ms.append(p)
        dec_ms.append(d)
    torch.cuda.synchronize()
    ck = clocks.stop()
    if dist:
        dist.barrier()
        t = torch.tensor([sum(dec_ms), sum(pre_ms), sum(wall)], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dec_total, pre_total, wall_total = t.tolist()
    else:
        dec_total, pre_total, wall_total = sum(dec_ms), sum(pre_ms), sum(wall)

    decoded = args.steps * (NEW - 1)
    value = decoded / (dec_total / 1e3)
    hbm_peak, tc_peak, peak_kind = _peaks()
    ctx_mean = PROMPT + NEW / 2
    bpt = decode_bytes_per_token(cfg, ctx_mean) / world
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round((dec_total + pre_total) / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded integer-hash INT4 weights, uniform token ids)",
        "config": bench_config(world, args.nccl_allreduce, cfg.layers),
        "prefill_tok_s": round(args.steps * PROMPT / (pre_total / 1e3), 1),
        "decode_ms_per_token": round(dec_total / decoded, 4),
        "decode_hbm_gbs_per_gpu": round(bpt * value / 1e9, 1),
        "decode_hbm_frac_per_gpu": round(bpt * value / 1e9 / hbm_peak, 3),
        "peaks": {"hbm_gbs": hbm_peak, "bf16_tflops": tc_peak, "kind": peak_kind},
        "clocks": ck,
        "e2e": {"value": round(args.steps * NEW / wall_total, 2),
                "unit": "tok/s", "h2d_bytes_per_step": PROMPT * 8, "d2h_bytes_per_step": NEW * 12 + 8},
        "e2e_definition": E2E_DEFINITION + " (am_session_generate)",
        "gpu_launches": None,
    }
    # kernel launches of this library in the timed region (from the plans): one
    # per kernel step, plus the split-K combine of an unfused decode attention,
    # the second pass of the two-phase argmax, and the decode-state advance
    try:
        dec_steps = sess.plan_steps(1, 1, 1)
        pre_steps = sess.plan_steps(0, 1, PROMPT)
        def launches(steps):
            n = sum(1 for l in steps if "<host>" not in l)
            n += sum(1 for l in steps if "AttnDecodeSplitK" in l)
            n += sum(1 for l in steps if l.split()[0] == "argmax")
            return n + 1
        line["gpu_launches"] = args.steps * (launches(pre_steps) + (NEW - 1) * launches(dec_steps))
    except Exception as e:  # pragma: no cover
        line["gpu_launches_error"] = str(e)
    if peer_error:
        line["allreduce_note"] = peer_error
    if not args.no_extra:
        try:
            line["configs"] = extra_configs(sess, cfg, rt, world, dist, hbm_peak, tc_peak)
        except Exception as e:  # pragma: no cover - reported, the headline line stands
            line["configs_error"] = f"{type(e).__name__}: {e}"
    if rank == 0 and world == 1 and not args.no_roofline:
        del sess, model
        torch.cuda.empty_cache()
        line["roofline"] = gemv_roofline(hbm_peak)
        line["roofline"]["peak_kind"] = f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
        line["prefill_roofline"] = gemm_prefill_timing(tc_peak)
        line["prefill_roofline"]["peak_kind"] = f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops, burst)"
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ccfg = dataclasses.replace(cfg, max_seq=64)
        cb = cpu_oracle_decode(cpu_oracle_model(ccfg), ccfg, 8, 2)
        line["cpu_baseline"] = {"value": round(cb["tok_s"], 4), "unit": "tok/s", "cores": cb["cores"], "kind": "port",
                                "sample": "8-token prompt + 2 greedy decode tokens of the same 32-layer 8B W4 "
                                          "synthetic model (oracle/am_oracle.c, OpenMP on all host threads)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
