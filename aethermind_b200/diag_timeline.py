"""Per-launch timeline of the decode step, from a diagnostics build.

A library built with ``-DAMCU_DIAG`` (``AMCU_EXTRA_NVCC_FLAGS=-DAMCU_DIAG python
-m aethermind_b200.build``) logs, for every CTA of the decode GEMV and fused
attention kernels, its SM and the globaltimer at entry, when its dependency
wait (griddepcontrol.wait) returned, two marks inside the kernel (GEMV:
activations staged, row blocks done; attention: q staged, key loop done),
and when it was done. This module runs a synthetic 8B W4 generation,
takes the log of its last decode steps and prints, per kernel role, medians
over the layers of:

  wait-prev   dependency wait released, after the previous launch's last CTA
  wait-sprd   spread of the wait release over the launch's CTAs
  med-done    median CTA done, after the first wait release
  max-done    last CTA done, after the first wait release
  span        last CTA done, after the previous launch's last CTA

Usage: python -m aethermind_b200.diag_timeline [--batch B] [--prompt T]
The default build has no timeline; this module then stops with a message.
"""
from __future__ import annotations

import argparse
import ctypes as C
import dataclasses

import numpy as np

REC = np.dtype([("tag", "u4"), ("cta", "u4"), ("smid", "u4"), ("grid", "u4"), ("t0", "u8"), ("tw", "u8"),
                ("td", "u8"), ("m1", "u8"), ("m2", "u8"), ("p3", "u8"), ("p4", "u8"), ("p5", "u8")])


def take(lib, name: str) -> np.ndarray:
    buf = np.zeros(1 << 18, REC)
    n = getattr(lib, name)(buf.ctypes.data_as(C.c_void_p), C.c_int(len(buf)))
    if n < 0:
        raise RuntimeError(f"{name} failed")
    return buf[:n]


def launches(rec: np.ndarray) -> list[dict]:
    """Groups the records into launches: a dependent launch's CTAs all finish
    after the previous launch's, so records sorted by finish time form one
    run per launch (consecutive launches differ in tag or grid)."""
    r = rec[np.argsort(rec["td"])]
    out, s = [], 0
    for i in range(1, len(r) + 1):
        if i == len(r) or not (r["tag"][i] == r["tag"][s] and r["grid"][i] == r["grid"][s]
                               and i - s < r["grid"][s]):
            g = r[s:i]
            out.append({"tag": int(g["tag"][0]), "grid": int(g["grid"][0]), **{k: g[k].astype(np.int64)
                        for k in ("t0", "tw", "td", "m1", "m2")}})
            s = i
    return out


def role(seq: list[dict], i: int) -> str:
    tag = seq[i]["tag"]
    if tag >= 2000:
        return "attention"
    if tag % 1000 // 10 == 2:
        return "gate_up"
    if tag % 1000 // 10 == 1:
        return "o" if i > 0 and seq[i - 1]["tag"] >= 2000 else "down"
    return "qkv" if i + 1 < len(seq) and seq[i + 1]["tag"] >= 2000 else "lm_head"


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--prompt", type=int, default=512)
    args = ap.parse_args()
    from aethermind_b200 import _lib as L
    from aethermind_b200 import session
    lib = L.lib()
    if not hasattr(lib, "amcu_diag_timeline_gemv"):
        raise SystemExit("this library has no timeline: build it with AMCU_EXTRA_NVCC_FLAGS=-DAMCU_DIAG")
    rt = session.Runtime(0)
    cfg = dataclasses.replace(session.LLAMA_8B_W4, max_seq=4096, max_batch=max(args.batch, 1))
    m = session.Model(rt, cfg)
    m.init_synthetic(0)
    s = session.Session(m)
    shape = (args.batch, args.prompt) if args.batch > 1 else args.prompt
    p = np.random.default_rng(1).integers(0, cfg.vocab, shape).astype(np.uint32)
    s.generate(p, 8)  # decode graph captured
    take(lib, "amcu_diag_timeline_gemv"), take(lib, "amcu_diag_timeline_attn")
    s.generate(p, 6)
    rec = np.concatenate([take(lib, "amcu_diag_timeline_gemv"), take(lib, "amcu_diag_timeline_attn")])
    _, dec, _ = s.timing()
    seq = launches(rec)
    per_step = 5 * cfg.layers + 1
    stats: dict[str, list] = {}
    for i in range(max(1, len(seq) - per_step), len(seq)):
        g, prev = seq[i], seq[i - 1]["td"].max()
        v = [(g["tw"].min() - prev) / 1e3, (g["tw"].max() - g["tw"].min()) / 1e3,
             (np.median(g["td"]) - g["tw"].min()) / 1e3, (g["td"].max() - g["tw"].min()) / 1e3,
             (g["td"].max() - prev) / 1e3]
        # marks: attention = q staged (m2), key loop done (m1); GEMV = activations staged (m2), row blocks done (m1)
        v += [(np.median(g["m2"]) - g["tw"].min()) / 1e3, (np.median(g["m1"] - g["m2"])) / 1e3,
              (np.median(g["td"] - g["m1"])) / 1e3]
        stats.setdefault(role(seq, i), []).append(v)
    print(f"decode ms per step (diagnostics build): {dec / 5:.3f}")
    print(f"{'role':10s} {'n':>3s} {'wait-prev':>9s} {'wait-sprd':>9s} {'med-done':>9s} {'max-done':>9s} {'span':>9s}  (us)")
    for k, vs in stats.items():
        a = np.median(np.array([x[:5] for x in vs]), axis=0)
        print(f"{k:10s} {len(vs):3d} " + " ".join(f"{x:9.2f}" for x in a))
    for k, vs in stats.items():
        a = np.median(np.array([x[5:] for x in vs]), axis=0)
        if k == "attention":
            print(f"attention phases (median CTA): q staged + append {a[0]:.2f}, key loop {a[1]:.2f}, "
                  f"merge + barriers + store {a[2]:.2f} us")
        else:
            print(f"{k} phases (median CTA): staging {a[0]:.2f}, row blocks {a[1]:.2f}, drain {a[2]:.2f} us")


if __name__ == "__main__":
    main()
