"""Builds libaethermind_b200.so in-tree with nvcc for sm_100a.

Every .cu / .cpp under csrc/ is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked into
``aethermind_b200/lib/libaethermind_b200.so`` (static CUDA runtime, so the
library does not depend on which libcudart another framework loaded first).
Objects are cached by content hash of the source and the headers it can see.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OBJ_DIR = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libaethermind_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _host_cxx() -> str:
    # The system g++ links libstdc++ dynamically (a wrapper elsewhere on PATH
    # may link it statically, which breaks loading next to numpy/torch).
    return "/usr/bin/g++" if Path("/usr/bin/g++").exists() else (shutil.which("g++") or "g++")


def _sources() -> list[Path]:
    return sorted([p for p in CSRC.rglob("*") if p.suffix in (".cu", ".cpp")])


def _headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) + list(INCLUDE.glob("*.h"))):
        h.update(p.read_bytes())
    return h.hexdigest()


def _flags() -> list[str]:
    return [
        "-std=c++20", "-O3", "-lineinfo", *ARCH,
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        "-ccbin", _host_cxx(),
        f"-I{INCLUDE}", f"-I{CSRC}",
        "-DAMCU_BUILD",
        *os.environ.get("AMCU_EXTRA_NVCC_FLAGS", "").split(),
    ]


def _compile(src: Path, hdr: str, verbose: bool) -> Path:
    key = hashlib.sha256(src.read_bytes() + hdr.encode() + " ".join(_flags()).encode()).hexdigest()[:16]
    obj = OBJ_DIR / f"{src.stem}-{key}.o"
    if obj.exists():
        return obj
    cmd = [_nvcc(), *_flags(), "-x", "cu" if src.suffix == ".cu" else "c++", "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu" and verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    hdr = _headers_digest()
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        objs = list(ex.map(lambda s: _compile(s, hdr, verbose), srcs))
    stamp = hashlib.sha256("".join(str(o) for o in objs).encode()).hexdigest()
    stamp_file = LIB_DIR / ".stamp"
    if LIB.exists() and stamp_file.exists() and stamp_file.read_text() == stamp:
        return LIB
    cmd = [_nvcc(), *ARCH, "-shared", "-ccbin", _host_cxx(), "-o", str(LIB), *map(str, objs),
           "-lcuda", "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
    stamp_file.write_text(stamp)
    # drop stale objects
    keep = {o.name for o in objs}
    for o in OBJ_DIR.glob("*.o"):
        if o.name not in keep:
            o.unlink()
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
