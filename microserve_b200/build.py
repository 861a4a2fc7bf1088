"""Build the in-tree CUDA library `libmicroserve_b200.so` for sm_100a.

Each `csrc/*.cu` is compiled with nvcc as relocatable device code (the
kernels share one device status word), then device-linked into a shared
library next to this file. Objects go to `_build/` at the repository root.
Rebuilds only what changed (source or header newer than its object).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libmicroserve_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC,-O2",
         "--expt-relaxed-constexpr", "-I", str(ROOT / "include")]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))
    nvcc = _nvcc()
    flags = FLAGS + (extra_flags or [])
    jobs = []
    for s in srcs:
        o = BUILD / (s.stem + ".o")
        if _stale(o, s, headers):
            jobs.append([nvcc, *ARCH, *flags, "-c", str(s), "-o", str(o)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(run, jobs))
    objs = [str(BUILD / (s.stem + ".o")) for s in srcs]
    if jobs or not LIB.exists() or any(Path(o).stat().st_mtime > LIB.stat().st_mtime for o in objs):
        run([nvcc, *ARCH, "-rdc=true", "-shared", "-Xcompiler", "-fPIC", *objs, "-o", str(LIB)])
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
