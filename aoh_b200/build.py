"""Build libaoh.so (all CUDA sources under csrc/) for sm_100a, in-tree.

    python -m aoh_b200.build [-v] [--force]

Each .cu is compiled to an object under aoh_b200/_build/ (in parallel), then
linked into aoh_b200/libaoh.so with the CUDA runtime linked statically, so the
library loads on machines without a GPU driver (the driver is resolved at the
first CUDA call).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libaoh.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found (CUDA toolkit required to build libaoh.so)")
    return cand


def sources():
    return sorted(CSRC.glob("*.cu"))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout.strip() or r.stderr.strip()):
        print(r.stdout + r.stderr, flush=True)
    return obj


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    hdr = _headers_mtime()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    todo = []
    for s in srcs:
        obj = BUILD / (s.stem + ".o")
        if force or ptxas_verbose or not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, hdr):
            todo.append(s)
    if todo:
        with ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            list(ex.map(lambda s: _compile(s, verbose or ptxas_verbose, extra), todo))
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print ptxas register/spill report")
    a = ap.parse_args(argv)
    p = build(verbose=a.verbose, force=a.force, ptxas_verbose=a.ptxas)
    print(p)


if __name__ == "__main__":
    sys.exit(main())
