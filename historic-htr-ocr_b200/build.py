"""Build libocrcuda.so in-tree (historic-htr-ocr_b200/lib/) for sm_100a with nvcc.

    python historic-htr-ocr_b200/build.py [--force] [--verbose]

Each translation unit under csrc/ compiles to an object under _build/ (skipped while newer than its sources), then
one shared library links them with the static CUDA runtime. No torch headers or libraries are involved: the library
is a plain C ABI (include/ocr_cuda.h).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libocrcuda.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
                  "-I", str(ROOT / "include"), "-I", str(CSRC)]


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers():
    return list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))


def _stale(obj: Path, src: Path, hdr_mtime: float) -> bool:
    return not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr_mtime)


def _compile(src: Path, verbose: bool, extra: list[str]) -> Path:
    obj = BUILD / (src.name + ".o")
    cmd = [NVCC, *CUFLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [NVCC, "-x", "cu", *CUFLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, flush=True)
    return obj


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    hdr = max((h.stat().st_mtime for h in _headers()), default=0.0)
    srcs = _sources()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    todo = [s for s in srcs if force or ptxas_info or _stale(BUILD / (s.name + ".o"), s, hdr)]
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda s: _compile(s, verbose or ptxas_info, extra), todo))
    objs = [BUILD / (s.name + ".o") for s in srcs]
    if force or todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="rebuild with -Xptxas -v (registers, spills, smem)")
    a = ap.parse_args()
    try:
        print(build(a.force, a.verbose, a.ptxas_info))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
