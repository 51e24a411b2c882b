"""Build the CPU oracle (test infrastructure): oracle/_build/liboracle.so from oracle.c and vision.c with gcc.

    python oracle/build.py [--force]

-ffp-contract=off keeps every a*b+c unfused, as Rust and WGSL evaluate it; OpenMP uses all host cores.
x86-64-v3 (AVX2 + FMA) is the baseline ISA so the library built here also runs on the GPU hosts.
The reference itself (Rust + WGSL on wgpu) cannot be compiled here: there is no Rust toolchain and no graphics
adapter, so there is no oracle/_ref build.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_build" / "liboracle.so"
FLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fno-math-errno", "-fPIC", "-shared",
         "-std=c11", "-Wall", "-Wno-unknown-pragmas"]


def build(force: bool = False) -> Path:
    src = [HERE / "oracle.c", HERE / "vision.c"]
    hdr = [HERE / "oracle.h"]
    if not force and OUT.exists() and OUT.stat().st_mtime >= max(p.stat().st_mtime for p in src + hdr):
        return OUT
    OUT.parent.mkdir(exist_ok=True)
    cmd = ["gcc", *FLAGS, *map(str, src), "-o", str(OUT), "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"gcc failed:\n{r.stdout}\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    try:
        print(build("--force" in sys.argv))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
