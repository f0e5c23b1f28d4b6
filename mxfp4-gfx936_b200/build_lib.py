"""Build libmxfp4_b200.so in this directory (nvcc, sm_100a).

    python mxfp4-gfx936_b200/build_lib.py [--verbose]

The library is one translation unit (csrc/capi.cu includes every kernel
header) compiled for ``sm_100a`` only; the CUDA runtime is linked statically,
so the .so depends only on the driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "libmxfp4_b200.so"
SOURCES = [HERE / "csrc" / "capi.cu"]
DEPS = sorted((HERE / "csrc").glob("*.cu*")) + [HERE.parent / "include" / "mxfp4_b200.h"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def flags(verbose: bool = False) -> list[str]:
    f = [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC,-O3", "-shared",
        "-cudart", "static",
        f"-I{HERE.parent / 'include'}",
    ]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def up_to_date() -> bool:
    if not LIB.is_file():
        return False
    t = LIB.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *flags(verbose), "-o", str(tmp), *map(str, SOURCES)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode}): {' '.join(cmd)}")
    if verbose:
        sys.stdout.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose="--verbose" in sys.argv))
