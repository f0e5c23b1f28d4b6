"""Build libmxfp4_b200.so in this directory (nvcc, sm_100a).

    python mxfp4-gfx936_b200/build_lib.py [--verbose]

The library is one translation unit (csrc/capi.cu includes every kernel
header) compiled for ``sm_100a`` only; the CUDA runtime is linked statically,
so the .so depends only on the driver at run time.  The benchmark's
tensor-core rate probe (csrc/probe_mma.cu) is built beside it as
libmxfp4_b200_probe.so.
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
DEPS = sorted((HERE / "csrc").glob("*.cuh")) + [HERE / "csrc" / "capi.cu", HERE.parent / "include" / "mxfp4_b200.h"]
# the tensor-core rate probe the benchmark reads its FP4 denominator from (not
# part of the operator library)
PROBE_LIB = HERE / "libmxfp4_b200_probe.so"
PROBE_SOURCES = [HERE / "csrc" / "probe_mma.cu"]
PROBE_DEPS = sorted((HERE / "csrc").glob("*.cuh")) + PROBE_SOURCES + [HERE.parent / "include" / "mxfp4_b200_probe.h"]


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


def up_to_date(lib: Path = LIB, deps=DEPS) -> bool:
    if not lib.is_file():
        return False
    t = lib.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in deps)


def _compile(lib: Path, sources, verbose: bool) -> None:
    tmp = lib.with_suffix(".so.tmp")
    cmd = [nvcc(), *flags(verbose), "-o", str(tmp), *map(str, sources)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode}): {' '.join(cmd)}")
    if verbose:
        sys.stdout.write(res.stderr)
    os.replace(tmp, lib)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Build the operator library and the rate probe; returns the former."""
    if force or not up_to_date(PROBE_LIB, PROBE_DEPS):
        _compile(PROBE_LIB, PROBE_SOURCES, verbose)
    if force or not up_to_date():
        _compile(LIB, SOURCES, verbose)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose="--verbose" in sys.argv))
