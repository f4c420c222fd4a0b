"""Build the in-tree CUDA extension ``leo_b200/libleo_b200.so`` for sm_100a.

Steps: generate ``include/leo_cuda_abi.h`` from ``cuda_abi.def``; generate the
libm exception tables (``csrc/libm_tables.inc``) by comparing the kernels'
double-precision exp/log against the platform libm; compile every ``.cu`` /
``.cpp`` under ``csrc/`` with nvcc for ``compute_100a``/``sm_100a`` and link
one shared library.  Device code is built with ``-fmad=false`` so no
multiply-add is fused (the reference's Rust arithmetic never fuses), host code
with ``-ffp-contract=off``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libleo_b200.so"
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["leo_wavefront.cu", "leo_merge_kernels.cu", "leo_shard_kernels.cu", "leo_sparse_apply.cu", "leo_schedule.cu",
              "leo_context_merge.cu", "leo_runtime.cu"]
CPP_SOURCES = ["leo_host_model.cpp"]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"command failed: {' '.join(cmd)}")


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def generate_tables() -> Path:
    inc = CSRC / "libm_tables.inc"
    gen_src = CSRC / "gen_libm_tables.cpp"
    gen_bin = BUILD / "gen_libm_tables"
    BUILD.mkdir(exist_ok=True)
    if _stale(gen_bin, [gen_src, CSRC / "leo_math.cuh"]):
        _run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-o", str(gen_bin), str(gen_src),
              "-lpthread"])
    if _stale(inc, [gen_bin]):
        _run([str(gen_bin), str(inc)])
    return inc


def build(verbose: bool = False) -> Path:
    from .abi.generate import write_header

    write_header()
    generate_tables()
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.inc")) + \
        list((ROOT / "include").glob("*.h"))
    objects = []
    common = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include")]
    for name in CU_SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        if _stale(obj, [src] + headers):
            cmd = [NVCC, *ARCH, *common, "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
                   "-Xcompiler", "-ffp-contract=off", "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd)
        objects.append(obj)
    for name in CPP_SOURCES:
        src = CSRC / name
        obj = BUILD / (name + ".o")
        if _stale(obj, [src] + headers):
            _run(["g++", "-std=c++17", "-O2", "-fPIC", "-ffp-contract=off", "-fno-fast-math", "-I",
                  str(ROOT / "include"), "-c", str(src), "-o", str(obj)])
        objects.append(obj)
    if _stale(LIB, objects):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objects), "-lcudart"])
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    _ = os
