"""Build libedgecore_b200.so in-tree: nvcc for the sm_100a kernels, gcc (C11)
for the host library, linked with the static CUDA runtime.

    python -m edgecore_b200.build [--force]

Objects go to edgecore_b200/_build/; the shared library to
edgecore_b200/libedgecore_b200.so.  Only the symbols of include/edgecore.h and
include/edgecore_b200.h are exported.  With EDGECORE_B200_TRACE=1 the same
sources build the diagnostic variant libedgecore_b200_trace.so (objects in
_build_trace/), whose decode kernel records the per-phase timeline that
ec_decode_trace returns.
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
LIB = PKG / "libedgecore_b200.so"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["ec_kernels.cu", "ec_decode.cu", "ec_tc.cu", "ec_noalloc.cu"]
C_SOURCES = ["ec_host.c", "ec_abi.c"]
HEADERS = [CSRC / "ec_launch.h", CSRC / "ec_common.cuh", CSRC / "ec_decode.h", ROOT / "include" / "edgecore.h",
           ROOT / "include" / "edgecore_b200.h"]


def _cc() -> str:
    return "/usr/bin/gcc" if Path("/usr/bin/gcc").exists() else (shutil.which("gcc") or "gcc")


def _nvcc() -> str:
    p = CUDA / "bin" / "nvcc"
    return str(p) if p.exists() else "nvcc"


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps if d.exists())


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} {cmd[-1]}")


def build(force: bool = False, verbose: bool = False) -> Path:
    trace = os.environ.get("EDGECORE_B200_TRACE") == "1"
    bdir = PKG / "_build_trace" if trace else BUILD
    lib = PKG / "libedgecore_b200_trace.so" if trace else LIB
    bdir.mkdir(exist_ok=True)
    objs: list[Path] = []
    inc = ["-I", str(ROOT / "include"), "-I", str(CSRC)] + (["-DEC_DECODE_TRACE"] if trace else [])
    for src in CU_SOURCES:
        s, o = CSRC / src, bdir / (Path(src).stem + ".o")
        if force or _stale(o, [s, *HEADERS]):
            cmd = [_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                   "--expt-relaxed-constexpr", *inc, "-c", str(s), "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd)
        objs.append(o)
    for src in C_SOURCES:
        s, o = CSRC / src, bdir / (Path(src).stem + ".o")
        if force or _stale(o, [s, *HEADERS]):
            _run([_cc(), "-std=c11", "-O2", "-fPIC", "-fvisibility=hidden", "-Wall", "-Wextra",
                  "-Wno-unused-parameter", *inc, "-I", str(CUDA / "include"), "-c", str(s), "-o", str(o)])
        objs.append(o)
    if force or _stale(lib, objs):
        tmp = lib.with_suffix(".so.tmp")
        _run([_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
              "-Xlinker", "--exclude-libs=ALL", "-Xlinker", "-Bsymbolic", "-lpthread", "-lm", "-ldl", "-lrt"])
        tmp.replace(lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
