"""Build the sm_100a C-ABI library qw3_b200/libds3cuda.so with nvcc.

The library is built in-tree so it travels with the repository snapshot to a
GPU machine. It links the CUDA runtime statically and exports only the
``ds3_cuda_*`` entry points declared in include/ds3_cuda.h.

Usage: python -m qw3_b200.build [--verbose-ptxas]
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
LIB = PKG / "libds3cuda.so"
SOURCES = ["ds3_cuda.cu", "norm.cu", "embed.cu", "rope.cu", "router.cu", "moe.cu", "moe_route.cu", "router_gemv.cu", "gguf.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


HOST_SRC = PKG / "host" / "ds3_chunk_pre.c"
HOST_BIN = PKG / "host" / "ds3_chunk_pre"
HOST_PROGRAMS = ("ds3_chunk_pre", "ds3_gguf_info")


def build_host(name: str = "ds3_chunk_pre") -> Path:
    """A C host program of qw3_b200/host/, linked against libds3cuda.so (found
    via rpath); builds all of them when called from build()."""
    src, out = PKG / "host" / f"{name}.c", PKG / "host" / name
    headers = list((ROOT / "include").glob("*.h"))
    if out.exists() and out.stat().st_mtime > max(p.stat().st_mtime for p in [src, LIB, *headers]):
        return out
    cc = shutil.which("gcc") or "cc"
    cmd = [cc, "-O2", "-std=c11", "-Wall", "-Wextra", "-I", str(ROOT / "include"), str(src),
           "-L", str(PKG), "-lds3cuda", "-Wl,-rpath,$ORIGIN/..", "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"building the C host program {name} failed")
    return out


def needs_rebuild() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps.append(ROOT / "include" / "ds3_cuda.h")
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, ptxas_verbose: bool = False) -> Path:
    if not force and not needs_rebuild():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared",
        "-Xcompiler", "-fPIC,-fvisibility=hidden", "-Xcompiler", "-O2",
        "-I", str(ROOT / "include"), "-I", str(CSRC),
        "-cudart", "static",
        "-o", str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if ptxas_verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libds3cuda.so")
    if ptxas_verbose:
        sys.stderr.write(res.stderr)
    tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    build(force=True, ptxas_verbose="--verbose-ptxas" in sys.argv)
    for prog in HOST_PROGRAMS:
        build_host(prog)
    print(LIB)
