"""Builds libqmoe.so (CUDA kernels + C-ABI) in-tree for sm_100a.

nvcc cross-compiles without a GPU, so this runs on a CPU-only machine too.
Object files go to ``_build/`` beside the package (git-ignored); the shared
library is written next to this file so it travels with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libqmoe.so"
EP_LIB = PKG / "libqmoe_ep.so"
CUDA = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "--expt-relaxed-constexpr", f"-I{CSRC}", f"-I{INCLUDE}"]
# k_synth must not contract multiply-adds (bit-identical host/device synth)
PER_FILE = {"k_synth.cu": ["-fmad=false"]}
CU_SOURCES = ["k_decode.cu", "k_gemv.cu", "k_synth.cu", "k_dispatch.cu", "k_prefill.cu", "k_tgemm.cu", "k_ep.cu", "qmoe_abi.cu"]
CPP_SOURCES = ["synth_host.cpp"]


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("qmoe.h"))
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        if force or _stale(o, [s] + headers):
            cmd = [NVCC, *ARCH, *NVFLAGS, *PER_FILE.get(src, []), "-c", str(s), "-o", str(o)]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
        objs.append(o)
    for src in CPP_SOURCES:
        s = CSRC / src
        o = BUILD / (src + ".o")
        if force or _stale(o, [s] + headers):
            cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-fopenmp", "-ffp-contract=off", "-fvisibility=hidden",
                   f"-I{CSRC}", f"-I{INCLUDE}", "-c", str(s), "-o", str(o)]
            _run(cmd)
        objs.append(o)
    if force or _stale(LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fopenmp", "-o", str(LIB), *map(str, objs)])
    # the expert-parallel host layer over NCCL: its own library, so libqmoe
    # itself does not depend on NCCL
    ep_src = ROOT / "cpp" / "ep_host.cpp"
    if force or _stale(EP_LIB, [ep_src, LIB, INCLUDE / "qmoe.h", INCLUDE / "qmoe_ep.h"]):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden", "-Wall", "-Wextra", "-Werror",
              f"-I{INCLUDE}", f"-I{CUDA}/include", str(ep_src), "-o", str(EP_LIB), f"-L{PKG}", "-lqmoe",
              "-lnccl", f"-L{CUDA}/lib64", "-lcudart", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{CUDA}/lib64"])
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
