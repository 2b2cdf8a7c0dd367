"""Build libsoc_b200.so in-tree with nvcc for sm_100a (no GPU needed to build), and the
soc_b200_cli runner beside it.

    python -m soc_b200.build            # incremental
    python -m soc_b200.build --force    # rebuild
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libsoc_b200.so"
CLI = PKG / "soc_b200_cli"
OBJ = PKG / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden"]

SOURCES = ["runtime.cu", "kernels.cu", "decode_mk.cu", "gemm_tc.cu", "attn_prefill.cu", "nccl_rt.cu", "attn_decode.cu", "tokenizer.cu",
           "attn_prefill_tc.cu", "tp_allreduce.cu", "linear_mma.cu"]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.h")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + \
        [PKG.parent / "include" / "soc_b200.h"]
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = OBJ / (s.stem + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", str(s), "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
                print(" ".join(cmd), flush=True)
            subprocess.run(cmd, check=True)
    if force or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcuda", "-ldl"]
        subprocess.run(cmd, check=True)
    # The command-line runner (host C++ over the C ABI; finds the library next to itself).
    cli_src = CSRC / "cli.cpp"
    if force or _stale(CLI, [cli_src, LIB, PKG.parent / "include" / "soc_b200.h"]):
        cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-I", str(PKG.parent / "include"), str(cli_src),
               "-o", str(CLI), "-L", str(PKG), "-lsoc_b200", "-Wl,-rpath,$ORIGIN"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
