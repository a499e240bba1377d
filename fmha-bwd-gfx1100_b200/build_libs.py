"""Builds the two sm_100a attention-backward libraries in-tree:

    build/libfmha_bwd_bf16.so   (fmha_bwd_full_py, fmha_bwd_full_stream, ...)
    build/libfmha_bwd_fp16.so   (fmha_bwd_full_fp16, fmha_bwd_full_fp16_stream, ...)

at the repository root, the paths the reference's ctypes host loads
(benchmark_pytorch_final.py:30 loads ./build/libfmha_bwd_bf16.so). nvcc
cross-compiles for sm_100a without a GPU. Run: python build_libs.py [--force]
"""
from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT = os.path.join(ROOT, "build")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xcompiler", "-fvisibility=hidden",
]

LIBS = {
    "libfmha_bwd_bf16.so": "fmha_bwd_bf16.cu",
    "libfmha_bwd_fp16.so": "fmha_bwd_fp16.cu",
}


def _sources_mtime() -> float:
    return max(os.path.getmtime(os.path.join(CSRC, f)) for f in os.listdir(CSRC))


def build(force: bool = False, verbose: bool = False) -> list[str]:
    os.makedirs(OUT, exist_ok=True)
    newest = _sources_mtime()
    built = []
    for lib, src in LIBS.items():
        out = os.path.join(OUT, lib)
        if not force and os.path.exists(out) and os.path.getmtime(out) >= newest:
            built.append(out)
            continue
        cmd = [NVCC, *FLAGS, "-o", out, os.path.join(CSRC, src)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True, cwd=CSRC)
        built.append(out)
    return built


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv, verbose="-v" in sys.argv):
        print(p)
