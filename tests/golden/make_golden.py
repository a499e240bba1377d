"""Generates the golden fixtures in this directory from the reference's own
CPU backward (src/kernel/correct/cpu_reference.hpp:74-126), built from the
reference tree by oracle/Makefile into oracle/_ref/libref_oracle.so.

Each fixture <name>.npz holds the seeded 16-bit inputs (raw bits, uint16) and
the reference's dQ/dK/dV (its half_t outputs, stored as float16), plus the
sizes. The reference itself is not available where the GPU tests run, so the
fixtures carry its answers there.

Run from the repository root after `make -C oracle`:
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402

# name: (M, N, d, H, dtype, seed, dO std)
CASES = {
    # the CPU-runnable correctness case: M=N=128, d=64, 2 heads, bf16
    "cpu_case_bf16": (128, 128, 64, 2, "bf16", 42, 1.0),
    "cpu_case_fp16": (128, 128, 64, 2, "fp16", 42, 1.0),
    # ragged tails in both M and N (not multiples of the 128 tile)
    "ragged_bf16_d128": (200, 136, 128, 3, "bf16", 7, 1.0),
    "ragged_fp16_d64": (77, 264, 64, 2, "fp16", 8, 1.0),
    # cross-attention shape: more queries than keys, small dO
    "cross_bf16_d128": (384, 64, 128, 2, "bf16", 9, 0.1),
    # smallest legal shape: one query row, 8 keys
    "tiny_bf16_d64": (1, 8, 64, 1, "bf16", 10, 1.0),
}


def main() -> None:
    if not O.have_reference():
        raise SystemExit("oracle/_ref/libref_oracle.so is not built (make -C oracle)")
    for name, (M, N, d, H, dtype, seed, std) in CASES.items():
        Q, K, V, P, dO = O.make_inputs(M, N, d, H, dtype, seed=seed, do_std=std)
        dQ, dK, dV = O.reference_bwd(Q, K, V, P, dO, dtype)
        path = os.path.join(HERE, f"{name}.npz")
        np.savez_compressed(
            path, M=M, N=N, d=d, H=H, dtype=dtype, seed=seed, do_std=std,
            Q=Q, K=K, V=V, P=P, dO=dO,
            dQ=dQ.astype(np.float16), dK=dK.astype(np.float16), dV=dV.astype(np.float16))
        print(f"{path}: {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
