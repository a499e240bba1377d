"""Python side of the CPU oracle. TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, and only as the checker; the product libraries never call it.

Two CPU implementations are exposed:

* ``oracle_bwd`` -- the restatement in ``fmha_bwd_oracle.cpp`` of the
  reference's ``fmha_backward_cpu`` (src/kernel/correct/cpu_reference.hpp:74-126),
  returning unrounded fp32 dQ/dK/dV and the rowsum D.
* ``reference_bwd`` -- the reference's own ``cpu_reference.hpp`` compiled from
  the reference tree by ``oracle/Makefile`` into ``oracle/_ref/``; its outputs
  are the reference's half_t results widened to fp32.

``make_inputs`` builds the seeded inputs of the workload definitions: Q, K, V,
dO ~ N(0, 1) (dO ~ N(0, 0.1) for the cross-attention case), and
P = softmax(Q K^T / sqrt(d)) computed in fp32 and then stored in the 16-bit
input type.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_oracle.so")

_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)

_libs: dict[str, ctypes.CDLL] = {}


def build(ref_root: str | None = None) -> None:
    """Compile the oracle libraries (and the reference one when its tree exists)."""
    args = ["make", "-s", "-C", HERE]
    if ref_root:
        args.append(f"REF={ref_root}")
    subprocess.run(args, check=True)


def _load(path: str) -> ctypes.CDLL:
    if path not in _libs:
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built (run make -C oracle)")
        lib = ctypes.CDLL(path)
        _libs[path] = lib
    return _libs[path]


def have_reference() -> bool:
    return os.path.exists(REF_SO)


def _u16(a: np.ndarray):
    assert a.dtype == np.uint16 and a.flags.c_contiguous
    return a.ctypes.data_as(_u16p)


def _f32(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_f32p)


def oracle_bwd(Q, K, V, P, dO, dtype: str, threads: int = 0):
    """Restated oracle. Inputs: uint16 bit arrays [H,M,d], [H,N,d], [H,N,d],
    [H,M,N], [H,M,d]. Returns fp32 (dQ, dK, dV, D)."""
    lib = _load(ORACLE_SO)
    H, M, d = Q.shape
    N = K.shape[1]
    dQ = np.empty((H, M, d), np.float32)
    dK = np.empty((H, N, d), np.float32)
    dV = np.empty((H, N, d), np.float32)
    Dsum = np.empty((H, M), np.float32)
    fn = lib.oracle_fmha_bwd_bf16 if dtype == "bf16" else lib.oracle_fmha_bwd_fp16
    fn.restype = ctypes.c_int
    threads = threads or min(H, os.cpu_count() or 1)
    rc = fn(_u16(Q), _u16(K), _u16(V), _u16(P), _u16(dO), _f32(dQ), _f32(dK),
            _f32(dV), _f32(Dsum), M, N, d, H, threads)
    if rc != 0:
        raise ValueError("oracle rejected the sizes")
    return dQ, dK, dV, Dsum


def reference_bwd(Q, K, V, P, dO, dtype: str, threads: int = 0):
    """The reference's own fmha_backward_cpu, one call per head."""
    lib = _load(REF_SO)
    H, M, d = Q.shape
    N = K.shape[1]
    dQ = np.empty((H, M, d), np.float32)
    dK = np.empty((H, N, d), np.float32)
    dV = np.empty((H, N, d), np.float32)
    lib.ref_fmha_bwd.restype = ctypes.c_int
    threads = threads or min(H, os.cpu_count() or 1)
    rc = lib.ref_fmha_bwd(_u16(Q), _u16(K), _u16(V), _u16(P), _u16(dO),
                          _f32(dQ), _f32(dK), _f32(dV), M, N, d, H,
                          1 if dtype == "bf16" else 0, threads)
    if rc != 0:
        raise ValueError("reference rejected the sizes")
    return dQ, dK, dV


# ---------------------------------------------------------------- inputs


def to_bits(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round fp32 to the 16-bit storage type (round-to-nearest-even) and
    return the raw bits as uint16."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == "fp16":
        return x.astype(np.float16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint16)
    out[nan] = 0x7FC0
    return out


def from_bits(b: np.ndarray, dtype: str) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint16)
    if dtype == "fp16":
        return b.view(np.float16).astype(np.float32)
    return (b.astype(np.uint32) << 16).view(np.float32)


def make_inputs(M: int, N: int, d: int, H: int, dtype: str = "bf16",
                seed: int = 42, do_std: float = 1.0):
    """Seeded inputs as uint16 bit arrays (Q, K, V, P, dO).

    Uses numpy's PCG64 generator so the same inputs can be rebuilt anywhere
    without a GPU. P is softmax(Q K^T / sqrt(d)) over the 16-bit-rounded Q
    and K, computed in fp32, then rounded to the storage type."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((H, M, d), dtype=np.float32)
    k = rng.standard_normal((H, N, d), dtype=np.float32)
    v = rng.standard_normal((H, N, d), dtype=np.float32)
    o = (rng.standard_normal((H, M, d), dtype=np.float32) * np.float32(do_std))
    Q, K, V, dO = (to_bits(a, dtype) for a in (q, k, v, o))
    qf, kf = from_bits(Q, dtype), from_bits(K, dtype)
    s = np.matmul(qf, kf.transpose(0, 2, 1)) * np.float32(1.0 / np.sqrt(d))
    s -= s.max(axis=-1, keepdims=True)
    np.exp(s, out=s)
    s /= s.sum(axis=-1, keepdims=True)
    P = to_bits(s, dtype)
    return Q, K, V, P, dO


# ---------------------------------------------------------------- metrics


def max_abs(a: np.ndarray, ref: np.ndarray) -> float:
    return float(np.max(np.abs(a.astype(np.float64) - ref.astype(np.float64)))) if a.size else 0.0


def rel_l2(a: np.ndarray, ref: np.ndarray) -> float:
    a = a.astype(np.float64)
    ref = ref.astype(np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(a - ref)
    return float(num / den) if den > 0 else float(num)


# Tolerances for 16-bit GPU outputs against the fp32 oracle (per output):
# relative L2 error and max-abs error as a fraction of max|ref|.
TOLERANCE = {
    "bf16": {"rel_l2": 1e-2, "max_abs_frac": 2e-2},
    "fp16": {"rel_l2": 5e-3, "max_abs_frac": 1e-2},
}


def check(name: str, got: np.ndarray, ref: np.ndarray, dtype: str) -> dict:
    """Return the error metrics of ``got`` against ``ref`` and whether they
    meet the tolerance for ``dtype``."""
    tol = TOLERANCE[dtype]
    r = rel_l2(got, ref)
    m = max_abs(got, ref)
    scale = float(np.max(np.abs(ref))) if ref.size else 0.0
    ok = (r <= tol["rel_l2"]) and (m <= tol["max_abs_frac"] * max(scale, 1e-30))
    return {"name": name, "rel_l2": r, "max_abs": m, "max_ref": scale, "ok": bool(ok)}
