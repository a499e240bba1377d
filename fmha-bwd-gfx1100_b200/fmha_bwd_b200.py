"""Host-side mirror of the reference's Python/ctypes interface for the
attention-backward path, backed by the sm_100a libraries in build/.

Reference interface (benchmark_pytorch_final.py):
  * ``lib = ctypes.CDLL('./build/libfmha_bwd_bf16.so')`` with argtypes of
    8 x c_void_p + 4 x c_int (:30-37)
  * ``custom_flash_attn_backward(Q, K, V, P, dO)`` (:39-53): zero-fills the
    outputs and calls ``fmha_bwd_full_py`` with device pointers
  * ``pytorch_naive_backward`` (:58-70): einsum reference (no scale)
  * ``benchmark_size(batch, heads, M, N, K_dim, ...)`` (:82-136)

This module keeps those names, argument meanings and return values. It
differs from the reference script in three deliberate ways:
  * ``total_heads`` is ``batch * heads`` (the reference passes ``heads``,
    :51, which only covers batch 1);
  * the library is chosen by dtype (bf16 -> libfmha_bwd_bf16.so, fp16 ->
    libfmha_bwd_fp16.so) instead of always loading the bf16 one;
  * a call the library rejects raises ``FmhaBwdError`` with the library's
    error code and message instead of silently returning zeros.

There is no fallback: if the CUDA library is missing or the device is not an
sm_100 GPU, calls raise.
"""
from __future__ import annotations

import ctypes
import os

import torch

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT_DIR = os.path.dirname(PKG_DIR)
BUILD_DIR = os.path.join(ROOT_DIR, "build")

LIB_NAMES = {
    torch.bfloat16: ("libfmha_bwd_bf16.so", "fmha_bwd_full_py", "fmha_bwd_full_stream"),
    torch.float16: ("libfmha_bwd_fp16.so", "fmha_bwd_full_fp16", "fmha_bwd_full_fp16_stream"),
}
# precomputed-rowsum entries (additive to the reference's ABI)
DELTA_NAMES = {
    torch.bfloat16: "fmha_bwd_full_delta",
    torch.float16: "fmha_bwd_full_fp16_delta",
}

# recompute-P entries: P = exp(scale Q K^T - LSE) formed on chip
LSE_NAMES = {
    torch.bfloat16: "fmha_bwd_full_lse",
    torch.float16: "fmha_bwd_full_fp16_lse",
}

ERROR_NAMES = {
    0: "OK",
    1: "INVALID_ARGUMENT",
    2: "MISALIGNED",
    3: "UNSUPPORTED_DEVICE",
    4: "OUT_OF_MEMORY",
    5: "LAUNCH",
    6: "DEVICE_TIMEOUT",
    7: "NO_DRIVER",
}


class FmhaBwdError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"fmha_bwd error {code} ({ERROR_NAMES.get(code, '?')}): {message}")
        self.code = code


_LIBS: dict[str, ctypes.CDLL] = {}

_PTR_ARGS = [ctypes.c_void_p] * 8
_INT_ARGS = [ctypes.c_int] * 4


def library_path(dtype: torch.dtype) -> str:
    if dtype not in LIB_NAMES:
        raise TypeError(f"unsupported dtype {dtype}; use torch.bfloat16 or torch.float16")
    return os.path.join(BUILD_DIR, LIB_NAMES[dtype][0])


def load_library(dtype: torch.dtype = torch.bfloat16) -> ctypes.CDLL:
    """Load (once) and return the ctypes handle for ``dtype``'s library, with
    the same argtypes the reference script declares (:32-37)."""
    path = library_path(dtype)
    lib = _LIBS.get(path)
    if lib is not None:
        return lib
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is missing: build it with python fmha-bwd-gfx1100_b200/build_libs.py")
    lib = ctypes.CDLL(path)
    _, full, stream = LIB_NAMES[dtype]
    getattr(lib, full).argtypes = _PTR_ARGS + _INT_ARGS
    getattr(lib, full).restype = None
    getattr(lib, stream).argtypes = _PTR_ARGS + _INT_ARGS + [ctypes.c_void_p]
    getattr(lib, stream).restype = ctypes.c_int
    delta = DELTA_NAMES[dtype]
    getattr(lib, delta).argtypes = _PTR_ARGS + [ctypes.c_void_p] + _INT_ARGS + [ctypes.c_void_p]
    getattr(lib, delta).restype = ctypes.c_int
    lse = LSE_NAMES[dtype]
    getattr(lib, lse).argtypes = (_PTR_ARGS + [ctypes.c_void_p] + _INT_ARGS +
                                  [ctypes.c_float, ctypes.c_void_p])
    getattr(lib, lse).restype = ctypes.c_int
    lib.fmha_bwd_last_error.argtypes = []
    lib.fmha_bwd_last_error.restype = ctypes.c_int
    lib.fmha_bwd_last_error_message.argtypes = []
    lib.fmha_bwd_last_error_message.restype = ctypes.c_char_p
    lib.fmha_bwd_poll_device_status.argtypes = []
    lib.fmha_bwd_poll_device_status.restype = ctypes.c_int
    lib.fmha_bwd_set_wait_timeout_ms.argtypes = [ctypes.c_int]
    lib.fmha_bwd_set_wait_timeout_ms.restype = None
    _LIBS[path] = lib
    return lib


def rowsum_delta(P, dO, V):
    """D = rowsum(P * (dO V^T)) in fp32, [H, M] (reference formula,
    cpu_reference.hpp:32-35), computed with torch for callers and tests of
    the precomputed-rowsum entry."""
    dP = torch.einsum("...mk,...nk->...mn", dO.float(), V.float())
    return (dP * P.float()).sum(dim=-1).contiguous()


def last_error(dtype: torch.dtype = torch.bfloat16) -> tuple[int, str]:
    lib = load_library(dtype)
    return lib.fmha_bwd_last_error(), (lib.fmha_bwd_last_error_message() or b"").decode()


def _raise_if_error(lib: ctypes.CDLL, rc: int | None = None) -> None:
    code = lib.fmha_bwd_last_error() if rc is None else rc
    if code != 0:
        msg = (lib.fmha_bwd_last_error_message() or b"").decode()
        raise FmhaBwdError(code, msg)


def _check_inputs(Q, K, V, P, dO):
    for name, t in (("Q", Q), ("K", K), ("V", V), ("P", P), ("dO", dO)):
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        if t.dtype != Q.dtype:
            raise TypeError(f"{name} has dtype {t.dtype}, expected {Q.dtype}")


def fmha_bwd(Q, K, V, P, dO, *, out=None, stream=None, sync: bool = True, delta=None):
    """Backward of attention for head-flattened tensors.

    Q, dO: [H, M, d]; K, V: [H, N, d]; P: [H, M, N] (any leading shape that
    flattens to these, contiguous). Returns (dQ, dK, dV) with the shapes of
    Q, K, V. ``out`` may supply preallocated (dQ, dK, dV) tensors, which are
    fully overwritten. With ``sync=True`` the call uses the reference entry
    (``fmha_bwd_full_py`` / ``fmha_bwd_full_fp16``), which returns after the
    work has finished; with ``sync=False`` it uses the stream-ordered entry
    on ``stream`` (default: torch's current stream) and returns at once.
    ``delta``, when given, is D = rowsum(P * dP) (equivalently rowsum(dO * O)
    for the forward output O), an fp32 CUDA tensor of H*M elements; the
    precomputed-rowsum entry then skips the rowsum and one GEMM-sized pass
    (stream-ordered; synchronised afterwards when ``sync`` is set).
    """
    _check_inputs(Q, K, V, P, dO)
    d = Q.shape[-1]
    M = Q.shape[-2]
    N = K.shape[-2]
    H = Q.numel() // (M * d)
    if K.numel() != H * N * d or V.numel() != H * N * d or dO.numel() != H * M * d \
            or P.numel() != H * M * N:
        raise ValueError("inconsistent shapes for Q, K, V, P, dO")
    lib = load_library(Q.dtype)
    if out is None:
        dQ, dK, dV = torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V)
    else:
        dQ, dK, dV = out
    args = (dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), Q.data_ptr(), K.data_ptr(),
            V.data_ptr(), P.data_ptr(), dO.data_ptr(), M, N, d, H)
    _, full, stream_fn = LIB_NAMES[Q.dtype]
    if delta is not None:
        if not delta.is_cuda or delta.dtype != torch.float32 or not delta.is_contiguous() \
                or delta.numel() != H * M:
            raise ValueError("delta must be a contiguous fp32 CUDA tensor of H*M elements")
        s = stream if stream is not None else torch.cuda.current_stream(Q.device)
        rc = getattr(lib, DELTA_NAMES[Q.dtype])(*args[:8], delta.data_ptr(), *args[8:],
                                               ctypes.c_void_p(s.cuda_stream))
        _raise_if_error(lib, rc)
        if sync:
            s.synchronize()
        return dQ, dK, dV
    if sync:
        getattr(lib, full)(*args)
        _raise_if_error(lib)
    else:
        s = stream if stream is not None else torch.cuda.current_stream(Q.device)
        rc = getattr(lib, stream_fn)(*args, ctypes.c_void_p(s.cuda_stream))
        _raise_if_error(lib, rc)
    return dQ, dK, dV


def fmha_bwd_lse(Q, K, V, O, dO, LSE, scale: float, *, out=None, stream=None,
                 sync: bool = True):
    """Backward that recomputes P = exp(scale Q K^T - LSE) on chip instead of
    reading it (the FlashAttention form). Q, O, dO: [H, M, d]; K, V: [H, N, d];
    LSE: fp32 [H, M] (natural log of the row sums of exp(scale Q K^T)).
    Returns (dQ, dK, dV) = (scale dS K, scale dS^T Q, P^T dO) with
    dS = P (dO V^T - rowsum(dO * O)). Stream-ordered on ``stream`` (default:
    torch's current stream); with ``sync`` the call waits and raises on an
    in-kernel wait timeout."""
    for name, t in (("Q", Q), ("K", K), ("V", V), ("O", O), ("dO", dO)):
        if not t.is_cuda or not t.is_contiguous() or t.dtype != Q.dtype:
            raise ValueError(f"{name} must be a contiguous CUDA tensor of {Q.dtype}")
    d = Q.shape[-1]
    M, N = Q.shape[-2], K.shape[-2]
    H = Q.shape[:-2].numel()
    if K.shape[-1] != d or V.shape != K.shape or O.shape != Q.shape or dO.shape != Q.shape:
        raise ValueError("shape mismatch among Q, K, V, O, dO")
    if not LSE.is_cuda or LSE.dtype != torch.float32 or not LSE.is_contiguous() or LSE.numel() != H * M:
        raise ValueError("LSE must be a contiguous fp32 CUDA tensor of H*M elements")
    lib = load_library(Q.dtype)
    if out is None:
        out = (torch.empty_like(Q), torch.empty_like(K), torch.empty_like(V))
    dQ, dK, dV = out
    s = stream if stream is not None else torch.cuda.current_stream(Q.device)
    rc = getattr(lib, LSE_NAMES[Q.dtype])(
        dQ.data_ptr(), dK.data_ptr(), dV.data_ptr(), Q.data_ptr(), K.data_ptr(), V.data_ptr(),
        O.data_ptr(), dO.data_ptr(), LSE.data_ptr(), M, N, d, H, float(scale),
        ctypes.c_void_p(s.cuda_stream))
    _raise_if_error(lib, rc)
    if sync:
        s.synchronize()
        if lib.fmha_bwd_poll_device_status() != 0:
            raise FmhaBwdError(6, "fmha_bwd_lse: an in-kernel wait gave up")
    return dQ, dK, dV


# ---------------------------------------------------------------- stage hooks
# The reference's test_* wrappers (src/fmha_bwd_kernels.hip:525-560,
# src/fmha_bwd_kernels_fp16.hip:284-314), one stage per launch with its
# 16-bit intermediate in global memory. bf16 names have no suffix, fp16
# names end in _fp16.
STAGE_NAMES = ("dp", "softmax_bwd", "dq", "dk", "dv")


def _stage_fn(lib: ctypes.CDLL, dtype: torch.dtype, stage: str):
    name = f"test_{stage}_kernel" + ("_fp16" if dtype == torch.float16 else "")
    f = getattr(lib, name)
    if stage == "softmax_bwd":
        f.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3
    else:
        f.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 4
    f.restype = None
    return f


def run_stage(stage: str, a, b, *, sync: bool = True):
    """Run one stage hook on [H, rows, cols] inputs in the reference's
    argument order and return its output:
      dp (dO, V) -> dP [H,M,N];  softmax_bwd (P, dP) -> dS [H,M,N];
      dq (dS, K) -> dQ [H,M,d];  dk (dS, Q) -> dK [H,N,d];
      dv (P, dO) -> dV [H,N,d].
    The hook launches on the legacy default stream; with ``sync`` the call
    waits for it and raises on an error or an in-kernel wait timeout."""
    if stage not in STAGE_NAMES:
        raise ValueError(f"unknown stage {stage!r}; one of {STAGE_NAMES}")
    for name, t in (("a", a), ("b", b)):
        if not t.is_cuda or not t.is_contiguous() or t.dtype != a.dtype or t.dim() < 3:
            raise ValueError(f"{name} must be a contiguous CUDA tensor [H, rows, cols] of {a.dtype}")
    lib = load_library(a.dtype)
    H = a.shape[:-2].numel()
    if stage == "dp":  # dO [H,M,d], V [H,N,d]
        M, d = a.shape[-2:]
        N = b.shape[-2]
        out = torch.empty(*a.shape[:-1], N, dtype=a.dtype, device=a.device)
        ints = (M, N, d, H)
    elif stage == "softmax_bwd":  # P, dP [H,M,N]
        M, N = a.shape[-2:]
        out = torch.empty_like(a)
        ints = (M, N, H)
    elif stage == "dq":  # dS [H,M,N], K [H,N,d]
        M, N = a.shape[-2:]
        d = b.shape[-1]
        out = torch.empty(*a.shape[:-1], d, dtype=a.dtype, device=a.device)
        ints = (M, N, d, H)
    else:  # dk: dS [H,M,N], Q [H,M,d]; dv: P [H,M,N], dO [H,M,d]
        M, N = a.shape[-2:]
        d = b.shape[-1]
        out = torch.empty(*a.shape[:-2], N, d, dtype=a.dtype, device=a.device)
        ints = (M, N, d, H)
    _stage_fn(lib, a.dtype, stage)(a.data_ptr(), b.data_ptr(), out.data_ptr(), *ints)
    _raise_if_error(lib)
    if sync:
        torch.cuda.synchronize(a.device)
        if lib.fmha_bwd_poll_device_status() != 0:
            raise FmhaBwdError(6, f"stage {stage}: an in-kernel wait gave up")
    return out


def custom_flash_attn_backward(Q, K, V, P, dO):
    """Mirror of the reference's custom_flash_attn_backward
    (benchmark_pytorch_final.py:39-53) for [batch, heads, M, d] inputs.
    Outputs are zero-filled first, as the reference does (:43-45), then fully
    overwritten by the library."""
    batch, heads, M, K_dim = Q.shape
    dQ = torch.zeros_like(Q)
    dK = torch.zeros_like(K)
    dV = torch.zeros_like(V)
    return fmha_bwd(Q, K, V, P, dO, out=(dQ, dK, dV))


def pytorch_naive_backward(Q, K, V, P, dO):
    """The reference script's einsum formula (benchmark_pytorch_final.py:58-70),
    computed here in fp32 on the inputs' device. Test/benchmark reference only."""
    Qf, Kf, Vf, Pf, dOf = (t.float() for t in (Q, K, V, P, dO))
    dP = torch.einsum("...mk,...nk->...mn", dOf, Vf)
    rowsum = (dP * Pf).sum(dim=-1, keepdim=True)
    dS = Pf * (dP - rowsum)
    dQ = torch.einsum("...mn,...nk->...mk", dS, Kf)
    dK = torch.einsum("...mn,...mk->...nk", dS, Qf)
    dV = torch.einsum("...mn,...mk->...nk", Pf, dOf)
    return dQ, dK, dV


def _einsum_backward_native(Q, K, V, P, dO):
    """The reference script's einsum backward (benchmark_pytorch_final.py:58-70)
    in the inputs' own dtype, as that script times it (:110-115)."""
    dP = torch.einsum("...mk,...nk->...mn", dO, V)
    rowsum = (dP * P).sum(dim=-1, keepdim=True)
    dS = P * (dP - rowsum)
    dQ = torch.einsum("...mn,...nk->...mk", dS, K)
    dK = torch.einsum("...mn,...mk->...nk", dS, Q)
    dV = torch.einsum("...mn,...mk->...nk", P, dO)
    return dQ, dK, dV


def benchmark_size(batch, heads, M, N, K_dim, dtype=torch.bfloat16, warmup=5, reps=20):
    """Mirror of the reference's benchmark_size (benchmark_pytorch_final.py:82-136):
    seeded inputs, warmup, CUDA-event timing of ``reps`` synchronous calls and
    of ``reps`` einsum backwards in the inputs' dtype (the PyTorch baseline),
    FLOPs = 4 * 2*M*N*d per head (:125-127, here summed over batch*heads),
    and the max difference against the einsum reference (computed here in
    fp32). Returns the reference's keys: M, N, K, custom_time_ms,
    pytorch_time_ms, speedup, max_diff, custom_tflops."""
    device = torch.device("cuda")
    torch.manual_seed(42)
    Q = torch.randn(batch, heads, M, K_dim, dtype=dtype, device=device)
    K = torch.randn(batch, heads, N, K_dim, dtype=dtype, device=device)
    V = torch.randn(batch, heads, N, K_dim, dtype=dtype, device=device)
    dO = torch.randn(batch, heads, M, K_dim, dtype=dtype, device=device)
    P = torch.softmax(torch.randn(batch, heads, M, N, dtype=dtype, device=device), dim=-1)
    for _ in range(warmup):
        custom_flash_attn_backward(Q, K, V, P, dO)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(reps):
        dQ, dK, dV = custom_flash_attn_backward(Q, K, V, P, dO)
    end.record()
    torch.cuda.synchronize()
    custom_ms = start.elapsed_time(end) / reps
    for _ in range(warmup):
        _einsum_backward_native(Q, K, V, P, dO)
    torch.cuda.synchronize()
    start.record()
    for _ in range(reps):
        _einsum_backward_native(Q, K, V, P, dO)
    end.record()
    torch.cuda.synchronize()
    pt_ms = start.elapsed_time(end) / reps
    rQ, rK, rV = pytorch_naive_backward(Q, K, V, P, dO)
    max_diff = max((dQ.float() - rQ).abs().max().item(), (dK.float() - rK).abs().max().item(),
                   (dV.float() - rV).abs().max().item())
    flops = 4 * 2.0 * M * N * K_dim * batch * heads
    return {
        "M": M, "N": N, "K": K_dim,
        "custom_time_ms": custom_ms,
        "pytorch_time_ms": pt_ms,
        "speedup": pt_ms / custom_ms if custom_ms > 0 else 0.0,
        "max_diff": max_diff,
        "custom_tflops": flops / (custom_ms * 1e-3) / 1e12 if custom_ms > 0 else 0.0,
    }
