"""CPU tests of the C-ABI boundary: both libraries load, export every entry
point include/fmha_bwd.h declares, and reject bad calls before touching the
GPU (so these run without one)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "fmha_bwd.h")
LIBS = {
    "bf16": os.path.join(ROOT, "build", "libfmha_bwd_bf16.so"),
    "fp16": os.path.join(ROOT, "build", "libfmha_bwd_fp16.so"),
}


def _ensure_built():
    if not all(os.path.exists(p) for p in LIBS.values()):
        import build_libs

        build_libs.build()


def header_functions():
    """{section: [function names]} from the header's ---- section markers."""
    text = open(HEADER).read()
    sections = {"bf16": [], "fp16": [], "both": []}
    current = None
    for line in text.splitlines():
        if "---- libfmha_bwd_bf16.so" in line:
            current = "bf16"
        elif "---- libfmha_bwd_fp16.so" in line:
            current = "fp16"
        elif "---- exported by both libraries" in line:
            current = "both"
        m = re.match(r"^\s*(?:void|int|const char\s*\*)\s+(\w+)\s*\(", line)
        if m and current:
            sections[current].append(m.group(1))
    return sections


def exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if l.strip()}


def test_header_declares_reference_entry_points():
    s = header_functions()
    assert "fmha_bwd_full_py" in s["bf16"]
    assert "fmha_bwd_full_fp16" in s["fp16"]
    assert "fmha_bwd_last_error" in s["both"]


@pytest.mark.parametrize("kind", ["bf16", "fp16"])
def test_library_exports_every_declared_symbol(kind):
    _ensure_built()
    s = header_functions()
    want = set(s[kind]) | set(s["both"])
    have = exported(LIBS[kind])
    assert want <= have, f"missing exports: {sorted(want - have)}"
    lib = ctypes.CDLL(LIBS[kind])
    for name in want:
        assert getattr(lib, name) is not None


def _call_full(lib, fn, ptrs, M, N, d, H):
    f = getattr(lib, fn)
    f.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int] * 4
    f.restype = None
    f(*ptrs, M, N, d, H)
    lib.fmha_bwd_last_error.restype = ctypes.c_int
    lib.fmha_bwd_last_error_message.restype = ctypes.c_char_p
    return lib.fmha_bwd_last_error(), lib.fmha_bwd_last_error_message().decode()


@pytest.mark.parametrize("kind,fn", [("bf16", "fmha_bwd_full_py"), ("fp16", "fmha_bwd_full_fp16")])
def test_rejects_bad_arguments_without_gpu(kind, fn):
    """Preconditions are checked on the host before any CUDA call; each bad
    call returns the documented error code (no GPU needed)."""
    _ensure_built()
    lib = ctypes.CDLL(LIBS[kind])
    good = [0x10000 * (i + 1) for i in range(8)]  # never dereferenced: rejected earlier
    code, msg = _call_full(lib, fn, [None] + good[1:], 128, 128, 64, 2)
    assert code == 1 and "null" in msg
    code, _ = _call_full(lib, fn, good, 0, 128, 64, 2)
    assert code == 1
    code, _ = _call_full(lib, fn, good, 128, -5, 64, 2)
    assert code == 1
    code, msg = _call_full(lib, fn, good, 128, 128, 96, 2)
    assert code == 1 and "K_dim" in msg
    code, _ = _call_full(lib, fn, good, 128, 128, 64, 0)
    assert code == 1
    code, msg = _call_full(lib, fn, good, 128, 130, 64, 2)
    assert code == 2
    code, msg = _call_full(lib, fn, [p + 2 for p in good], 128, 128, 64, 2)
    assert code == 2 and "aligned" in msg


def test_stream_entry_rejects_with_return_code():
    _ensure_built()
    lib = ctypes.CDLL(LIBS["bf16"])
    f = lib.fmha_bwd_full_stream
    f.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    f.restype = ctypes.c_int
    assert f(*([None] * 8), 128, 128, 64, 2, None) == 1


def test_python_mirror_fails_loudly_without_cuda_tensors():
    import torch

    import fmha_bwd_b200 as F

    x = torch.zeros(1, 128, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        F.fmha_bwd(x, x, x, torch.zeros(1, 128, 128, dtype=torch.bfloat16), x)
    with pytest.raises(TypeError):
        F.library_path(torch.float32)
    # the stage hooks and the recompute-P entry check their tensors the same way
    with pytest.raises(ValueError):
        F.run_stage("dp", x, x)
    with pytest.raises(ValueError):
        F.run_stage("no_such_stage", x, x)
    with pytest.raises(ValueError):
        F.fmha_bwd_lse(x, x, x, x, x, torch.zeros(1, 128), 0.125)


@pytest.mark.parametrize("kind", ["bf16", "fp16"])
def test_selftest_rejects_bad_timeout_without_gpu(kind):
    _ensure_built()
    lib = ctypes.CDLL(LIBS[kind])
    f = lib.fmha_bwd_selftest_wait_timeout
    f.argtypes = [ctypes.c_int]
    f.restype = ctypes.c_int
    assert f(0) == 1
    assert f(20000) == 1


@pytest.mark.parametrize("kind,fn", [("bf16", "fmha_bwd_full_delta"), ("fp16", "fmha_bwd_full_fp16_delta")])
def test_delta_entry_requires_rowsum(kind, fn):
    """The precomputed-rowsum entry rejects a null D before touching the GPU."""
    _ensure_built()
    lib = ctypes.CDLL(LIBS[kind])
    f = getattr(lib, fn)
    f.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    f.restype = ctypes.c_int
    good = [0x10000 * (i + 1) for i in range(8)]
    assert f(*good, None, 128, 128, 64, 2, None) == 1


STAGE_HOOKS = ["dp", "softmax_bwd", "dq", "dk", "dv"]


@pytest.mark.parametrize("kind", ["bf16", "fp16"])
@pytest.mark.parametrize("stage", STAGE_HOOKS)
def test_stage_hooks_reject_bad_arguments_without_gpu(kind, stage):
    """Every stage hook checks its arguments on the host before any CUDA call
    and reports through fmha_bwd_last_error()."""
    _ensure_built()
    lib = ctypes.CDLL(LIBS[kind])
    lib.fmha_bwd_last_error.restype = ctypes.c_int
    lib.fmha_bwd_last_error_message.restype = ctypes.c_char_p
    f = getattr(lib, f"test_{stage}_kernel" + ("_fp16" if kind == "fp16" else ""))
    nints = 3 if stage == "softmax_bwd" else 4
    f.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * nints
    f.restype = None
    good = [0x10000 * (i + 1) for i in range(3)]  # never dereferenced: rejected first

    def call(ptrs, M, N, d, H):
        ints = (M, N, H) if stage == "softmax_bwd" else (M, N, d, H)
        f(*ptrs, *ints)
        return lib.fmha_bwd_last_error(), lib.fmha_bwd_last_error_message().decode()

    code, msg = call([None] + good[1:], 128, 128, 64, 2)
    assert code == 1 and "null" in msg
    assert call(good, 0, 128, 64, 2)[0] == 1
    assert call(good, 128, 128, 64, 0)[0] == 1
    assert call(good, 128, 130, 64, 2)[0] == 2
    code, msg = call([p + 2 for p in good], 128, 128, 64, 2)
    assert code == 2 and "aligned" in msg
    if stage != "softmax_bwd":
        code, msg = call(good, 128, 128, 96, 2)
        assert code == 1 and "K_dim" in msg


@pytest.mark.parametrize("kind,fn", [("bf16", "fmha_bwd_full_lse"), ("fp16", "fmha_bwd_full_fp16_lse")])
def test_lse_entry_rejects_bad_arguments_without_gpu(kind, fn):
    """The recompute-P entry checks LSE, the scale and the usual sizes on the
    host; N needs no alignment there (no P rows are read)."""
    _ensure_built()
    lib = ctypes.CDLL(LIBS[kind])
    lib.fmha_bwd_last_error_message.restype = ctypes.c_char_p
    f = getattr(lib, fn)
    f.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_void_p]
    f.restype = ctypes.c_int
    good = [0x10000 * (i + 1) for i in range(8)]
    lse = 0x90000
    assert f(*good, None, 128, 128, 64, 2, 1.0, None) == 1          # null LSE
    assert f(*good, lse + 2, 128, 128, 64, 2, 1.0, None) == 2       # misaligned LSE
    assert f(*good, lse, 128, 128, 64, 2, 0.0, None) == 1           # scale must be > 0
    assert f(*good, lse, 128, 128, 64, 2, float("nan"), None) == 1
    assert f(*good, lse, 128, 128, 96, 2, 1.0, None) == 1           # K_dim
    assert f(None, *good[1:], lse, 128, 128, 64, 2, 1.0, None) == 1
