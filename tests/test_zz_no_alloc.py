"""The allocation-free entry point fmha_bwd_full_noalloc (libfmha_bwd_bf16.so),
called through the C-ABI and checked against the allocating entry point
fmha_bwd_full_py on the same inputs, on two calls in a row.

Tolerance (bf16, as in the parity tests): rel-L2 <= 1e-2 and
max-abs <= 2e-2 * max|ref| per output.

Named so pytest collects it last; it passes alone in a fresh process and
after the other tests (the scratch is shared by every call and needs no
state from earlier calls).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest

from conftest import ROOT

LIB = os.path.join(ROOT, "build", "libfmha_bwd_bf16.so")
MAX_ROWS = 1 << 20  # total_heads * M limit of the no-alloc scratch


def _lib():
    if not os.path.exists(LIB):
        import build_libs

        build_libs.build()
    lib = ctypes.CDLL(LIB)
    f = lib.fmha_bwd_full_noalloc
    f.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int] * 4 + [ctypes.c_void_p]
    f.restype = ctypes.c_int
    lib.fmha_bwd_last_error_message.restype = ctypes.c_char_p
    return lib


def _noalloc(lib, outs, ins, M, N, d, H, stream):
    ptrs = [t.data_ptr() for t in outs] + [t.data_ptr() for t in ins]
    return lib.fmha_bwd_full_noalloc(*ptrs, M, N, d, H, ctypes.c_void_p(stream))


def test_noalloc_rejects_oversize_before_any_cuda_call():
    """total_heads * M above the scratch limit is refused on the host."""
    lib = _lib()
    fake = [0x10000 * (i + 1) for i in range(8)]  # never dereferenced: rejected first
    rc = lib.fmha_bwd_full_noalloc(*fake, MAX_ROWS // 128 + 1, 128, 64, 128, None)
    assert rc == 1
    assert b"no-alloc" in lib.fmha_bwd_last_error_message()
    rc = lib.fmha_bwd_full_noalloc(None, *fake[1:], 128, 128, 64, 2, None)
    assert rc == 1


def _check(got, ref):
    from oracle.oracle import check

    for name, g, r in zip(("dQ", "dK", "dV"), got, ref):
        res = check(name, g.float().cpu().numpy(), r.float().cpu().numpy(), "bf16")
        assert res["ok"], res


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,d,H", [(1000, 520, 128, 2), (640, 1024, 64, 3),
                                     (4096, 256, 128, 256)])
def test_noalloc_matches_allocating_entry(M, N, d, H):
    """Two no-alloc calls in a row each match fmha_bwd_full_py; the last
    shape fills the scratch to its limit (H * M = 2^20)."""
    import torch

    import fmha_bwd_b200 as F
    from oracle.oracle import make_inputs

    lib = _lib()
    if H * M <= 4096:
        bits = make_inputs(M, N, d, H, "bf16", seed=21)
        ins = [torch.from_numpy(b.view(np.int16).copy()).view(torch.bfloat16).cuda()
               for b in bits]
    else:  # large case: seeded device-side inputs, P a row softmax
        g = torch.Generator(device="cuda").manual_seed(21)
        Q = torch.randn(H, M, d, device="cuda", generator=g).bfloat16()
        K = torch.randn(H, N, d, device="cuda", generator=g).bfloat16()
        V = torch.randn(H, N, d, device="cuda", generator=g).bfloat16()
        P = torch.softmax(torch.randn(H, M, N, device="cuda", generator=g) * 2.0,
                          dim=-1).bfloat16()
        dO = torch.randn(H, M, d, device="cuda", generator=g).bfloat16()
        ins = [Q, K, V, P, dO]
    assert H * M <= MAX_ROWS
    ref = F.fmha_bwd(*ins)  # allocating entry, fmha_bwd_full_py
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        outs = [torch.full_like(ins[0], float("nan")), torch.full_like(ins[1], float("nan")),
                torch.full_like(ins[2], float("nan"))]
        torch.cuda.synchronize()
        rc = _noalloc(lib, outs, ins, M, N, d, H, stream)
        assert rc == 0, lib.fmha_bwd_last_error_message()
        assert not any(torch.isnan(t).any().item() for t in outs)
        _check(outs, ref)


@pytest.mark.gpu
def test_noalloc_oversize_leaves_outputs_untouched():
    import torch

    lib = _lib()
    M, N, d, H = 128, 64, 64, MAX_ROWS // 128 + 1
    ins = [torch.empty(H, M, d, dtype=torch.bfloat16, device="cuda"),
           torch.empty(H, N, d, dtype=torch.bfloat16, device="cuda"),
           torch.empty(H, N, d, dtype=torch.bfloat16, device="cuda"),
           torch.empty(H, M, N, dtype=torch.bfloat16, device="cuda"),
           torch.empty(H, M, d, dtype=torch.bfloat16, device="cuda")]
    outs = [torch.full_like(ins[0], 7.0), torch.full_like(ins[1], 7.0),
            torch.full_like(ins[2], 7.0)]
    torch.cuda.synchronize()
    rc = _noalloc(lib, outs, ins, M, N, d, H, torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    torch.cuda.synchronize()
    assert all(bool((t == 7.0).all()) for t in outs)
