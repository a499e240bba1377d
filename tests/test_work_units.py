"""The work-unit plan (how a call's items are spread over the persistent
CTAs and which tails are split into parts), through the host-only C-ABI
query fmha_bwd_work_units, and the bench's launch count derived from it.
CPU only: nothing is launched."""
from __future__ import annotations

import ctypes
import itertools

import pytest

from test_abi import LIBS, _ensure_built


def _plan(lib, items, grid, length, allow=1):
    out = (ctypes.c_int * 3)()
    assert lib.fmha_bwd_work_units(items, grid, length, allow, out) == 0
    return tuple(out)


@pytest.fixture(scope="module")
def lib():
    _ensure_built()
    lib = ctypes.CDLL(LIBS["bf16"])
    lib.fmha_bwd_work_units.argtypes = [ctypes.c_int] * 4 + [ctypes.c_void_p]
    lib.fmha_bwd_work_units.restype = ctypes.c_int
    return lib


@pytest.mark.parametrize("items,length,expect", [
    (864, 36, (864, 1, 864)),      # FLUX: a tail of 124 of 148 stays whole
    (192, 32, (148, 3, 280)),      # cross-attention dK/dV: 44 tail items, thirds in one wave
    (1536, 4, (1536, 1, 1536)),    # cross-attention dQ: 4-step items are never split
    (640, 128, (592, 3, 736)),     # 5-head 16384^2 shard: tail 48 -> 144 parts
    (1280, 128, (1184, 3, 1472)),  # 10-head shard: tail 96 -> 288 parts in two waves
    (2048, 16, (2048, 1, 2048)),   # fp16 2048^2 d=64: tail 124, nothing to gain
    (148, 64, (148, 1, 148)),      # whole waves only
])
def test_plan_of_the_measured_workloads(lib, items, length, expect):
    assert _plan(lib, items, 148, length) == expect


def test_plan_invariants(lib):
    for items, grid, length in itertools.product(range(0, 700, 7), (1, 2, 74, 148), (1, 8, 15, 16, 17, 40, 128)):
        full, parts, units = _plan(lib, items, grid, length)
        assert 1 <= parts <= 4
        if parts == 1:
            assert (full, units) == (items, items)
            continue
        tail = items - full
        assert full % grid == 0 and 0 < tail < grid
        assert units == full + parts * tail
        assert length >= 16 and length // parts >= 8
        # the split tail costs less than the whole tail (at least a tenth of an item)
        cost = -(-parts * tail // grid) / parts
        assert cost <= 0.9
        # no workspace, no split
        assert _plan(lib, items, grid, length, allow=0) == (items, 1, items)


def test_rejects_bad_arguments(lib):
    assert lib.fmha_bwd_work_units(10, 148, 16, 1, None) != 0
    out = (ctypes.c_int * 3)()
    assert lib.fmha_bwd_work_units(-1, 148, 16, 1, out) != 0


def test_bench_launch_count_follows_the_library_plan(lib):
    import bench
    import workloads

    for w in workloads.WORKLOADS.values():
        for heads in sorted({w.heads, 1, 5, 10, 13}):
            mt, nt = -(-w.M // 128), -(-w.N // 128)
            expect = 2 + (_plan(lib, mt * heads, 148, nt)[1] > 1) + (_plan(lib, nt * heads, 148, mt)[1] > 1)
            assert bench.launches_per_call(w, heads, 148) == expect, (w.name, heads)
