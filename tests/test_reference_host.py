"""The reference's own Python host (benchmark_pytorch_final.py) against the new
library, through the binding recorded in tests/golden/reference_host.json
(tests/golden/make_reference_host.py reads the script with `ast` where the
reference lies; the script itself is not part of this repository).

CPU: the recorded binding names a library this build produces, with the
argument types the host mirror declares, and the mirror's benchmark_size
returns the reference's result keys. GPU: the library is loaded and called
exactly as recorded -- ctypes.CDLL of the recorded relative path from the
repository root, the recorded argtypes, zero-filled [batch, heads, M, d]
outputs, the recorded argument order with total_heads = heads -- on the
recorded configurations and seed, and checked against the einsum backward.
"""
from __future__ import annotations

import ctypes
import json
import os

import pytest

from conftest import GOLDEN, ROOT

FIXTURE = os.path.join(GOLDEN, "reference_host.json")


def _rec():
    with open(FIXTURE) as f:
        return json.load(f)


def test_recorded_binding_matches_this_build():
    import fmha_bwd_b200 as F
    import torch

    rec = _rec()
    assert rec["function"] == "fmha_bwd_full_py"
    # the relative path the reference host loads is this build's bf16 library
    lib_rel = os.path.normpath(rec["library"])
    assert lib_rel == os.path.join("build", F.LIB_NAMES[torch.bfloat16][0])
    assert os.path.normpath(os.path.join(ROOT, lib_rel)) == F.library_path(torch.bfloat16)
    types = [getattr(ctypes, t.split(".")[-1]) for t in rec["argtypes"]]
    assert types == F._PTR_ARGS + F._INT_ARGS
    assert rec["call_args"][:8] == [f"{n}.data_ptr()" for n in
                                    ("dQ", "dK", "dV", "Q", "K", "V", "P", "dO")]
    assert rec["call_args"][8:] == ["M", "N", "K_dim", "heads"]
    assert rec["zero_filled"] == ["dQ", "dK", "dV"]


def test_mirror_benchmark_size_returns_reference_keys():
    """The mirror's benchmark_size builds its result with every key the
    reference's returns (read from its source, since it needs a GPU to run)."""
    import ast
    import inspect

    import fmha_bwd_b200 as F

    tree = ast.parse(inspect.getsource(F.benchmark_size))
    keys = set()
    for node in ast.walk(tree):
        if isinstance(node, ast.Return) and isinstance(node.value, ast.Dict):
            keys |= {ast.literal_eval(k) for k in node.value.keys}
    assert set(_rec()["result_keys"]) <= keys


def test_reference_script_unchanged_when_present():
    """When FMHA_BWD_REFERENCE_TREE names a reference checkout, the recorded
    binding is still what its host script says."""
    tree = os.environ.get("FMHA_BWD_REFERENCE_TREE")
    if not tree or not os.path.exists(os.path.join(tree, "benchmark_pytorch_final.py")):
        pytest.skip("no reference checkout named by FMHA_BWD_REFERENCE_TREE")
    import hashlib
    import sys

    sys.path.insert(0, GOLDEN)
    import make_reference_host as R

    raw = open(os.path.join(tree, "benchmark_pytorch_final.py"), "rb").read()
    rec = _rec()
    assert hashlib.sha256(raw).hexdigest() == rec["sha256"]
    fresh = R.extract(raw.decode())
    for k, v in fresh.items():
        assert rec[k] == v, k


def _bound_library(rec):
    """ctypes.CDLL(recorded path) from the repository root, with the recorded
    argtypes, as the reference host does at import time."""
    cwd = os.getcwd()
    try:
        os.chdir(ROOT)
        lib = ctypes.CDLL(rec["library"])
    finally:
        os.chdir(cwd)
    fn = getattr(lib, rec["function"])
    fn.argtypes = [getattr(ctypes, t.split(".")[-1]) for t in rec["argtypes"]]
    return lib, fn


@pytest.mark.gpu
def test_reference_host_binding_on_recorded_configs():
    import torch

    from fmha_bwd_b200 import pytorch_naive_backward

    rec = _rec()
    lib, fn = _bound_library(rec)
    dev = torch.device("cuda")
    for batch, heads, M, N, K_dim in rec["configs"]:
        # the reference host's inputs (benchmark_size), in bf16: its own
        # default, float16, is the other library's type
        torch.manual_seed(rec["seed"])
        dt = torch.bfloat16
        Q = torch.randn(batch, heads, M, K_dim, dtype=dt, device=dev)
        K = torch.randn(batch, heads, N, K_dim, dtype=dt, device=dev)
        V = torch.randn(batch, heads, N, K_dim, dtype=dt, device=dev)
        dO = torch.randn(batch, heads, M, K_dim, dtype=dt, device=dev)
        P = torch.softmax(torch.randn(batch, heads, M, N, dtype=dt, device=dev), dim=-1)
        outs = {n: torch.zeros_like(t) for n, t in (("dQ", Q), ("dK", K), ("dV", V))}
        env = dict(outs, Q=Q, K=K, V=V, P=P, dO=dO, M=M, N=N, K_dim=K_dim, heads=heads)
        args = [env[a[:-len(".data_ptr()")]].data_ptr() if a.endswith(".data_ptr()") else env[a]
                for a in rec["call_args"]]
        fn(*args)
        torch.cuda.synchronize()
        ref = pytorch_naive_backward(Q, K, V, P, dO)
        for name, r in zip(("dQ", "dK", "dV"), ref):
            got = outs[name].float()
            rel = float((got - r).norm() / r.norm().clamp_min(1e-30))
            mx = float((got - r).abs().max())
            # bf16 tolerance of the parity tests: rel-L2 <= 1e-2, max-abs <= 2e-2 max|ref|
            assert rel <= 1e-2 and mx <= 2e-2 * float(r.abs().max()), (batch, heads, M, name,
                                                                         rel, mx)


@pytest.mark.gpu
def test_mirror_benchmark_size_on_gpu():
    import torch

    import fmha_bwd_b200 as F

    res = F.benchmark_size(1, 24, 512, 512, 128, dtype=torch.bfloat16, warmup=2, reps=5)
    assert set(_rec()["result_keys"]) <= set(res)
    assert res["custom_time_ms"] > 0 and res["pytorch_time_ms"] > 0
    assert res["speedup"] == pytest.approx(res["pytorch_time_ms"] / res["custom_time_ms"])
    assert res["max_diff"] < 0.1
