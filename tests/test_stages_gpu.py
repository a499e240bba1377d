"""Stage hooks on the GPU (test_dp_kernel, test_softmax_bwd_kernel,
test_dq_kernel, test_dk_kernel, test_dv_kernel and their _fp16 twins),
called through the C-ABI:

  * each stage against an fp32 PyTorch recompute of its formula from the
    same 16-bit inputs the hook read;
  * the chain dp -> softmax_bwd -> dq / dk / dv (16-bit dP and dS in global
    memory, as in the reference's five-launch GPU path) against the restated
    oracle and against the reference's own answers in the golden fixtures.

Tolerance (per output): bf16 rel-L2 <= 1e-2 and max-abs <= 2e-2 * max|ref|;
fp16 rel-L2 <= 5e-3 and max-abs <= 1e-2 * max|ref|.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden

pytestmark = pytest.mark.gpu

# (M, N, d, heads, dtype): ragged tiles in every dimension, both head sizes,
# a single-row case, and a FLUX-sized head pair whose contractions run 72
# blocks through the load ring.
SHAPES = [
    (200, 136, 128, 2, "bf16"),
    (77, 264, 64, 3, "fp16"),
    (1000, 520, 128, 2, "bf16"),
    (384, 64, 64, 2, "bf16"),
    (1, 8, 64, 1, "fp16"),
    (640, 1024, 64, 3, "fp16"),
    (4608, 4608, 128, 2, "bf16"),
]


def _dt(name):
    return torch.bfloat16 if name == "bf16" else torch.float16


def _to_dev(bits: np.ndarray, dtype: torch.dtype) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(dtype).cuda()


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


@pytest.fixture(scope="module")
def F():
    import fmha_bwd_b200 as F

    F.load_library(torch.bfloat16)
    F.load_library(torch.float16)
    return F


def _inputs(O, M, N, d, H, name, seed):
    if M * H <= 4096:
        bits = O.make_inputs(M, N, d, H, name, seed=seed)
        return bits, [_to_dev(b, _dt(name)) for b in bits]
    import workloads

    w = workloads.Workload("stage", M, N, d, H, name)
    return None, list(workloads.make_inputs(w, seed=seed))


def _ok(O, label, got, ref, name):
    r = O.check(label, _np(got), ref.detach().cpu().numpy() if torch.is_tensor(ref) else ref, name)
    assert r["ok"], r


@pytest.mark.parametrize("M,N,d,H,name", SHAPES)
def test_each_stage_matches_fp32(F, oracle_built, M, N, d, H, name):
    O = oracle_built
    _, (Q, K, V, P, dO) = _inputs(O, M, N, d, H, name, seed=51)
    dP = F.run_stage("dp", dO, V)
    _ok(O, "dP", dP, torch.einsum("hmk,hnk->hmn", dO.float(), V.float()), name)
    dS = F.run_stage("softmax_bwd", P, dP)
    Pf, dPf = P.float(), dP.float()
    _ok(O, "dS", dS, Pf * (dPf - (Pf * dPf).sum(-1, keepdim=True)), name)
    del Pf, dPf
    dQ = F.run_stage("dq", dS, K)
    _ok(O, "dQ", dQ, torch.einsum("hmn,hnk->hmk", dS.float(), K.float()), name)
    dK = F.run_stage("dk", dS, Q)
    _ok(O, "dK", dK, torch.einsum("hmn,hmk->hnk", dS.float(), Q.float()), name)
    dV = F.run_stage("dv", P, dO)
    _ok(O, "dV", dV, torch.einsum("hmn,hmk->hnk", P.float(), dO.float()), name)


def _chain(F, Q, K, V, P, dO):
    dP = F.run_stage("dp", dO, V)
    dS = F.run_stage("softmax_bwd", P, dP)
    return F.run_stage("dq", dS, K), F.run_stage("dk", dS, Q), F.run_stage("dv", P, dO)


@pytest.mark.parametrize("M,N,d,H,name", [s for s in SHAPES if s[0] * s[3] <= 4096])
def test_stage_chain_matches_oracle(F, oracle_built, M, N, d, H, name):
    """The five hooks in sequence reproduce the full backward."""
    O = oracle_built
    bits, (Q, K, V, P, dO) = _inputs(O, M, N, d, H, name, seed=52)
    got = _chain(F, Q, K, V, P, dO)
    ref = O.oracle_bwd(*bits, name)
    for label, g, r in zip(("dQ", "dK", "dV"), got, ref[:3]):
        _ok(O, label, g, r, name)


@pytest.mark.parametrize("gname", golden_names())
def test_stage_chain_matches_golden(F, oracle_built, gname):
    """The chain against the reference's cpu_reference.hpp answers."""
    O = oracle_built
    g = load_golden(gname)
    dt = _dt(g["dtype"])
    Q, K, V, P, dO = (_to_dev(g[k], dt) for k in ("Q", "K", "V", "P", "dO"))
    got = _chain(F, Q, K, V, P, dO)
    for label, x, key in zip(("dQ", "dK", "dV"), got, ("dQ", "dK", "dV")):
        _ok(O, label, x, g[key].astype(np.float32), g["dtype"])


def test_stage_hook_rejects_without_launch(F):
    """A rejected hook call (N % 8 != 0) leaves its output untouched."""
    dO = torch.randn(1, 64, 64, device="cuda").bfloat16()
    V = torch.randn(1, 64, 64, device="cuda").bfloat16()
    out = torch.full((1, 64, 60), 3.0, device="cuda").bfloat16()
    lib = F.load_library(torch.bfloat16)
    f = F._stage_fn(lib, torch.bfloat16, "dp")
    f(dO.data_ptr(), V.data_ptr(), out.data_ptr(), 64, 60, 64, 1)
    assert lib.fmha_bwd_last_error() == 2
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())
