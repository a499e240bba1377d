"""CPU tests of the oracle: the restatement against the golden fixtures made
by the reference's own cpu_reference.hpp, and (where the reference tree was
built here) against the reference library directly."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_names, load_golden


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_golden(oracle_built, name):
    """The restated oracle (fp32 outputs) agrees with the reference's outputs
    (half_t, rounded) to fp16 rounding: every element within one fp16 ulp
    plus a small absolute slack, and rel-L2 <= 1e-3."""
    O = oracle_built
    g = load_golden(name)
    dQ, dK, dV, D = O.oracle_bwd(g["Q"], g["K"], g["V"], g["P"], g["dO"], g["dtype"])
    for got, ref in ((dQ, g["dQ"]), (dK, g["dK"]), (dV, g["dV"])):
        ref32 = ref.astype(np.float32)
        assert O.rel_l2(got, ref32) <= 1e-3
        ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
        assert np.all(np.abs(got - ref32) <= ulp + 1e-3 * (1 + np.abs(ref32)))


@pytest.mark.parametrize("name", golden_names())
def test_rowsum_definition(oracle_built, name):
    """D[m] = sum_n P[m,n] dP[m,n] (cpu_reference.hpp:32-35) equals
    sum_k dO[m,k] (P V)[m,k], the identity the GPU rowsum kernel uses."""
    O = oracle_built
    g = load_golden(name)
    dt = g["dtype"]
    _, _, _, D = O.oracle_bwd(g["Q"], g["K"], g["V"], g["P"], g["dO"], dt)
    P = O.from_bits(g["P"], dt).astype(np.float64)
    V = O.from_bits(g["V"], dt).astype(np.float64)
    dO = O.from_bits(g["dO"], dt).astype(np.float64)
    alt = np.einsum("hmk,hmk->hm", dO, np.matmul(P, V))
    assert np.allclose(D, alt, rtol=1e-4, atol=1e-4 * (1 + np.abs(alt).max()))


def test_oracle_matches_reference_library(oracle_built):
    """Fresh seeded inputs through both CPU implementations (needs the
    reference tree built into oracle/_ref)."""
    O = oracle_built
    if not O.have_reference():
        pytest.skip("reference library not built here")
    for (M, N, d, H, dt) in ((64, 72, 64, 2, "bf16"), (130, 40, 128, 1, "fp16")):
        Q, K, V, P, dO = O.make_inputs(M, N, d, H, dt, seed=123)
        a = O.oracle_bwd(Q, K, V, P, dO, dt)
        b = O.reference_bwd(Q, K, V, P, dO, dt)
        for x, y in zip(a[:3], b):
            assert O.rel_l2(x, y) <= 1e-3


def test_oracle_detects_planted_error(oracle_built):
    """A mistake planted in the oracle's output is caught by the tolerance
    check (the check is not vacuous)."""
    O = oracle_built
    g = load_golden("cpu_case_bf16")
    dQ, dK, dV, _ = O.oracle_bwd(g["Q"], g["K"], g["V"], g["P"], g["dO"], "bf16")
    ref = g["dQ"].astype(np.float32)
    assert O.check("dQ", dQ, ref, "bf16")["ok"]
    bad = dQ.copy()
    bad[0, 5, :] *= 1.5  # one wrong row
    assert not O.check("dQ", bad, ref, "bf16")["ok"]
    scaled = dQ * np.float32(1.0 / np.sqrt(64))  # a softmax scale the reference never applies
    assert not O.check("dQ", scaled, ref, "bf16")["ok"]


def test_bits_roundtrip():
    from oracle import oracle as O

    x = np.array([0.0, 1.0, -2.5, 3.14159, 1e-3, 65504.0], np.float32)
    for dt in ("bf16", "fp16"):
        y = O.from_bits(O.to_bits(x, dt), dt)
        tol = 2 ** -8 if dt == "bf16" else 2 ** -11
        assert np.allclose(y, x, rtol=tol, atol=0)


def test_make_inputs_is_seeded_softmax():
    from oracle import oracle as O

    a = O.make_inputs(16, 24, 64, 2, "bf16", seed=5)
    b = O.make_inputs(16, 24, 64, 2, "bf16", seed=5)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    P = O.from_bits(a[3], "bf16")
    assert np.allclose(P.sum(-1), 1.0, atol=2e-2)
    assert (P >= 0).all()
