"""Muon's Newton-Schulz orthogonalisation: the oracle (oracle/muon.py) and the host-side
coefficient computation of macrogpt_jax_b200.muon, on the CPU."""
import numpy as np
import pytest

from oracle import muon as om


def test_optimal_composition_matches_between_host_and_oracle():
    from macrogpt_jax_b200 import muon
    for speed, steps in ((1e-3, 5), (1e-2, 3), (0.1, 8)):
        a = np.array(muon.optimal_composition(speed, steps))
        b = np.array(om.optimal_composition(speed, steps))
        np.testing.assert_allclose(a, b, rtol=1e-12)
    assert muon.ns_coefficients(4, "muon") == (muon.MUON_COEFFS,) * 4
    with pytest.raises(ValueError, match="Unknown value"):
        muon.ns_coefficients(5, "newton")


@pytest.mark.parametrize("method,lo,hi", [("muon", 0.68, 1.21), ("optimal", 0.87, 1.13)])
def test_composed_polynomial_maps_singular_values_near_one(method, lo, hi):
    """The composed odd polynomials take every singular value in [1e-2, 1] (muon) or [1e-3, 1]
    (optimal, convergence_speed 1e-3) into a band around 1; the muon band is the known
    [0.68, 1.2] of its fixed coefficients."""
    x = np.linspace(1e-2 if method == "muon" else 1e-3, 1.0, 5000)
    y = x.copy()
    for a, b, c in om.coefficients(5, method):
        y = a * y + b * y ** 3 + c * y ** 5
    assert lo <= y.min() and y.max() <= hi


@pytest.mark.parametrize("shape", [(2, 64, 128), (1, 96, 48), (3, 32, 32)])
def test_orthogonalize_oracles(shape):
    """float64 evaluation: singular values of the result in the coefficients' band (rectangular
    slices, whose singular values after normalisation lie in its reach); the bf16
    storage-point evaluation the kernel follows stays within bf16 noise of it; transposed slices
    (m > n) give the transpose of orthogonalising the transpose."""
    rng = np.random.default_rng(sum(shape))
    g = rng.standard_normal(shape).astype(np.float32)
    co = om.coefficients(5, "muon")
    r = om.orthogonalize_f64(g, co)
    if shape[1] != shape[2]:  # a square Gaussian slice has singular values below the band's reach
        for sl in r:
            sv = np.linalg.svd(sl, compute_uv=False)
            assert sv.min() > 0.6 and sv.max() < 1.25
    b = om.orthogonalize_bf16(g, co)
    cos = (r * b).sum() / (np.linalg.norm(r) * np.linalg.norm(b))
    assert cos > 0.999
    rt = om.orthogonalize_f64(np.swapaxes(g, 1, 2).copy(), co)
    np.testing.assert_allclose(np.swapaxes(rt, 1, 2), r, rtol=1e-9, atol=1e-12)
