"""Radial basis and cutoff against the reference's golden vectors (``nn/radial.py:8-245``).

Values and the first derivative with respect to the distance, float64, on distances that
include r = 0, r = r_min, r = r_max and beyond the cutoff; tolerance 1e-12 as in the
reference's own radial tests (``tests/nn/test_radial.py:9-43``). The vectors come from
``tests/golden/make_radial_golden.py`` run against the reference source.
"""

import os

import pytest
import torch

from flashcart_b200.nn.radial import BesselBasis, ChebyshevBasis, PolynomialCutoff

CASES = {
    "cheb_cosine_8": lambda: ChebyshevBasis(8, 5.0, mapping="cosine"),
    "cheb_affine_8": lambda: ChebyshevBasis(8, 5.0, mapping="affine"),
    "cheb_cosine_5_rmin": lambda: ChebyshevBasis(5, 5.0, r_min=0.5, mapping="cosine"),
    "cheb_affine_1": lambda: ChebyshevBasis(1, 5.0, mapping="affine"),
    "bessel_8": lambda: BesselBasis(8, 5.0),
    "cutoff_6": lambda: PolynomialCutoff(5.0, 6),
    "cutoff_3": lambda: PolynomialCutoff(5.0, 3),
}


@pytest.fixture(scope="module")
def radial_golden():
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "radial_golden.pt")
    return torch.load(path, map_location="cpu", weights_only=True)


@pytest.mark.parametrize("name", sorted(CASES))
def test_radial_functions_match_reference_golden(radial_golden, name):
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)  # buffers built in float64, as the vectors were
    try:
        m = CASES[name]()
    finally:
        torch.set_default_dtype(prev)
    r = radial_golden["r"].clone().requires_grad_(True)
    y = m(r)
    ref = radial_golden[f"{name}/value"]
    assert y.shape == ref.shape
    assert (y.detach() - ref).abs().max().item() <= 1e-12 * max(1.0, ref.abs().max().item()), name
    w = radial_golden[f"{name}/weights"]
    if y.requires_grad:
        (dy,) = torch.autograd.grad((y * w).sum(), [r])
    else:
        dy = torch.zeros_like(r)
    ref_g = radial_golden[f"{name}/grad_r"]
    assert torch.isfinite(dy).all(), name
    assert (dy - ref_g).abs().max().item() <= 1e-10 * max(1.0, ref_g.abs().max().item()), name
