"""Radial basis, cutoff and edge geometry against the reference's golden vectors
(``nn/radial.py:8-245``, ``utils/geometry.py:25-77``).

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


def test_edge_geometry_matches_reference_golden(radial_golden):
    """get_edge_vectors (two structures, orthorhombic and triclinic cells, image shifts; with
    and without shifts) with its position and cell gradients, and to_voigt6, against the
    reference's ``utils/geometry.py:25-77``."""
    from flashcart_b200.model.flashcart import get_edge_vectors, to_voigt6

    G = {k.split("/", 1)[1]: v for k, v in radial_golden.items() if k.startswith("geom/")}
    pos = G["positions"].clone().requires_grad_(True)
    cell = G["cell"].clone().requires_grad_(True)
    vec = get_edge_vectors(pos, cell, G["shifts"], G["edge_index"], G["batch"], use_shifts=True)
    assert (vec.detach() - G["vectors"]).abs().max().item() < 1e-12
    dpos, dcell = torch.autograd.grad((vec * G["weights"]).sum(), [pos, cell])
    assert (dpos - G["grad_positions"]).abs().max().item() < 1e-12
    assert (dcell - G["grad_cell"]).abs().max().item() < 1e-12
    plain = get_edge_vectors(G["positions"], G["cell"], G["shifts"], G["edge_index"], G["batch"], use_shifts=False)
    assert (plain - G["vectors_noshift"]).abs().max().item() < 1e-12
    assert torch.equal(to_voigt6(G["voigt_in"]), G["voigt_out"])
