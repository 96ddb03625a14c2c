"""Generate golden vectors of the radial basis and cutoff from the REFERENCE implementation.

Run where the reference source tree is available (never needed at test time)::

    PYTHONPATH=<reference>/src python tests/golden/make_radial_golden.py [<reference>/src]

Evaluates the reference's ``ChebyshevBasis`` (cosine and affine mappings, with and
without r_min), ``BesselBasis`` and ``PolynomialCutoff`` (``nn/radial.py:8-245``) in
float64 on distances that cover the interior, r = 0 (Bessel's removable singularity),
r = r_min, r = r_max and beyond the cutoff, and records the values and the first
derivative with respect to the distance (autograd of the summed, seeded-weighted output),
which the forces depend on. Also the edge geometry of ``utils/geometry.py:25-77``:
``get_edge_vectors`` on a two-structure batch (one orthorhombic, one triclinic cell,
integer image shifts) with the gradients of a seeded weighted sum with respect to the
positions and the cells, and ``to_voigt6`` of random 3 x 3 tensors.

Output: ``tests/golden/radial_golden.pt``.
"""

from __future__ import annotations

import os
import sys

import torch


def main(src: str) -> None:
    import importlib.util

    spec = importlib.util.spec_from_file_location("ref_radial", os.path.join(src, "flashcart", "nn", "radial.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    torch.set_default_dtype(torch.float64)
    g = torch.Generator().manual_seed(21)
    r_max = 5.0
    r = torch.cat([torch.tensor([0.0, 1e-6, 0.5, r_max - 1e-6, r_max, r_max + 0.25, 2 * r_max]),
                   torch.rand(57, generator=g, dtype=torch.float64) * r_max])
    cases = {
        "cheb_cosine_8": mod.ChebyshevBasis(8, r_max, mapping="cosine"),
        "cheb_affine_8": mod.ChebyshevBasis(8, r_max, mapping="affine"),
        "cheb_cosine_5_rmin": mod.ChebyshevBasis(5, r_max, r_min=0.5, mapping="cosine"),
        "cheb_affine_1": mod.ChebyshevBasis(1, r_max, mapping="affine"),
        "bessel_8": mod.BesselBasis(8, r_max),
        "cutoff_6": mod.PolynomialCutoff(r_max, 6),
        "cutoff_3": mod.PolynomialCutoff(r_max, 3),
    }
    out = {"r": r}
    for name, m in cases.items():
        x = r.clone().requires_grad_(True)
        y = m(x)
        w = torch.randn(y.shape, generator=g, dtype=torch.float64)
        if y.requires_grad:
            (dy,) = torch.autograd.grad((y * w).sum(), [x])
        else:  # a single Chebyshev term is the constant 1: no dependence on r
            dy = torch.zeros_like(r)
        out[f"{name}/value"] = y.detach()
        out[f"{name}/weights"] = w
        out[f"{name}/grad_r"] = dy
    gspec = importlib.util.spec_from_file_location("ref_geometry",
                                                   os.path.join(src, "flashcart", "utils", "geometry.py"))
    geo = importlib.util.module_from_spec(gspec)
    gspec.loader.exec_module(geo)
    pos = torch.rand(10, 3, generator=g, dtype=torch.float64) * 6.0
    cell = torch.stack([torch.diag(torch.tensor([6.0, 7.0, 8.0])),
                        torch.tensor([[6.0, 0.0, 0.0], [1.5, 6.5, 0.0], [-0.7, 1.1, 7.2]])])
    batch = torch.tensor([0] * 5 + [1] * 5)
    recv = torch.tensor([0, 0, 1, 2, 3, 4, 4, 5, 6, 6, 7, 8, 9, 9])
    send = torch.tensor([1, 3, 2, 2, 4, 0, 1, 6, 7, 9, 5, 9, 8, 5])
    edge_index = torch.stack([recv, send])
    shifts = torch.randint(-1, 2, (recv.numel(), 3), generator=g, dtype=torch.int32)
    p_leaf, c_leaf = pos.clone().requires_grad_(True), cell.clone().requires_grad_(True)
    vec = geo.get_edge_vectors(p_leaf, c_leaf, shifts, edge_index, batch, use_shifts=True)
    wv = torch.randn(vec.shape, generator=g, dtype=torch.float64)
    dpos, dcell = torch.autograd.grad((vec * wv).sum(), [p_leaf, c_leaf])
    t = torch.randn(4, 3, 3, generator=g, dtype=torch.float64)
    out.update({"geom/positions": pos, "geom/cell": cell, "geom/batch": batch, "geom/edge_index": edge_index,
                "geom/shifts": shifts, "geom/vectors": vec.detach(),
                "geom/vectors_noshift": geo.get_edge_vectors(pos, cell, shifts, edge_index, batch, use_shifts=False),
                "geom/weights": wv, "geom/grad_positions": dpos, "geom/grad_cell": dcell,
                "geom/voigt_in": t, "geom/voigt_out": geo.to_voigt6(t)})
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "radial_golden.pt")
    torch.save(out, path)
    print("wrote", path, len(out), "tensors")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.environ.get("PYTHONPATH", "").split(":")[0]))
