"""Generate golden vectors of the radial basis and cutoff from the REFERENCE implementation.

Run where the reference source tree is available (never needed at test time)::

    PYTHONPATH=<reference>/src python tests/golden/make_radial_golden.py [<reference>/src]

Evaluates the reference's ``ChebyshevBasis`` (cosine and affine mappings, with and
without r_min), ``BesselBasis`` and ``PolynomialCutoff`` (``nn/radial.py:8-245``) in
float64 on distances that cover the interior, r = 0 (Bessel's removable singularity),
r = r_min, r = r_max and beyond the cutoff, and records the values and the first
derivative with respect to the distance (autograd of the summed, seeded-weighted output),
which the forces depend on.

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
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "radial_golden.pt")
    torch.save(out, path)
    print("wrote", path, len(out), "tensors")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.environ.get("PYTHONPATH", "").split(":")[0]))
