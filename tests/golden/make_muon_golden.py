"""Generate golden vectors of the Muon Newton-Schulz step from the REFERENCE implementation.

Run where the reference source tree is available (never needed at test time)::

    PYTHONPATH=<reference>/src python tests/golden/make_muon_golden.py [<reference>/src]

Calls the reference's ``_batched_newtonschulz`` (``training/muon.py:27-61``) on the CPU
with its default coefficients (5 iterations of (3.4445, -4.7750, 2.0315), eps 1e-7) on
seeded updates of the shapes the optimizer batches (wide, tall -> transposed, a small
hidden layer), plus one case with two polishing iterations. Inputs are float32; outputs
bfloat16, as the reference returns them.

Output: ``tests/golden/muon_golden.pt``.
"""

from __future__ import annotations

import os
import sys

import torch


def main(src: str) -> None:
    # load training/muon.py by path: the package's __init__ pulls in training-only
    # dependencies (torch_ema) that the Newton-Schulz function does not use
    import importlib.util

    spec = importlib.util.spec_from_file_location("ref_muon", os.path.join(src, "flashcart", "training", "muon.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    NS_COEFF_FAST, NS_COEFF_POLISH, _batched_newtonschulz = mod.NS_COEFF_FAST, mod.NS_COEFF_POLISH, \
        mod._batched_newtonschulz

    g = torch.Generator().manual_seed(11)
    cases = {}
    for name, shape, polish in [("wide", (3, 64, 448), 0), ("tall", (2, 192, 128), 0), ("small", (4, 8, 64), 0),
                                ("square_polish", (2, 128, 128), 2)]:
        u = torch.randn(*shape, generator=g)
        out = _batched_newtonschulz(u, NS_COEFF_FAST, 5, 1e-7, NS_COEFF_POLISH, polish)
        cases[name] = {"update": u, "out": out.clone(), "polish_steps": polish}
    torch.save({"coeffs": list(NS_COEFF_FAST), "polish": list(NS_COEFF_POLISH), "steps": 5, "eps": 1e-7,
                "cases": cases}, os.path.join(os.path.dirname(os.path.abspath(__file__)), "muon_golden.pt"))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLASHCART_REF_SRC", "."))
