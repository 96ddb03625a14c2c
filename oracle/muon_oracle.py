"""CPU restatement of the Muon Newton-Schulz orthogonalisation (test infrastructure).

Follows the reference's ``_batched_newtonschulz`` (``training/muon.py:27-61``), the
quintic iteration of the Muon optimizer as in ``torch.optim._muon``:

    X = bf16(U), transposed when rows > cols;  X <- X / max(||X||_F, eps)
    for each (a, b, c) step:  G = X X^T;  G' = b G + c G G;  X = a X + G' X

in bfloat16 tensors (each product accumulated in fp32 and rounded once, as torch's
bf16 bmm / baddbmm do), and in float64 for reference without rounding. Only the
tests and the CPU legs of the benchmark import this module.
"""

from __future__ import annotations

from typing import Sequence

import torch


def newton_schulz(update: torch.Tensor, coeffs: Sequence[float], steps: int, eps: float,
                  polish: Sequence[float] = (2.0, -1.5, 0.5), polish_steps: int = 0,
                  dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    x = update.to(dtype)
    transposed = x.size(1) > x.size(2)
    if transposed:
        x = x.transpose(1, 2)
    x = x / x.norm(dim=(1, 2), keepdim=True).clamp(min=eps)
    for (a, b, c), n in ((tuple(coeffs), steps), (tuple(polish), polish_steps)):
        for _ in range(n):
            g = torch.bmm(x, x.transpose(1, 2))
            g2 = torch.baddbmm(g, g, g, beta=b, alpha=c)
            x = torch.baddbmm(x, g2, x, beta=a)
    return x.transpose(1, 2) if transposed else x
