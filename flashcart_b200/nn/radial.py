"""Radial bases and the cutoff envelope (same modules and buffers as reference ``nn/radial.py``)."""

import math
from typing import Literal

import torch
import torch.nn as nn


class BesselBasis(nn.Module):
    """sqrt(2/r_max) sin(n pi r / r_max) / r, n = 1..n_radial (reference ``nn/radial.py:8-57``)."""

    def __init__(self, n_radial: int, r_max: float):
        super().__init__()
        if n_radial <= 0:
            raise ValueError(f"n_radial must be positive. Provided: {n_radial}.")
        if r_max <= 0.0:
            raise ValueError(f"r_max must be positive. Provided: {r_max}.")
        dt = torch.get_default_dtype()
        self.n_radial = n_radial
        self.register_buffer("bessel_weights", (math.pi / r_max) * torch.arange(1, n_radial + 1, dtype=dt))
        self.register_buffer("r_cutoff", torch.tensor(r_max, dtype=dt))
        self.register_buffer("pre_factor", torch.tensor(math.sqrt(2.0 / r_max), dtype=dt))

    def forward(self, distances: torch.Tensor) -> torch.Tensor:
        x = distances.unsqueeze(-1) * self.bessel_weights
        return self.pre_factor * self.bessel_weights * torch.sinc(x / math.pi)


class ChebyshevBasis(nn.Module):
    """T_0..T_{n-1} of cos(pi t) ("cosine") or 2t-1 ("affine"), t = (r - r_min)/(r_max - r_min).

    Reference ``nn/radial.py:60-128``; evaluated with the three-term recurrence.
    """

    def __init__(self, n_radial: int, r_max: float, r_min: float = 0.0,
                 mapping: Literal["cosine", "affine"] = "affine"):
        super().__init__()
        if r_max <= r_min:
            raise ValueError(f"Expected r_max > r_min. Provided: r_min={r_min}, r_max={r_max}.")
        if mapping not in ("cosine", "affine"):
            raise ValueError(f"Expected mapping to be 'cosine' or 'affine'. Provided: {mapping}.")
        dt = torch.get_default_dtype()
        self.n_radial = n_radial
        self.mapping = mapping
        self.register_buffer("r_min", torch.tensor(r_min, dtype=dt))
        self.register_buffer("r_max", torch.tensor(r_max, dtype=dt))

    def forward(self, distances: torch.Tensor) -> torch.Tensor:
        t = (distances - self.r_min) / (self.r_max - self.r_min)
        x = torch.cos(t * math.pi) if self.mapping == "cosine" else 2.0 * t - 1.0
        if self.n_radial == 1:
            return torch.ones_like(x).unsqueeze(-1)
        terms = [torch.ones_like(x), x]
        for _ in range(2, self.n_radial):
            terms.append(2.0 * x * terms[-1] - terms[-2])
        return torch.stack(terms, dim=-1)


class PolynomialCutoff(nn.Module):
    """1 - c1 t^p + c2 t^(p+1) - c3 t^(p+2), t = r/r_max, zero at and beyond r_max.

    Reference ``nn/radial.py:131-245`` (same buffers, same evaluation order).
    """

    def __init__(self, r_max: float, poly_order: int = 6):
        super().__init__()
        if poly_order < 2:
            raise ValueError(f"Polynomial order must be >= 2. Provided: {poly_order}.")
        dt = torch.get_default_dtype()
        p = int(poly_order)
        self.poly_order_value = p
        self.register_buffer("poly_order", torch.tensor(p, dtype=torch.long))
        self.register_buffer("r_max", torch.tensor(r_max, dtype=dt))
        self.register_buffer("coeff1", torch.tensor((p + 1.0) * (p + 2.0) / 2.0, dtype=dt))
        self.register_buffer("coeff2", torch.tensor(p * (p + 2.0), dtype=dt))
        self.register_buffer("coeff3", torch.tensor(p * (p + 1.0) / 2.0, dtype=dt))

    def forward(self, distances: torch.Tensor) -> torch.Tensor:
        d = torch.clamp(distances, min=0.0)
        t = d / self.r_max
        p = self.poly_order_value
        if p <= 4:
            tp, tp1, tp2 = torch.pow(t, p), torch.pow(t, p + 1), torch.pow(t, p + 2)
        else:
            tp = t.clone()
            for _ in range(p - 1):
                tp = tp * t
            tp1 = tp * t
            tp2 = tp1 * t
        env = 1.0 - self.coeff1 * tp + self.coeff2 * tp1 - self.coeff3 * tp2
        mask = (d < self.r_max).to(dtype=env.dtype)
        return torch.clamp(env * mask, min=0.0, max=1.0)
