"""Seeded synthetic structures used by the benchmark and the tests.

Water-like boxes (the reference's water MD example stands in here; its datasets are
not used): one H2O per site of a jittered simple-cubic lattice with spacing
12.42/4 A (about 1 g/cm^3), O-H 0.96 A, H-O-H 104.5 degrees, a uniformly random
orientation per molecule (random unit quaternion), periodic orthorhombic cell.
Atoms are ordered O, H, H per molecule; elements are ["H", "O"] (types 1 = O).
"""

from __future__ import annotations

import math
from typing import Dict, Tuple

import numpy as np
import torch

WATER_SPACING = 12.42 / 4.0
OH_BOND = 0.96
HOH_ANGLE = math.radians(104.5)


def _random_rotations(rng: np.random.Generator, n: int) -> np.ndarray:
    """Uniform random rotation matrices from uniform unit quaternions (Shoemake 1992)."""
    u1, u2, u3 = rng.random(n), rng.random(n), rng.random(n)
    a, b = np.sqrt(1.0 - u1), np.sqrt(u1)
    q = np.stack([a * np.sin(2 * np.pi * u2), a * np.cos(2 * np.pi * u2),
                  b * np.sin(2 * np.pi * u3), b * np.cos(2 * np.pi * u3)], axis=1)  # (x, y, z, w)
    x, y, z, w = q.T
    return np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)], -1),
        np.stack([2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)], -1),
        np.stack([2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)], -1)], axis=1)


def water_box(nx: int, ny: int, nz: int, seed: int = 0, jitter: float = 0.3,
              spacing: float = WATER_SPACING) -> Dict[str, np.ndarray]:
    """nx*ny*nz molecules; returns positions (3M, 3), atom_types (3M,), cell (3, 3), pbc."""
    rng = np.random.default_rng(seed)
    grid = np.stack(np.meshgrid(np.arange(nx), np.arange(ny), np.arange(nz), indexing="ij"), -1).reshape(-1, 3)
    o = (grid + 0.5) * spacing + rng.uniform(-jitter, jitter, size=grid.shape)
    half = HOH_ANGLE / 2.0
    local = np.array([[math.sin(half), 0.0, math.cos(half)], [-math.sin(half), 0.0, math.cos(half)]]) * OH_BOND
    rot = _random_rotations(rng, len(o))
    h = o[:, None, :] + np.einsum("mij,hj->mhi", rot, local)
    pos = np.concatenate([o[:, None, :], h], axis=1).reshape(-1, 3)
    types = np.tile(np.array([1, 0, 0], dtype=np.int64), len(o))
    cell = np.diag([nx * spacing, ny * spacing, nz * spacing]).astype(np.float64)
    return {"positions": pos.astype(np.float64), "atom_types": types, "cell": cell, "pbc": np.array([True] * 3)}


def config0_water() -> Dict[str, np.ndarray]:
    """192-atom box (64 H2O, 12.42 A edge)."""
    return water_box(4, 4, 4, seed=0)


def config3_water() -> Dict[str, np.ndarray]:
    """27,648-atom box (9,216 H2O, 24 x 24 x 16 sites, 74.52 x 74.52 x 49.68 A)."""
    return water_box(24, 24, 16, seed=0)


def graph_from_structure(s: Dict[str, np.ndarray], edge_index: np.ndarray, shifts: np.ndarray,
                         device="cpu", dtype=torch.float32) -> Dict[str, torch.Tensor]:
    """Tensor dict accepted by FlashCartPotential.forward / predict (one periodic graph)."""
    n = len(s["positions"])
    return {
        "positions": torch.as_tensor(s["positions"], dtype=dtype, device=device),
        "cell": torch.as_tensor(s["cell"], dtype=dtype, device=device).unsqueeze(0),
        "atom_types": torch.as_tensor(s["atom_types"], dtype=torch.int64, device=device),
        "edge_index": torch.as_tensor(edge_index, dtype=torch.int64, device=device),
        "shifts": torch.as_tensor(shifts, dtype=torch.int32, device=device),
        "batch": torch.zeros(n, dtype=torch.int64, device=device),
        "n_atoms": torch.tensor([n], dtype=torch.int64, device=device),
        "pbc": torch.tensor([bool(v) for v in s["pbc"]], device=device),
    }
