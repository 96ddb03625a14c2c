"""Layout helpers of the o3 operators (same API as the reference ``o3/utils.py``).

Path counting and ordering, rank-block slices, per-path weight application,
conversion between stored and full Cartesian components and rotation of stored
features. The stored<->full maps come from the exact tables of
:mod:`flashcart_b200.codegen.stf`.
"""

from __future__ import annotations

import functools
from typing import List, Literal, Optional, Sequence, Tuple

import torch

from flashcart_b200.codegen import stf

DotInputPrecision = Literal["ieee", "tf32", "tf32x3"]


def get_triton_dot_input_precision() -> DotInputPrecision:
    """Matrix-product precision selected by the PyTorch flags (reference ``o3/utils.py:14-33``).

    ``"tf32"`` when CUDA is available, TF32 matmuls are allowed and the float32
    matmul precision is ``"high"``; ``"ieee"`` otherwise. The name is kept for
    drop-in compatibility; the value selects the linear-map arithmetic of the
    B200 kernels.
    """
    if not torch.cuda.is_available() or not torch.backends.cuda.matmul.allow_tf32:
        return "ieee"
    return "tf32" if torch.get_float32_matmul_precision() == "high" else "ieee"


def get_linear_triton_kernel_options(dtype: torch.dtype) -> Tuple[bool, DotInputPrecision]:
    """(use float64 accumulation, dot precision) for an input dtype (reference ``o3/utils.py:36-50``)."""
    if dtype == torch.float64:
        return True, "ieee"
    return False, get_triton_dot_input_precision()


@functools.lru_cache(maxsize=None)
def _full_from_stored_cpu(l: int) -> torch.Tensor:
    rows = stf.full_from_stored(l)
    return torch.tensor([[float(v) for v in r] for r in rows], dtype=torch.float64)


def _full_to_stored_matrix(l: int) -> torch.Tensor:
    """(3**l, 2l+1) matrix rebuilding full Cartesian components from stored ones."""
    return _full_from_stored_cpu(l).to(torch.get_default_dtype())


@functools.lru_cache(maxsize=None)
def _stored_full_indices(l: int) -> Tuple[int, ...]:
    out = []
    for a, b, c in stf.stored_basis(l):
        flat = 0
        for d in (0,) * a + (1,) * b + (2,) * c:
            flat = flat * 3 + d
        out.append(flat)
    return tuple(out)


def apply_path_weight(x: torch.Tensor, weights: torch.Tensor, path_idx: int, out_features: int,
                      shared: bool) -> torch.Tensor:
    """Scale one path's output block by its per-feature weights (reference ``o3/utils.py:127-154``)."""
    start = path_idx * out_features
    if shared:
        w = weights[start:start + out_features]
    else:
        w = weights[:, start:start + out_features]
        w = w.reshape(w.shape[0], *([1] * (x.dim() - 2)), w.shape[1])
    return x * w


def count_output_paths(in1_l_max: int, in2_l_max: int, out_l_max: int,
                       symmetric_product: bool = False) -> Tuple[List[int], int]:
    """Allowed coupling paths per output rank and their total (reference ``o3/utils.py:157-203``)."""
    paths = stf.enumerate_paths(in1_l_max, in2_l_max, out_l_max, symmetric_product)
    out = [0] * (out_l_max + 1)
    for _, _, lo in paths:
        out[lo] += 1
    return out, sum(out)


def get_irreps_slices(l_max: int, n_features: int, n_paths: Optional[List[int]] = None) -> list:
    if n_paths is None:
        n_paths = [1] * (l_max + 1)
    slices, start = [], 0
    for l in range(l_max + 1):
        size = (2 * l + 1) * n_features * n_paths[l]
        slices.append((start, start + size))
        start += size
    return slices


def get_irreps_shapes(l_max: int, n_features: int, n_paths: Optional[List[int]] = None,
                      mode: str = "flattened") -> list:
    if n_paths is None:
        n_paths = [1] * (l_max + 1)
    if mode == "factorized":
        return [(2 * l + 1, n_features, n_paths[l]) for l in range(l_max + 1)]
    return [(2 * l + 1, n_features * n_paths[l]) for l in range(l_max + 1)]


def get_cartesian_slices(l_max: int, n_features: int, n_paths: Optional[List[int]] = None) -> list:
    if n_paths is None:
        n_paths = [1] * (l_max + 1)
    slices, start = [], 0
    for l in range(l_max + 1):
        size = (3 ** l) * n_features * n_paths[l]
        slices.append((start, start + size))
        start += size
    return slices


def _feature_count(total: int, per: int, l_max: int) -> int:
    if total % per != 0:
        raise ValueError(f"Tensor size {total} incompatible with l_max={l_max}.")
    return total // per


def irreps_to_cartesian(irreps: torch.Tensor, l_max: int, n_paths: Optional[List[int]] = None) -> torch.Tensor:
    """Full Cartesian components from stored ones (reference ``o3/utils.py:289-342``)."""
    n = irreps.shape[0]
    n_paths = [1] * (l_max + 1) if n_paths is None else list(n_paths)
    feats = _feature_count(irreps.shape[1], sum((2 * l + 1) * n_paths[l] for l in range(l_max + 1)), l_max)
    parts, off = [], 0
    for l in range(l_max + 1):
        size = (2 * l + 1) * feats * n_paths[l]
        blk = irreps[:, off:off + size]
        off += size
        if l == 0:
            parts.append(blk)
            continue
        m = _full_from_stored_cpu(l).to(device=blk.device, dtype=blk.dtype)
        full = torch.einsum("fk,bku->bfu", m, blk.reshape(n, 2 * l + 1, feats * n_paths[l]))
        parts.append(full.reshape(n, -1))
    return torch.cat(parts, dim=-1)


def cartesian_to_irreps(tensors: torch.Tensor, l_max: int, n_paths: Optional[List[int]] = None) -> torch.Tensor:
    """Stored components of symmetric traceless full tensors (reference ``o3/utils.py:345-397``)."""
    n = tensors.shape[0]
    n_paths = [1] * (l_max + 1) if n_paths is None else list(n_paths)
    feats = _feature_count(tensors.shape[1], sum((3 ** l) * n_paths[l] for l in range(l_max + 1)), l_max)
    parts, off = [], 0
    for l in range(l_max + 1):
        size = (3 ** l) * feats * n_paths[l]
        blk = tensors[:, off:off + size]
        off += size
        if l == 0:
            parts.append(blk)
            continue
        idx = torch.as_tensor(_stored_full_indices(l), device=blk.device, dtype=torch.long)
        parts.append(blk.reshape(n, 3 ** l, feats * n_paths[l]).index_select(1, idx).reshape(n, -1))
    return torch.cat(parts, dim=1)


def rotate_irreps(irreps: torch.Tensor, rot_matrix: torch.Tensor, l_max: int,
                  n_paths: Optional[List[int]] = None) -> torch.Tensor:
    """Apply an orthogonal 3x3 map to every Cartesian index (reference ``o3/utils.py:400-468``)."""
    if rot_matrix.dim() != 2 or rot_matrix.shape != (3, 3):
        raise ValueError(f"Rotation matrix must be of shape [3, 3]. Provided shape: {rot_matrix.shape}.")
    if l_max > 13:
        raise NotImplementedError(f"rotate_irreps supports l_max <= 13, got l_max={l_max}.")
    n = irreps.shape[0]
    n_paths = [1] * (l_max + 1) if n_paths is None else list(n_paths)
    feats = _feature_count(irreps.shape[1], sum((2 * l + 1) * n_paths[l] for l in range(l_max + 1)), l_max)
    cart = irreps_to_cartesian(irreps, l_max, n_paths)
    parts, off = [], 0
    for l in range(l_max + 1):
        size = (3 ** l) * feats * n_paths[l]
        blk = cart[:, off:off + size]
        off += size
        if l == 0:
            parts.append(blk)
            continue
        t = blk.reshape(n, *([3] * l), feats * n_paths[l])
        outs = "abcdefghijklm"[:l]
        ins = "nopqrstuvwxyz"[:l]
        spec = ",".join(f"{o}{i}" for o, i in zip(outs, ins)) + f",B{ins}F->B{outs}F"
        parts.append(torch.einsum(spec, *([rot_matrix] * l), t).reshape(n, -1))
    return cartesian_to_irreps(torch.cat(parts, dim=1), l_max, n_paths)
