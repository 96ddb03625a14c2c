"""Equivariant linear map module (drop-in for reference ``o3/linear.py``)."""

from typing import Optional, Sequence

import torch
import torch.nn as nn

from flashcart_b200 import ops  # noqa: F401  (registers torch.ops.flashcart.*)
from flashcart_b200.o3.utils import get_irreps_slices, get_linear_triton_kernel_options


def make_linear_metadata(device, in_l_max: int, out_l_max: int, in_features: int, out_features: int,
                         in_paths: Sequence[int], weight_scale: Optional[float]):
    """Per-rank layout metadata and scales (reference ``o3/_linear.py:113-166``).

    Rows of metadata: (input offset, output offset, weight offset, components,
    input width, output width) for each rank shared by input and output.
    """
    common = min(in_l_max, out_l_max)
    paths = list(in_paths)
    in_slices = get_irreps_slices(in_l_max, in_features, paths)
    out_slices = get_irreps_slices(out_l_max, out_features, [1] * (out_l_max + 1))
    if weight_scale is not None:
        scales = [float(weight_scale)] * (common + 1)
    else:
        scales = [float(in_features * paths[l]) ** -0.5 for l in range(common + 1)]
    meta, w_off = [], 0
    for l in range(common + 1):
        f_in = in_features * paths[l]
        meta.append([in_slices[l][0], out_slices[l][0], w_off, 2 * l + 1, f_in, out_features])
        w_off += f_in * out_features
    meta_t = torch.tensor(meta, dtype=torch.int64, device=device).reshape(-1, 6)
    out_size = sum((2 * l + 1) * out_features for l in range(out_l_max + 1))
    return meta_t, torch.tensor(scales, device=device), w_off, out_size


class LinearLayer(nn.Module):
    """Per-rank channel mixing ``y_l = x_l (scale_l W_l)^T``; output ranks above ``in_l_max`` are zero.

    Same constructor, ``weight`` ParameterList (state_dict keys ``weight.{l}``) and
    N(0,1) initialisation as the reference (``o3/linear.py:11-128``); evaluation
    runs in the sm_100a kernels through ``flashcart::linear_fwd``.
    """

    def __init__(self, in_l_max: int, out_l_max: int, in_features: int, out_features: int,
                 in_paths: Optional[Sequence[int]] = None, weight_scale: Optional[float] = None,
                 use_triton: bool = False):
        super().__init__()
        self.in_l_max = in_l_max
        self.out_l_max = out_l_max
        self.in_features = in_features
        self.out_features = out_features
        self.in_paths = [1] * (in_l_max + 1) if in_paths is None else [int(p) for p in in_paths]
        self.weight_scale = weight_scale
        self.use_triton = use_triton
        if len(self.in_paths) != in_l_max + 1:
            raise ValueError(f"Expected {in_l_max + 1} in_paths, got {len(self.in_paths)}.")
        self.common_l_max = min(in_l_max, out_l_max)
        self.in_dim = sum((2 * l + 1) * in_features * self.in_paths[l] for l in range(in_l_max + 1))
        self.out_dim = sum((2 * l + 1) * out_features for l in range(out_l_max + 1))
        meta, scale, n_weight, out_size = make_linear_metadata(torch.device("cpu"), in_l_max, out_l_max,
                                                               in_features, out_features, self.in_paths,
                                                               weight_scale)
        rows = [[int(v) for v in r] for r in meta.tolist()]
        self.meta_lists = tuple([r[i] for r in rows] for i in range(6))
        self.register_buffer("meta", meta, persistent=False)
        self.register_buffer("scale", scale, persistent=False)
        self.n_weight = int(n_weight)
        if int(out_size) != self.out_dim:
            raise RuntimeError(f"Metadata out_size mismatch: {out_size} != {self.out_dim}.")
        self.weight = nn.ParameterList()
        for l in range(self.common_l_max + 1):
            self.weight.append(nn.Parameter(torch.randn(out_features, in_features * self.in_paths[l])))

    def forward(self, x: torch.Tensor, input_scale: Optional[torch.Tensor] = None,
                residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``input_scale`` (optional, 0-d tensor) multiplies the input: the map is linear, so
        it is applied to the per-rank scales instead of to every element of ``x``.
        ``residual`` (optional, laid out like the output) is added to the result: inside the
        GEMM's epilogue where ``ops.linear_residual_fusable`` allows (first-order
        evaluation, frozen float32 weights), else as a separate sum."""
        if x.shape[-1] != self.in_dim:
            raise RuntimeError(f"Incorrect last dimension for x. Expected {self.in_dim}, got {x.shape[-1]}.")
        if x.dim() != 2:
            raise ValueError(f"x must be 2D [N, packed_dim], got shape {tuple(x.shape)}.")
        use_fp64, precision = get_linear_triton_kernel_options(x.dtype)
        weights = [w if w.dtype == x.dtype else w.to(x.dtype) for w in self.weight]
        scale = self.scale if input_scale is None else self.scale * input_scale
        if residual is not None:
            in_offs, out_offs, _, m, fi, fo = self.meta_lists
            if ops.linear_residual_fusable(x, weights, self.out_dim, m, fi, fo, in_offs, out_offs, residual):
                return torch.ops.flashcart.linear_residual_fwd(x, weights, residual, self.out_dim, precision, in_offs,
                                                               out_offs, m, fi, fo, scale)
            return torch.ops.flashcart.linear_fwd(x, weights, self.meta, self.out_dim, use_fp64, precision,
                                                  *self.meta_lists, scale) + residual
        return torch.ops.flashcart.linear_fwd(x, weights, self.meta, self.out_dim, use_fp64, precision,
                                              *self.meta_lists, scale)

    def extra_repr(self) -> str:
        return (f"in_l_max={self.in_l_max}, out_l_max={self.out_l_max}, in_features={self.in_features}, "
                f"out_features={self.out_features}, in_paths={self.in_paths}, out_dim={self.out_dim}, "
                f"n_weights={self.n_weight}, use_triton={self.use_triton}")
