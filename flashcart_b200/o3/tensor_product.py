"""Weighted Cartesian tensor product module (drop-in for reference ``o3/tensor_product.py``)."""

from typing import List, Optional

import torch
import torch.nn as nn

from flashcart_b200 import ops  # noqa: F401  (registers torch.ops.flashcart.*)
from flashcart_b200._native import FC_MAX_L
from flashcart_b200.o3.utils import count_output_paths, get_irreps_slices


class TensorProduct(nn.Module):
    """Weighted natural-parity products of irreducible Cartesian tensor features.

    Constructor, attributes (``in1_dim``, ``in2_dim``, ``out_paths``,
    ``n_total_paths``, slices) and ``forward(in1, in2, weights, idx_i, idx_j)``
    follow the reference (``o3/tensor_product.py:12-172``): with both index arrays
    given it is an edge convolution (in1 gathered at senders ``idx_j``, summed at the
    ascending receivers ``idx_i``). The product runs in the sm_100a kernels through
    ``flashcart::tp_fwd``; ``use_triton`` is accepted for configuration compatibility.
    """

    def __init__(self, in1_l_max: int, in2_l_max: int, out_l_max: int, in1_features: int, in2_features: int,
                 symmetric_product: bool = False, use_triton: bool = False, shared_weights: bool = False,
                 reduce_paths: bool = False):
        super().__init__()
        if not (in1_features == in2_features or in1_features == 1 or in2_features == 1):
            raise ValueError(f"Input dimensions must match unless one of them is 1. "
                             f"Provided: {in1_features=} and {in2_features=}.")
        self.in1_l_max = in1_l_max
        self.in2_l_max = in2_l_max
        self.out_l_max = out_l_max
        self.in1_features = in1_features
        self.in2_features = in2_features
        self.symmetric_product = symmetric_product
        self.use_triton = use_triton
        self.shared_weights = shared_weights
        self.reduce_paths = reduce_paths
        self.in1_dim = sum((2 * l + 1) * in1_features for l in range(in1_l_max + 1))
        self.in2_dim = sum((2 * l + 1) * in2_features for l in range(in2_l_max + 1))
        self.in1_slices = get_irreps_slices(in1_l_max, in1_features)
        self.in2_slices = get_irreps_slices(in2_l_max, in2_features)
        self.out_paths, self.n_total_paths = count_output_paths(in1_l_max, in2_l_max, out_l_max,
                                                                symmetric_product=symmetric_product)
        self.out_features = max(in1_features, in2_features)
        # scalar arguments of flashcart::tp_fwd, padded to the kernel rank limit like the reference
        n_slots = FC_MAX_L + 1
        self._in1_offs = [int(self.in1_slices[l][0]) if l <= in1_l_max else 0 for l in range(n_slots)]
        self._in2_offs = [int(self.in2_slices[l][0]) if l <= in2_l_max else 0 for l in range(n_slots)]
        self._n_paths_per_l = [int(self.out_paths[l]) if l < len(self.out_paths) else 0 for l in range(n_slots)]
        F = self.out_features
        self._out_sizes = [((2 * l + 1) * F if n > 0 else 0) if reduce_paths else n * (2 * l + 1) * F
                           for l, n in enumerate(self._n_paths_per_l)]

    def forward(self, in1: torch.Tensor, in2: torch.Tensor, weights: torch.Tensor,
                idx_i: Optional[torch.Tensor] = None, idx_j: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not in1.shape[-1] == self.in1_dim:
            raise RuntimeError(f"Incorrect last dimension for in1. Expected {self.in1_dim}, got {in1.shape[-1]}.")
        if not in2.shape[-1] == self.in2_dim:
            raise RuntimeError(f"Incorrect last dimension for in2. Expected {self.in2_dim}, got {in2.shape[-1]}.")
        if max(self.in1_l_max, self.in2_l_max, self.out_l_max) > FC_MAX_L:
            raise NotImplementedError(
                f"flashcart_b200 tensor product supports l_max <= {FC_MAX_L}; got in1_l_max={self.in1_l_max}, "
                f"in2_l_max={self.in2_l_max}, out_l_max={self.out_l_max}.")
        if self.symmetric_product and in1 is not in2 and in1.is_cuda:
            # the reference's device assert (o3/tensor_product.py:131) as a status-word bit
            from flashcart_b200 import ops

            ops.flag_if((in1 != in2).any(), ops.DEV_NOT_SYMMETRIC, in1.device)
        conv = idx_i is not None and idx_j is not None
        rows = in2.shape[0] if conv else in1.shape[0]
        expected = self.n_total_paths * self.out_features
        if self.shared_weights:
            if weights.dim() != 1:
                raise ValueError(f"Shared weights must be 1D. Got shape {weights.shape}.")
            if weights.shape[0] != expected:
                raise ValueError(f"Shared weights must have size {expected}, got {weights.shape[0]}.")
        else:
            if weights.dim() != 2:
                raise ValueError(f"Non-shared weights must be 2D. Got shape {weights.shape}.")
            if weights.shape[0] != rows:
                raise ValueError(f"Non-shared weights must have weights.shape[0] = {rows}, got {weights.shape[0]}.")
            if weights.shape[1] != expected:
                raise ValueError(f"Non-shared weights must have weights.shape[1] = {expected}, "
                                 f"got {weights.shape[1]}.")
        return torch.ops.flashcart.tp_fwd(
            in1, in2, weights, idx_i, idx_j, self.in1_l_max, self.in2_l_max, self.out_l_max, self.in1_features,
            self.in2_features, self.symmetric_product, self.shared_weights, self._in1_offs, self._in2_offs,
            self._out_sizes, self._n_paths_per_l, self.n_total_paths, self.reduce_paths)

    def __repr__(self) -> str:
        return (f"{self.__class__.__name__}({self.in1_l_max} x {self.in2_l_max} -> {self.out_l_max}, "
                f"in1_features={self.in1_features}, in2_features={self.in2_features}, "
                f"symmetric={self.symmetric_product}, use_triton={self.use_triton}, paths={self.out_paths}, "
                f"total_paths={self.n_total_paths}, reduce_paths={self.reduce_paths})")
