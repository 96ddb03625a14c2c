"""Direction-tensor expansion module (drop-in for reference ``o3/irreps.py``)."""

import torch
import torch.nn as nn

from flashcart_b200 import ops  # noqa: F401  (registers torch.ops.flashcart.*)
from flashcart_b200._native import FC_MAX_L


class Irreps(nn.Module):
    """Stored STF components of T^l(x), l = 0..l_max, of unit vectors x: (n, 3) -> (n, (l_max+1)^2).

    Same constructor, attributes and behaviour as the reference (``o3/irreps.py:9-80``);
    ``use_triton`` is accepted for configuration compatibility. Evaluation always uses
    the sm_100a kernels (``flashcart::irreps_fwd``); CPU tensors raise.
    """

    def __init__(self, l_max: int, use_triton: bool = False):
        super().__init__()
        if l_max > FC_MAX_L:
            raise RuntimeError(f"Irreps supports l_max <= {FC_MAX_L}, got {l_max=}.")
        self.l_max = l_max
        self.use_triton = use_triton

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = torch.nn.functional.normalize(x, dim=-1)
        return self.forward_normalized(x)

    def forward_normalized(self, x: torch.Tensor) -> torch.Tensor:
        r2 = x.pow(2).sum(dim=-1)
        torch._assert_async(((r2 - 1.0).abs() <= 1.0e-5).all(),
                            "Irreps.forward_normalized requires unit-length input vectors.")
        return torch.ops.flashcart.irreps_fwd(x, self.l_max)

    def __repr__(self):
        return (f"{self.__class__.__name__}(l_max={self.l_max}, use_triton={self.use_triton}, "
                f"output_dim={(self.l_max + 1) ** 2})")
