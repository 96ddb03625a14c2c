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
        # the reference asserts unit length on the device (o3/irreps.py:66-69); here a
        # violation sets a bit of the status word (raised by ops.check_device_status) so that
        # bad input never takes down the CUDA context
        if x.is_cuda:
            from flashcart_b200 import ops

            ops.flag_if((x.pow(2).sum(dim=-1) - 1.0).abs().gt(1.0e-5).any(), ops.DEV_NOT_UNIT, x.device)
        return torch.ops.flashcart.irreps_fwd(x, self.l_max)

    def __repr__(self):
        return (f"{self.__class__.__name__}(l_max={self.l_max}, use_triton={self.use_triton}, "
                f"output_dim={(self.l_max + 1) ** 2})")
