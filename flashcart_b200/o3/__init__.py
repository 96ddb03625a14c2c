"""Cartesian tensor expansions, tensor products and equivariant linear maps on B200.

Drop-in for the reference package ``flashcart.o3`` (``src/flashcart/o3/__init__.py``):
same module classes, constructor arguments, attributes and state_dict keys; the
computation runs in the sm_100a kernels of ``flashcart_b200`` through the
``torch.ops.flashcart.*`` operators.
"""

from flashcart_b200.o3.irreps import Irreps
from flashcart_b200.o3.tensor_product import TensorProduct
from flashcart_b200.o3.linear import LinearLayer
from flashcart_b200.o3 import utils

__all__ = ["Irreps", "TensorProduct", "LinearLayer", "utils"]
