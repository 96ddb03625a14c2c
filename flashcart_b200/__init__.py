"""flashcart_b200: B200-native (sm_100a) kernels behind FlashCart's o3 operators.

``flashcart_b200.o3`` is a drop-in for ``flashcart.o3`` (Irreps, TensorProduct,
LinearLayer, utils) and ``flashcart_b200.ops`` registers the ``torch.ops.flashcart.*``
operators. The kernels live in ``_lib/libflashcart_b200.so`` and are reached
through the C ABI declared in ``include/flashcart_b200.h``.
"""

__version__ = "0.1.0"
