"""Dense channel-pair product kernels (fc_tp_fwd / fc_tp_bwd with rowptr == NULL, float32,
both inputs with 64 or 128 channels, weights per row): the product layers' node-level
tensor products (reference ``nn/layers.py:768-1018`` -> ``o3/_tensor_product.py``).

Checked against the float64 evaluation of the same inputs on the generic kernels (which
the golden tests pin to the reference's outputs): forward and all three gradients,
relative to the largest value of each tensor, tolerance 2e-6 (float32 sums of a few
hundred products). Rows that do not fill the last CTA, a row count of one, and the
layouts that stay on the generic kernels (other channel counts, shared weights) are
covered too.
"""

import pytest
import torch

from flashcart_b200 import o3
from flashcart_b200.ops import check_device_status

pytestmark = pytest.mark.gpu


def _run(tp, in1, in2, w, g):
    leaves = [t.detach().clone().requires_grad_(True) for t in (in1, in2, w)]
    out = tp(*leaves)
    grads = torch.autograd.grad(out, leaves, g)
    return out.detach(), grads


def _rel(a, b):
    return (a.double() - b).abs().max().item() / max(1.0, b.abs().max().item())


@pytest.mark.parametrize("sig", [(3, 3, 3), (3, 3, 0), (2, 2, 2), (2, 2, 0), (1, 2, 3), (0, 1, 1)])
@pytest.mark.parametrize("C,n", [(128, 1000), (64, 333), (128, 1)])
def test_gpu_dense_pair_matches_float64(cuda_device, sig, C, n):
    l1, l2, lo = sig
    dev = cuda_device
    tp = o3.TensorProduct(l1, l2, lo, C, C)
    g = torch.Generator(device=dev).manual_seed(7 + C + n)
    in1 = torch.randn(n, tp.in1_dim, device=dev, generator=g)
    in2 = torch.randn(n, tp.in2_dim, device=dev, generator=g)
    w = torch.randn(n, tp.n_total_paths * C, device=dev, generator=g)
    out = tp(in1, in2, w)
    go = torch.randn(out.shape, device=dev, generator=g)
    o32, g32 = _run(tp, in1, in2, w, go)
    o64, g64 = _run(tp, in1.double(), in2.double(), w.double(), go.double())
    assert _rel(o32, o64) < 2e-6
    for a, b in zip(g32, g64):
        assert _rel(a, b) < 2e-6
    check_device_status(dev)


@pytest.mark.parametrize("C", [128, 64])
def test_gpu_dense_pair_shared_weights_without_weight_gradient(cuda_device, C):
    """Shared frozen weights (the element-agnostic product layers): forward and both input
    gradients on the pair kernels."""
    dev = cuda_device
    tp = o3.TensorProduct(3, 3, 3, C, C, shared_weights=True)
    g = torch.Generator(device=dev).manual_seed(5)
    n = 515
    in1 = torch.randn(n, tp.in1_dim, device=dev, generator=g)
    in2 = torch.randn(n, tp.in2_dim, device=dev, generator=g)
    w = torch.randn(tp.n_total_paths * C, device=dev, generator=g)
    go = torch.randn(n, tp(in1, in2, w).shape[1], device=dev, generator=g)

    def run(a, b, ww, gg):
        leaves = [a.clone().requires_grad_(True), b.clone().requires_grad_(True)]
        out = tp(leaves[0], leaves[1], ww)
        return out.detach(), torch.autograd.grad(out, leaves, gg)

    o32, g32 = run(in1, in2, w, go)
    o64, g64 = run(in1.double(), in2.double(), w.double(), go.double())
    assert _rel(o32, o64) < 2e-6
    for a, b in zip(g32, g64):
        assert _rel(a, b) < 2e-6
    check_device_status(dev)


@pytest.mark.parametrize("C,shared", [(96, False), (128, True)])
def test_gpu_dense_products_outside_the_pair_layout(cuda_device, C, shared):
    """96 channels, and shared weights with their gradient requested, take the generic
    kernels; same check."""
    dev = cuda_device
    tp = o3.TensorProduct(3, 3, 3, C, C, shared_weights=shared)
    g = torch.Generator(device=dev).manual_seed(3)
    n = 257
    in1 = torch.randn(n, tp.in1_dim, device=dev, generator=g)
    in2 = torch.randn(n, tp.in2_dim, device=dev, generator=g)
    w = (torch.randn(tp.n_total_paths * C, device=dev, generator=g) if shared else
         torch.randn(n, tp.n_total_paths * C, device=dev, generator=g))
    go = torch.randn(n, tp(in1, in2, w).shape[1], device=dev, generator=g)
    o32, g32 = _run(tp, in1, in2, w, go)
    o64, g64 = _run(tp, in1.double(), in2.double(), w.double(), go.double())
    assert _rel(o32, o64) < 2e-6
    for a, b in zip(g32, g64):
        assert _rel(a, b) < 5e-6
    check_device_status(dev)
