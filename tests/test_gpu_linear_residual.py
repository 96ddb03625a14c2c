"""Residual forms of the float32 linear maps (fc_linear_fwd_residual / fc_linear_bwd_residual,
flashcart::linear_residual_fwd): map(x) + residual and map^T(g) + residual with the sum in
the GEMM's epilogue, as the node-level layers use them for their residual connections
(reference ``nn/layers.py:395-405, 609-635``).

Checked against the separate sum on the same kernels (forward and both input gradients,
float32, tolerance 2e-6 of the output scale: the epilogue adds the residual to the
float32 accumulation instead of rounding first), an accumulation into the output buffer
itself, a layout the epilogue does not take (256 output channels per rank: the separate
sum), and the C-ABI's refusals.
"""

import ctypes

import pytest
import torch

from flashcart_b200 import _native as N
from flashcart_b200 import o3, ops
from flashcart_b200.ops import check_device_status

pytestmark = pytest.mark.gpu


def _frozen(lin):
    for p in lin.parameters():
        p.requires_grad_(False)
    return lin


def _rel(a, b):
    return (a.double() - b.double()).abs().max().item() / max(1.0, b.double().abs().max().item())


@pytest.mark.parametrize("shape", [(3, 3, 128, 128, 2000), (2, 2, 64, 64, 777), (3, 3, 128, 128, 1)])
def test_gpu_linear_residual_matches_separate_sum(cuda_device, shape):
    li, lo, fi, fo, n = shape
    dev = cuda_device
    torch.manual_seed(n)
    lin = _frozen(o3.LinearLayer(li, lo, fi, fo).to(dev))
    x = torch.randn(n, lin.in_dim, device=dev)
    r = torch.randn(n, lin.out_dim, device=dev)
    g = torch.randn(n, lin.out_dim, device=dev)
    with ops.first_order_only():
        x1, r1 = x.clone().requires_grad_(True), r.clone().requires_grad_(True)
        in_offs, out_offs, _, m, f_in, f_out = lin.meta_lists
        assert ops.linear_residual_fusable(x1, list(lin.weight), lin.out_dim, m, f_in, f_out, in_offs, out_offs, r1)
        y1 = lin(x1, residual=r1)
        gx1, gr1 = torch.autograd.grad(y1, [x1, r1], g)
    x2, r2 = x.clone().requires_grad_(True), r.clone().requires_grad_(True)
    y2 = lin(x2) + r2
    gx2, gr2 = torch.autograd.grad(y2, [x2, r2], g)
    assert _rel(y1, y2) < 2e-6
    assert _rel(gx1, gx2) < 2e-6
    assert torch.equal(gr1, gr2)
    check_device_status(dev)


def test_gpu_linear_residual_accumulates_in_place_through_the_c_abi(cuda_device):
    """grad_x += map^T(g) with the residual and the output the same buffer, twice."""
    dev = cuda_device
    torch.manual_seed(3)
    lin = _frozen(o3.LinearLayer(3, 3, 128, 128).to(dev))
    n = 1500
    g = torch.randn(n, lin.out_dim, device=dev)
    base = torch.randn(n, lin.in_dim, device=dev)
    in_offs, out_offs, _, m, f_in, f_out = lin.meta_lists
    lists = (in_offs, out_offs, [0] * len(in_offs), m, f_in, f_out)
    gx_alone = ops._linear_input_grad(g, lin.in_dim, list(lin.weight), lists, "ieee", lin.scale)
    buf = base.clone()
    for _ in range(2):
        ops._linear_residual_impl(g, list(lin.weight), lin.in_dim, lists, "ieee", lin.scale, buf, True, out=buf)
    want = base + 2 * gx_alone
    assert _rel(buf, want) < 2e-6
    check_device_status(dev)


def test_gpu_linear_residual_outside_the_epilogue_layout(cuda_device):
    """256 output channels per rank are not taken by the epilogue: the layer sums separately."""
    dev = cuda_device
    torch.manual_seed(4)
    lin = _frozen(o3.LinearLayer(1, 1, 64, 256).to(dev))
    x = torch.randn(300, lin.in_dim, device=dev)
    r = torch.randn(300, lin.out_dim, device=dev)
    in_offs, out_offs, _, m, f_in, f_out = lin.meta_lists
    with ops.first_order_only():
        assert not ops.linear_residual_fusable(x, list(lin.weight), lin.out_dim, m, f_in, f_out, in_offs, out_offs, r)
        y = lin(x, residual=r)
    assert _rel(y, lin(x) + r) < 1e-6
    check_device_status(dev)


def test_gpu_linear_residual_c_abi_refusals(cuda_device):
    dev = cuda_device
    lib = N.lib()
    lin = _frozen(o3.LinearLayer(1, 1, 8, 8).to(dev))
    x = torch.randn(10, lin.in_dim, device=dev)
    r = torch.randn(10, lin.out_dim, device=dev)
    out = torch.empty_like(r)
    ws = list(lin.weight)
    arr = (ctypes.c_void_p * len(ws))(*[w.data_ptr() for w in ws])
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    in_offs, out_offs, _, m, f_in, f_out = lin.meta_lists
    d = ops._linear_desc(x, lin.out_dim, in_offs, out_offs, m, f_in, f_out, "ieee", N.FC_ACT_SILU)
    rc = lib.fc_linear_fwd_residual(ctypes.byref(d), ctypes.c_void_p(x.data_ptr()), arr, None,
                                    ctypes.c_void_p(lin.scale.data_ptr()), 10, ctypes.c_void_p(r.data_ptr()),
                                    ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(status.data_ptr()), None)
    assert rc == N.FC_ERR_UNSUPPORTED and b"activation" in lib.fc_last_error()
    xd = x.double()
    d = ops._linear_desc(xd, lin.out_dim, in_offs, out_offs, m, f_in, f_out, "ieee", 0)
    rc = lib.fc_linear_fwd_residual(ctypes.byref(d), ctypes.c_void_p(xd.data_ptr()), arr, None,
                                    ctypes.c_void_p(lin.scale.data_ptr()), 10, ctypes.c_void_p(r.data_ptr()),
                                    ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(status.data_ptr()), None)
    assert rc == N.FC_ERR_UNSUPPORTED


@pytest.mark.parametrize("gate", ["sigmoid", "silu"])
def test_gpu_gated_layer_single_node_matches_composed(cuda_device, gate):
    """EquivariantGatedLayer as one autograd node (first-order evaluation, frozen weights:
    the value map's input gradient takes the residual's gradient in its epilogue) against
    the composed layer, output and input gradient."""
    from flashcart_b200.nn.layers import EquivariantGatedLayer

    dev = cuda_device
    torch.manual_seed(7)
    layer = _frozen(EquivariantGatedLayer(3, 128, 128, gate_activation=gate).to(dev))
    with torch.no_grad():
        for w in layer.output_linear.weight:
            w.normal_()  # zero at initialisation: make the gated branch contribute
    x = torch.randn(1200, layer.in_dim, device=dev)
    g = torch.randn_like(x)
    with ops.first_order_only():
        x1 = x.clone().requires_grad_(True)
        assert layer._fused_ok(x1)
        y1 = layer(x1)
        (gx1,) = torch.autograd.grad(y1, [x1], g)
    x2 = x.clone().requires_grad_(True)
    y2 = layer(x2)
    (gx2,) = torch.autograd.grad(y2, [x2], g)
    assert _rel(y1, y2) < 2e-6
    assert _rel(gx1, gx2) < 2e-6
    check_device_status(dev)


@pytest.mark.parametrize("out_l_max,C", [(3, 128), (0, 128), (2, 64)])
def test_gpu_product_layer_single_node_matches_composed(cuda_device, out_l_max, C):
    """ProductLayer as one autograd node (first-order evaluation, frozen weights: the dense
    products' backward adds the sum's gradient to their in1 gradient and accumulates their
    in2 gradient into the node-feature gradient, fc_tp_bwd_residual) against the composed
    layer, for a layer that keeps every rank and one that keeps the low ranks only."""
    from flashcart_b200.nn.layers import ProductLayer

    dev = cuda_device
    torch.manual_seed(11 + out_l_max)
    in_l_max = 3 if C == 128 else 2
    layer = ProductLayer(in_l_max, min(out_l_max, in_l_max), C, correlation=3, use_sc=True,
                         use_layer_norm=True).to(dev)
    _frozen(layer)
    with torch.no_grad():
        for p in layer.parameters():
            if p.dim() > 0:
                p.add_(0.1 * torch.randn_like(p))
    x = torch.randn(900, layer.in_dim, device=dev) * 0.5
    with ops.first_order_only():
        x1 = x.clone().requires_grad_(True)
        assert layer._single_node_ok(x1)
        y1 = layer(x1)
        g = torch.randn_like(y1)
        (gx1,) = torch.autograd.grad(y1, [x1], g)
    x2 = x.clone().requires_grad_(True)
    y2 = layer(x2)
    (gx2,) = torch.autograd.grad(y2, [x2], g)
    assert _rel(y1, y2) < 5e-6
    assert _rel(gx1, gx2) < 5e-6
    check_device_status(dev)


def test_gpu_tp_bwd_residual_through_the_c_abi(cuda_device):
    """fc_tp_bwd_residual against fc_tp_bwd plus the residuals, twice into the same in2 buffer."""
    dev = cuda_device
    torch.manual_seed(12)
    C, n = 128, 700
    tp = o3.TensorProduct(3, 3, 3, C, C, shared_weights=True)
    in1 = torch.randn(n, tp.in1_dim, device=dev)
    in2 = torch.randn(n, tp.in2_dim, device=dev)
    w = torch.randn(tp.n_total_paths * C, device=dev)
    with torch.no_grad():
        out = tp(in1, in2, w)
    go = torch.randn_like(out)
    a, b = in1.clone().requires_grad_(True), in2.clone().requires_grad_(True)
    ref1, ref2 = torch.autograd.grad(tp(a, b, w), [a, b], go)
    r1 = torch.randn(n, 4 * C, device=dev)  # the first 4 components (l <= 1) of each in1 row
    r2 = torch.randn(n, tp.in2_dim, device=dev)
    acc = r2.clone()
    for _ in range(2):
        g1, acc = ops.tp_dense_bwd_residual(tp, go, in1, in2, w, r1, 4, acc, out_in2=acc)
    want1 = ref1.clone()
    want1[:, :4 * C] += r1
    assert _rel(g1, want1) < 2e-6
    assert _rel(acc, r2 + 2 * ref2) < 2e-6
    check_device_status(dev)
