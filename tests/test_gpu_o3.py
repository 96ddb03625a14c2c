"""GPU parity of the sm_100a kernels (torch ops and the raw C ABI) against the reference.

float64: against the reference's golden vectors at the reference's own tolerances
(1e-12 forward / backward, 1e-10 second derivatives). float32: against the oracle in
float64 with fp32 tolerances. Larger convolutions check size-independent
properties (linearity in the weights, invariance to the edge order of a receiver).
"""

import pytest
import torch

import abi_calls as A
from flashcart_b200 import _native as N
from flashcart_b200 import o3
from flashcart_b200.ops import check_device_status
from oracle import stf_oracle as O

pytestmark = pytest.mark.gpu


def _tp_keys(golden):
    return sorted({k.rsplit("/", 1)[0] for k in golden if k.startswith("tp/")})


def _dev(golden, key, dev):
    t = golden.get(key)
    return None if t is None else t.to(dev)


def _second_order(fn, leaves, g, tangents):
    leaves = [t.detach().clone().requires_grad_(True) for t in leaves]
    g_leaf = g.detach().clone().requires_grad_(True)
    out = fn(*leaves)
    grads = torch.autograd.grad(out, leaves, g_leaf, create_graph=True, allow_unused=True)
    s = sum((gr * v).sum() for gr, v in zip(grads, tangents) if gr is not None)
    second = torch.autograd.grad(s, leaves + [g_leaf], allow_unused=True)
    second = [torch.zeros_like(t) if d is None else d for t, d in zip(leaves + [g_leaf], second)]
    grads = [torch.zeros_like(l) if gr is None else gr for l, gr in zip(leaves, grads)]
    return out.detach(), [x.detach() for x in grads], second


def test_gpu_tensor_products_match_reference_golden(golden, cuda_device):
    dev = cuda_device
    for key in _tp_keys(golden):
        l1, l2, lo, f1, f2, sym, shared, red, conv = [int(v) for v in golden[key + "/meta"]]
        tp = o3.TensorProduct(l1, l2, lo, f1, f2, symmetric_product=bool(sym), shared_weights=bool(shared),
                              reduce_paths=bool(red))
        idx_i, idx_j = _dev(golden, key + "/idx_i", dev), _dev(golden, key + "/idx_j", dev)
        names = ("in1", "w") if sym else ("in1", "in2", "w")
        leaves = [golden[f"{key}/{n}"].to(dev) for n in names]
        tangents = [golden[f"{key}/tan_{n}"].to(dev) for n in names]
        if sym:
            fn = lambda a, w: tp(a, a, w, idx_i, idx_j)  # noqa: E731
        else:
            fn = lambda a, b, w: tp(a, b, w, idx_i, idx_j)  # noqa: E731
        out, grads, second = _second_order(fn, leaves, golden[key + "/g"].to(dev), tangents)
        assert (out.cpu() - golden[key + "/out"]).abs().max() < 1e-12, key
        for n, gr in zip(names, grads):
            assert (gr.cpu() - golden[f"{key}/grad_{n}"]).abs().max() < 1e-12, (key, n)
        for n, d in zip(names + ("g",), second):
            assert (d.cpu() - golden[f"{key}/dd_{n}"]).abs().max() < 1e-10, (key, "dd", n)
    check_device_status(dev)


@pytest.mark.parametrize("l", range(4))
def test_gpu_irreps_match_reference_golden(golden, cuda_device, l):
    k = f"irreps/l{l}"
    ir = o3.Irreps(l)
    fn = lambda a: ir.forward_normalized(a) + 0.0 * a.sum()  # noqa: E731
    out, grads, second = _second_order(fn, [golden[k + "/x"].to(cuda_device)], golden[k + "/g"].to(cuda_device),
                                       [golden[k + "/tan_x"].to(cuda_device)])
    assert (out.cpu() - golden[k + "/out"]).abs().max() < 1e-12
    assert (grads[0].cpu() - golden[k + "/grad_x"]).abs().max() < 1e-12
    assert (second[0].cpu() - golden[k + "/dd_x"]).abs().max() < 1e-10
    assert (second[1].cpu() - golden[k + "/dd_g"]).abs().max() < 1e-10


def test_gpu_linear_matches_reference_golden(golden, cuda_device):
    names = sorted({k.split("/")[1] for k in golden if k.startswith("linear/")})
    for name in names:
        k = f"linear/{name}"
        meta = [int(v) for v in golden[k + "/meta"]]
        li, lo, fi, fo, has_ws = meta[:5]
        paths = meta[5:]
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.float64)  # scales computed in float64, as in the reference's fp64 tests
        try:
            lin = o3.LinearLayer(li, lo, fi, fo, in_paths=paths, weight_scale=1.0 if has_ws == 1 else None)
        finally:
            torch.set_default_dtype(prev)
        lin = lin.to(cuda_device, torch.float64)
        common = min(li, lo)
        ws = [golden[f"{k}/w{l}"].to(cuda_device) for l in range(common + 1)]
        with torch.no_grad():
            for l in range(common + 1):
                lin.weight[l].copy_(ws[l])
        x = golden[k + "/x"].to(cuda_device).requires_grad_(True)
        g = golden[k + "/g"].to(cuda_device).requires_grad_(True)
        out = lin(x)
        assert (out.detach().cpu() - golden[k + "/out"]).abs().max() < 1e-12, name
        params = list(lin.weight)
        grads = torch.autograd.grad(out, [x] + params, g, create_graph=True)
        assert (grads[0].detach().cpu() - golden[k + "/grad_x"]).abs().max() < 1e-12, name
        for l in range(common + 1):
            assert (grads[1 + l].detach().cpu() - golden[f"{k}/grad_w{l}"]).abs().max() < 1e-12, (name, l)
        tangents = [golden[k + "/tan_x"].to(cuda_device)] + [golden[f"{k}/tan_w{l}"].to(cuda_device)
                                                            for l in range(common + 1)]
        s = sum((gr * v).sum() for gr, v in zip(grads, tangents))
        second = torch.autograd.grad(s, [x] + params + [g])
        assert (second[0].cpu() - golden[k + "/dd_x"]).abs().max() < 1e-10, name
        for l in range(common + 1):
            assert (second[1 + l].cpu() - golden[f"{k}/dd_w{l}"]).abs().max() < 1e-10, (name, l)
        assert (second[-1].cpu() - golden[k + "/dd_g"]).abs().max() < 1e-10, name


def test_gpu_raw_c_abi_matches_golden(golden, cuda_device):
    """The C entry points called directly with device pointers (no torch operator layer)."""
    lib = N.lib()
    for key in ("tp/l3x3to3_f21/conv", "tp/l3x3to3_f22_shared_reduce/dense", "tp/l2x2to2_f41/conv"):
        m = [int(v) for v in golden[key + "/meta"]]
        t = {n: golden[f"{key}/{n}"].to(cuda_device) for n in ("in1", "in2", "w", "g")}
        idx_i, idx_j = _dev(golden, key + "/idx_i", cuda_device), _dev(golden, key + "/idx_j", cuda_device)
        status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
        out = A.tp_fwd(lib, m, t["in1"], t["in2"], t["w"], idx_i, idx_j, status)
        g1, g2, gw = A.tp_bwd(lib, m, t["g"], t["in1"], t["in2"], t["w"], idx_i, idx_j, status=status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert (out.cpu() - golden[key + "/out"]).abs().max() < 1e-12, key
        assert (g1.cpu() - golden[key + "/grad_in1"]).abs().max() < 1e-12, key
        assert (g2.cpu() - golden[key + "/grad_in2"]).abs().max() < 1e-12, key
        assert (gw.cpu() - golden[key + "/grad_w"]).abs().max() < 1e-12, key


def _conv_inputs(n_nodes, n_edges, C, l1, l2, seed, dtype, dev):
    g = torch.Generator().manual_seed(seed)
    idx_i = torch.sort(torch.randint(0, n_nodes, (n_edges,), generator=g)).values
    idx_j = torch.randint(0, n_nodes, (n_edges,), generator=g)
    in1 = torch.randn(n_nodes, (l1 + 1) ** 2 * C, generator=g, dtype=torch.float64)
    r = torch.nn.functional.normalize(torch.randn(n_edges, 3, generator=g, dtype=torch.float64), dim=-1)
    in2 = O.irreps(r, l2)
    return [t.to(dev) for t in (idx_i, idx_j)] + [t.to(dev, dtype) for t in (in1, in2)]


@pytest.mark.parametrize("sig", [(2, 2, 2, 64), (3, 3, 3, 128), (0, 3, 3, 128), (2, 3, 3, 32), (2, 2, 2, 256),
                                 (1, 2, 2, 64), (3, 3, 3, 64), (3, 3, 2, 128), (1, 3, 3, 192)])
def test_gpu_fp32_convolution_vs_oracle(cuda_device, sig):
    l1, l2, lo, C = sig
    dev = cuda_device
    n_nodes, n_edges = 96, 1536
    idx_i, idx_j, in1, in2 = _conv_inputs(n_nodes, n_edges, C, l1, l2, 3, torch.float32, dev)
    tp = o3.TensorProduct(l1, l2, lo, C, 1)
    w = torch.randn(n_edges, tp.n_total_paths * C, device=dev)
    leaves = [in1.requires_grad_(True), in2.requires_grad_(True), w.requires_grad_(True)]
    out = tp(*leaves, idx_i, idx_j)
    g = torch.randn_like(out)
    grads = torch.autograd.grad(out, leaves, g)
    ref_leaves = [t.detach().double().cpu().requires_grad_(True) for t in leaves]
    ref = O.tensor_product(*ref_leaves, idx_i.cpu(), idx_j.cpu(), l1, l2, lo, C, 1)
    ref_grads = torch.autograd.grad(ref, ref_leaves, g.double().cpu())
    scale = ref.abs().max().item()
    # fp32 accumulation over ~16 edges x tens of paths: relative 1e-5 of the output range
    assert (out.detach().double().cpu() - ref).abs().max().item() < 2e-5 * scale
    for a, b in zip(grads, ref_grads):
        assert (a.double().cpu() - b).abs().max().item() < 2e-5 * b.abs().max().item()
    check_device_status(dev)


def test_gpu_convolution_linearity_and_edge_order_at_size(cuda_device):
    """Config-1 shapes (E = 2^20 edges, N = 2^16 nodes, C = 64, (2,2)->2): properties that need no oracle."""
    dev = cuda_device
    n_nodes, n_edges, C = 65536, 1048576, 64
    idx_i, idx_j, in1, in2 = _conv_inputs(n_nodes, n_edges, C, 2, 2, 11, torch.float32, dev)
    tp = o3.TensorProduct(2, 2, 2, C, 1)
    w1 = torch.randn(n_edges, tp.n_total_paths * C, device=dev)
    w2 = torch.randn_like(w1)
    with torch.no_grad():
        a = tp(in1, in2, w1, idx_i, idx_j)
        b = tp(in1, in2, w2, idx_i, idx_j)
        ab = tp(in1, in2, 0.5 * w1 - 2.0 * w2, idx_i, idx_j)
        assert (ab - (0.5 * a - 2.0 * b)).abs().max().item() < 1e-4 * ab.abs().max().item()
        # reverse the edge order inside every receiver segment: same sums up to rounding
        perm = torch.arange(n_edges, device=dev)
        key = idx_i * n_edges + (n_edges - 1 - perm)
        order = torch.argsort(key)
        c = tp(in1, in2[order], w1[order], idx_i[order], idx_j[order])
        assert (c - a).abs().max().item() < 1e-4 * a.abs().max().item()
    check_device_status(dev)


@pytest.mark.parametrize("C", [64, 128])
def test_gpu_out_of_range_sender_is_reported_and_skipped(cuda_device, C):
    """A sender index past in1's rows: flagged in the status word, the edge contributes
    nothing (forward and backward), every other edge as usual."""
    dev = cuda_device
    n_nodes, n_edges = 40, 600
    idx_i, idx_j, in1, in2 = _conv_inputs(n_nodes, n_edges, C, 2, 2, 5, torch.float32, dev)
    tp = o3.TensorProduct(2, 2, 2, C, 1)
    w = torch.randn(n_edges, tp.n_total_paths * C, device=dev)
    bad = idx_j.clone()
    bad[123] = n_nodes + 7
    check_device_status(dev)
    leaves = [in1.requires_grad_(True), in2.requires_grad_(True), w.requires_grad_(True)]
    out = tp(*leaves, idx_i, bad)
    g = torch.randn_like(out)
    grads = torch.autograd.grad(out, leaves, g)
    with pytest.raises(RuntimeError):
        check_device_status(dev)
    keep = torch.ones(n_edges, dtype=torch.bool, device=dev)
    keep[123] = False
    ref_leaves = [t.detach().double().cpu().requires_grad_(True) for t in leaves]
    w_ref = ref_leaves[2] * keep.cpu().double().unsqueeze(1)
    ref = O.tensor_product(ref_leaves[0], ref_leaves[1], w_ref, idx_i.cpu(), idx_j.cpu(), 2, 2, 2, C, 1)
    assert (out.detach().double().cpu() - ref).abs().max().item() < 2e-5 * ref.abs().max().item()
    ref_g1 = torch.autograd.grad(ref, ref_leaves[0], g.double().cpu())[0]
    assert (grads[0].double().cpu() - ref_g1).abs().max().item() < 2e-5 * ref_g1.abs().max().item()
    check_device_status(dev)


def test_gpu_unsorted_receivers_are_reported(cuda_device):
    dev = cuda_device
    tp = o3.TensorProduct(1, 1, 1, 4, 1)
    in1 = torch.randn(5, tp.in1_dim, device=dev)
    in2 = torch.randn(4, tp.in2_dim, device=dev)
    w = torch.randn(4, tp.n_total_paths * 4, device=dev)
    idx_i = torch.tensor([0, 3, 1, 2], device=dev)
    idx_j = torch.tensor([1, 2, 3, 4], device=dev)
    check_device_status(dev)
    tp(in1, in2, w, idx_i, idx_j)
    with pytest.raises(RuntimeError, match="receiver-sorted"):
        check_device_status(dev)


def test_gpu_cpu_tensors_raise(cuda_device):
    tp = o3.TensorProduct(1, 1, 1, 4, 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        tp(torch.randn(3, tp.in1_dim), torch.randn(3, tp.in2_dim), torch.randn(3, tp.n_total_paths * 4))


@pytest.mark.parametrize("shape", [(3, 3, 128, 128, [4, 6, 7, 6], 300), (2, 2, 64, 64, [1, 1, 1], 1000),
                                   (3, 1, 20, 5, [1, 2, 1, 3], 77), (1, 3, 200, 136, None, 129)])
def test_gpu_fp32_linear_tensor_cores_vs_float64(cuda_device, shape):
    """fp32 linear maps run on tcgen05 as 3xTF32: fp32-level agreement with float64."""
    li, lo, fi, fo, paths, n = shape
    torch.manual_seed(5)
    lin = o3.LinearLayer(li, lo, fi, fo, in_paths=paths).to(cuda_device)
    x = torch.randn(n, lin.in_dim, device=cuda_device, requires_grad=True)
    out = lin(x)
    g = torch.randn_like(out)
    (gx,) = torch.autograd.grad(out, [x], g)
    ws = [w.detach().double().cpu() for w in lin.weight]
    xd = x.detach().double().cpu().requires_grad_(True)
    scales = [float(s) for s in lin.scale.cpu()]
    ref = O.linear(xd, ws, li, lo, fi, fo, paths, scales=scales)
    (rgx,) = torch.autograd.grad(ref, [xd], g.double().cpu())
    err = (out.detach().double().cpu() - ref).abs().max().item()
    assert err < 2e-5 * max(1.0, ref.abs().max().item()), err
    err_g = (gx.double().cpu() - rgx).abs().max().item()
    assert err_g < 2e-5 * max(1.0, rgx.abs().max().item()), err_g
    check_device_status(cuda_device)


@pytest.mark.parametrize("shape", [(64, 2944, 1000), (8, 64, 4099), (2944, 64, 300), (64, 64, 129), (7, 50, 77),
                                   (96, 200, 3001), (128, 416, 777)])
def test_gpu_fp32_dense_layer_shapes_vs_float64(cuda_device, shape):
    """Radial-MLP shapes (edge rows x 64 -> paths*F and back) on the TMA-fed tensor-core GEMM."""
    from flashcart_b200.nn.layers import LinearLayer

    k, n, rows = shape
    torch.manual_seed(11)
    lay = LinearLayer(k, n).to(cuda_device)
    x = torch.randn(rows, k, device=cuda_device, requires_grad=True)
    out = lay(x)
    g = torch.randn_like(out)
    (gx,) = torch.autograd.grad(out, [x], g)
    w = lay.weight.detach().double().cpu()
    sc = float(lay.scale)
    xd = x.detach().double().cpu()
    ref = sc * xd @ w.t()
    rgx = sc * g.double().cpu() @ w
    err = (out.detach().double().cpu() - ref).abs().max().item()
    assert err < 2e-5 * max(1.0, ref.abs().max().item()), err
    err_g = (gx.double().cpu() - rgx).abs().max().item()
    assert err_g < 2e-5 * max(1.0, rgx.abs().max().item()), err_g
    check_device_status(cuda_device)


def test_gpu_tf32_mode_is_single_tf32_product(cuda_device):
    """With TF32 matmuls allowed (the reference's "tf32" dot precision) one tf32 product is used."""
    torch.manual_seed(6)
    lin = o3.LinearLayer(2, 2, 128, 128).to(cuda_device)
    x = torch.randn(512, lin.in_dim, device=cuda_device)
    exact = lin(x)
    prev = (torch.backends.cuda.matmul.allow_tf32, torch.get_float32_matmul_precision())
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.set_float32_matmul_precision("high")
    try:
        fast = lin(x)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev[0]
        torch.set_float32_matmul_precision(prev[1])
    rel = ((fast - exact).abs().max() / exact.abs().max()).item()
    # reference tolerance for its tf32 path: atol 3e-3 / rtol 2e-3 (tests/o3/test_linear.py:37)
    assert 0 < rel < 3e-3, rel


@pytest.mark.parametrize("sig", [(3, 3, 3, 32), (2, 2, 2, 64), (0, 3, 3, 32), (1, 2, 2, 96), (3, 2, 1, 32),
                                 (3, 3, 3, 64), (2, 3, 3, 128)])
def test_gpu_fp64_shared_attribute_convolution_vs_oracle(cuda_device, sig):
    """The shared-edge-attribute convolution kernels (path groups, edge matrices in shared
    memory) in float64 against the oracle, forward and all three gradients. (3,3,3,64) and
    (2,3,3,128) are split into path groups with a channel count divisible by 64, so their
    forward runs two channels per thread."""
    l1, l2, lo, C = sig
    dev = cuda_device
    idx_i, idx_j, in1, in2 = _conv_inputs(40, 700, C, l1, l2, 9, torch.float64, dev)
    tp = o3.TensorProduct(l1, l2, lo, C, 1)
    w = torch.randn(700, tp.n_total_paths * C, device=dev, dtype=torch.float64)
    leaves = [in1.requires_grad_(True), in2.requires_grad_(True), w.requires_grad_(True)]
    out = tp(*leaves, idx_i, idx_j)
    g = torch.randn_like(out)
    grads = torch.autograd.grad(out, leaves, g)
    ref_leaves = [t.detach().cpu().requires_grad_(True) for t in leaves]
    ref = O.tensor_product(*ref_leaves, idx_i.cpu(), idx_j.cpu(), l1, l2, lo, C, 1)
    ref_grads = torch.autograd.grad(ref, ref_leaves, g.cpu())
    assert (out.detach().cpu() - ref).abs().max().item() < 1e-11 * max(1.0, ref.abs().max().item())
    for a, b in zip(grads, ref_grads):
        assert (a.cpu() - b).abs().max().item() < 1e-11 * max(1.0, b.abs().max().item())
    check_device_status(dev)


def test_gpu_split_weight_cache_follows_in_place_updates(cuda_device):
    """Frozen float32 weights are split into tf32 hi / lo once and reused; an in-place
    update of the weights (a new _version) must be seen by the next forward and backward."""
    from flashcart_b200 import o3 as O3

    torch.manual_seed(2)
    lin = O3.LinearLayer(2, 2, 64, 64).to(cuda_device)
    for p in lin.parameters():
        p.requires_grad_(False)
    x = torch.randn(500, 9 * 64, device=cuda_device, requires_grad=True)

    def check():
        y = lin(x)
        (g,) = torch.autograd.grad(y.square().sum(), [x])
        xr = x.detach().double().cpu().requires_grad_(True)
        yr = O.linear(xr, [w.double().cpu() for w in lin.weight], 2, 2, 64, 64)
        (gr,) = torch.autograd.grad(yr.square().sum(), [xr])
        assert (y.detach().double().cpu() - yr).abs().max().item() < 2e-5 * yr.abs().max().item()
        assert (g.double().cpu() - gr).abs().max().item() < 2e-5 * gr.abs().max().item()
        return y.detach()

    y1 = check()
    assert torch.equal(y1, lin(x).detach())  # the cached split gives the same result
    with torch.no_grad():
        for w in lin.weight:
            w.mul_(-0.5).add_(0.1)
    y2 = check()
    assert not torch.equal(y1, y2)
    check_device_status(cuda_device)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("sig", [(2, 2, 2, 64), (3, 3, 3, 32), (0, 3, 3, 128)])
def test_gpu_convolution_without_edges(cuda_device, sig, dtype):
    """Isolated atoms only (E = 0): zero messages, zero first and second derivatives, the
    per-edge gradients with no rows; the reference's gather / scatter_sum does the same."""
    l1, l2, lo, C = sig
    dev = cuda_device
    tp = o3.TensorProduct(l1, l2, lo, C, 1)
    in1 = torch.randn(7, tp.in1_dim, device=dev, dtype=dtype)
    in2 = torch.zeros(0, tp.in2_dim, device=dev, dtype=dtype)
    w = torch.zeros(0, tp.n_total_paths * C, device=dev, dtype=dtype)
    idx = torch.zeros(0, dtype=torch.int64, device=dev)
    leaves = [in1, in2, w]
    tangents = [torch.randn_like(t) for t in leaves]
    out = tp(in1, in2, w, idx, idx)
    g = torch.randn_like(out)
    out, grads, second = _second_order(lambda a, b, c: tp(a, b, c, idx, idx), leaves, g, tangents)
    assert out.shape[0] == 7 and (out == 0).all()
    assert all((t == 0).all() and t.shape == l.shape for t, l in zip(grads, leaves))
    assert all((t == 0).all() for t in second)
    check_device_status(dev)


def _ragged_inputs(degrees, C, l1, l2, seed, dtype, dev):
    g = torch.Generator().manual_seed(seed)
    n_nodes = len(degrees)
    idx_i = torch.repeat_interleave(torch.arange(n_nodes), torch.tensor(degrees))
    idx_j = torch.randint(0, n_nodes, (idx_i.numel(),), generator=g)
    in1 = torch.randn(n_nodes, (l1 + 1) ** 2 * C, generator=g, dtype=torch.float64)
    r = torch.nn.functional.normalize(torch.randn(idx_i.numel(), 3, generator=g, dtype=torch.float64), dim=-1)
    in2 = O.irreps(r, l2)
    return [t.to(dev) for t in (idx_i, idx_j)] + [t.to(dev, dtype) for t in (in1, in2)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("sig", [(3, 3, 3, 128), (0, 3, 3, 128), (2, 2, 2, 64), (2, 3, 3, 32)])
def test_gpu_convolution_ragged_degrees_vs_oracle(cuda_device, sig, dtype):
    """Isolated receivers first, last and in between, one receiver with 1,500 edges (many
    edge chunks through the prefetch ring), the rest of degree 1-5: forward and all three
    gradients against the oracle in float64."""
    l1, l2, lo, C = sig
    dev = cuda_device
    g = torch.Generator().manual_seed(11)
    degrees = torch.randint(1, 6, (60,), generator=g)
    degrees[[0, 1, 17, 30, 31, 58, 59]] = 0
    degrees[23] = 1500
    degrees = degrees.tolist()
    idx_i, idx_j, in1, in2 = _ragged_inputs(degrees, C, l1, l2, 12, dtype, dev)
    tp = o3.TensorProduct(l1, l2, lo, C, 1)
    w = torch.randn(idx_i.numel(), tp.n_total_paths * C, device=dev, dtype=dtype)
    leaves = [in1.requires_grad_(True), in2.requires_grad_(True), w.requires_grad_(True)]
    out = tp(*leaves, idx_i, idx_j)
    gout = torch.randn_like(out)
    grads = torch.autograd.grad(out, leaves, gout)
    ref_leaves = [t.detach().double().cpu().requires_grad_(True) for t in leaves]
    ref = O.tensor_product(*ref_leaves, idx_i.cpu(), idx_j.cpu(), l1, l2, lo, C, 1)
    ref_grads = torch.autograd.grad(ref, ref_leaves, gout.double().cpu())
    # float32: the 1,500-edge receiver sums ~1e3 terms, so a larger relative bound than 2e-5
    tol = 1e-11 if dtype == torch.float64 else 1e-4
    assert (out.detach().double().cpu() - ref).abs().max().item() < tol * max(1.0, ref.abs().max().item())
    for node, deg in enumerate(degrees):
        if deg == 0:
            assert (out[node] == 0).all()
    for a, b in zip(grads, ref_grads):
        assert (a.double().cpu() - b).abs().max().item() < tol * max(1.0, b.abs().max().item())
    check_device_status(dev)


def test_gpu_raw_c_abi_linear_double_backward(golden, cuda_device):
    """fc_linear_dbwd through the C ABI: float64 against the reference's VJP-of-VJP at its
    1e-10 tolerance; float32 (3xTF32 GEMMs, a pool workspace for the two-tangent sum)
    against the float64 result."""
    lib = N.lib()
    for name in sorted({k.split("/")[1] for k in golden if k.startswith("linear/")}):
        k = f"linear/{name}"
        meta = [int(v) for v in golden[k + "/meta"]]
        li, lo, fi, fo, has_ws = meta[:5]
        paths = meta[5:]
        common = min(li, lo)
        scale = torch.tensor([1.0 if has_ws == 1 else (fi * paths[l]) ** -0.5 for l in range(common + 1)],
                             dtype=torch.float64)
        for dtype in (torch.float64, torch.float32):
            dev = lambda t: t.to(cuda_device, dtype)  # noqa: E731
            ws = [dev(golden[f"{k}/w{l}"]) for l in range(common + 1)]
            vws = [dev(golden[f"{k}/tan_w{l}"]) for l in range(common + 1)]
            d = A.linear_desc(li, lo, fi, fo, paths, dtype)
            dg, dx, dws = A.linear_dbwd(lib, d, dev(golden[k + "/g"]), dev(golden[k + "/x"]), ws,
                                        dev(golden[k + "/tan_x"]), vws, dev(scale))
            pairs = [(dg, golden[k + "/dd_g"]), (dx, golden[k + "/dd_x"])]
            pairs += [(dws[l], golden[f"{k}/dd_w{l}"]) for l in range(common + 1)]
            for got, ref in pairs:
                err = (got.double().cpu() - ref).abs().max().item()
                bound = 1e-10 if dtype == torch.float64 else 2e-5 * max(1.0, ref.abs().max().item())
                assert err < bound, (name, dtype, err)
    check_device_status(cuda_device)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_gpu_raw_c_abi_halo_pack_and_unpack(cuda_device, dtype):
    """Row gather / copy / atomic row sum at feature width 2048 (l <= 3, C = 128) over
    tens of thousands of rows, against index_select / index_copy / index_add; a bad index
    is flagged in the status word and skipped."""
    lib = N.lib()
    g = torch.Generator().manual_seed(4)
    x = torch.randn(30000, 2048, generator=g).to(cuda_device, dtype)
    send = torch.randint(0, 30000, (12000,), generator=g).to(cuda_device)
    buf = A.halo_pack(lib, x, send)
    assert torch.equal(buf, x.index_select(0, send))
    ghosts = torch.randperm(30000, generator=g)[:12000].to(cuda_device)
    y = x.clone()
    A.halo_unpack(lib, buf, ghosts, y, accumulate=False)
    assert torch.equal(y, x.index_copy(0, ghosts, buf))
    owners = torch.randint(0, 500, (12000,), generator=g).to(cuda_device)  # ~24 contributions per owner
    acc = torch.zeros(500, 2048, device=cuda_device, dtype=dtype)
    A.halo_unpack(lib, buf, owners, acc, accumulate=True)
    ref = torch.zeros_like(acc).index_add_(0, owners, buf)
    tol = 1e-5 if dtype == torch.float32 else 1e-12
    assert (acc - ref).abs().max().item() < tol * ref.abs().max().item()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    A.halo_pack(lib, x, torch.tensor([1, 30000], device=cuda_device), status)
    torch.cuda.synchronize()
    assert int(status.item()) & N.FC_DEV_BAD_INDEX


@pytest.mark.parametrize("case", [(3, 3, 3, 8, "conv", False, False), (2, 3, 3, 4, "conv", False, False),
                                  (0, 3, 3, 4, "conv", False, False), (3, 3, 3, 4, "dense", False, True),
                                  (2, 2, 2, 4, "dense", True, False), (3, 3, 2, 8, "dense", False, False)])
def test_gpu_rotation_equivariance(cuda_device, case):
    """TP(R in1, R in2) = R TP(in1, in2) on the kernels, float64, for convolutions and dense
    products (symmetric, path-reduced), as the reference's
    ``tests/o3/test_tensor_product.py:326-349`` checks it (atol 1e-10)."""
    from flashcart_b200.o3.utils import rotate_irreps

    l1, l2, lo, C, kind, sym, red = case
    dev, f64 = cuda_device, torch.float64
    conv = kind == "conv"
    tp = o3.TensorProduct(l1, l2, lo, C, 1 if conv else C, symmetric_product=sym, reduce_paths=red)
    g = torch.Generator().manual_seed(3)
    n, e = 30, 240
    in1 = torch.randn(n, tp.in1_dim, generator=g, dtype=f64)
    if conv:
        idx_i = torch.sort(torch.randint(0, n, (e,), generator=g)).values.to(dev)
        idx_j = torch.randint(0, n, (e,), generator=g).to(dev)
        in2 = O.irreps(torch.nn.functional.normalize(torch.randn(e, 3, generator=g, dtype=f64), dim=-1), l2)
        w = torch.randn(e, tp.n_total_paths * C, generator=g, dtype=f64)
    else:
        idx_i = idx_j = None
        in2 = in1 if sym else torch.randn(n, tp.in2_dim, generator=g, dtype=f64)
        w = torch.randn(n, tp.n_total_paths * C, generator=g, dtype=f64)
    q, r = torch.linalg.qr(torch.randn(3, 3, generator=g, dtype=f64))
    R = q * torch.sign(torch.diagonal(r))
    in1_r = rotate_irreps(in1, R, l1)
    in2_r = in1_r if sym else rotate_irreps(in2, R, l2)
    with torch.no_grad():
        out = tp(in1.to(dev), in2.to(dev), w.to(dev), idx_i, idx_j).cpu()
        out_r = tp(in1_r.to(dev), in2_r.to(dev), w.to(dev), idx_i, idx_j).cpu()
    n_paths = [min(1, p) for p in tp.out_paths] if red else tp.out_paths
    expect = rotate_irreps(out, R, lo, n_paths=n_paths)
    assert (out_r - expect).abs().max().item() < 1e-10 * max(1.0, expect.abs().max().item())
    assert out.abs().max().item() > 1e-3
    check_device_status(dev)


@pytest.mark.parametrize("nodes", [3000, 129, 1])
def test_gpu_bf16_linear_map_storage_path(cuda_device, nodes):
    """bf16 storage path of the equivariant linear map (fc_linear_fwd with FC_BF16: tcgen05
    kind::f16, fp32 accumulation, one bf16 rounding of the result): against the float64 map
    of the same bf16-rounded inputs (only the output rounding and the fp32 accumulation
    differ) and against the float32 map (bf16 input rounding included). Tolerances: 2^-8
    relative to the output scale (one bf16 rounding), 2e-2 for the float32 comparison."""
    torch.manual_seed(nodes)
    lin = o3.LinearLayer(3, 3, 128, 128, weight_scale=1.0).to(cuda_device)
    with torch.no_grad():
        for w in lin.weight:
            w.normal_(0.0, (2.0 / 256) ** 0.5)
    x = torch.randn(nodes, 16 * 128, device=cuda_device)
    with torch.no_grad():
        y32 = lin(x)
        xb = x.to(torch.bfloat16)
        yb = lin(xb)
        assert yb.dtype == torch.bfloat16 and yb.shape == y32.shape
        lin64 = o3.LinearLayer(3, 3, 128, 128, weight_scale=1.0).to(cuda_device, torch.float64)
        for w64, w in zip(lin64.weight, lin.weight):
            w64.copy_(w.to(torch.bfloat16).double())
        y64 = lin64(xb.double())
    scale = float(y64.abs().max())
    assert float((yb.double() - y64).abs().max()) <= 2.0 ** -8 * scale
    assert float((yb.float() - y32).abs().max()) <= 2e-2 * float(y32.abs().max())
    check_device_status(cuda_device)


def test_gpu_bf16_linear_rejects_unaligned_and_backward(cuda_device):
    lin = o3.LinearLayer(1, 1, 12, 12).to(cuda_device)  # 12 channels: rows not 16-byte multiples
    x = torch.randn(10, 4 * 12, device=cuda_device, dtype=torch.bfloat16)
    with torch.no_grad(), pytest.raises(NotImplementedError):
        lin(x)
    lin2 = o3.LinearLayer(1, 1, 16, 16).to(cuda_device)
    x2 = torch.randn(10, 4 * 16, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    y = lin2(x2)
    with pytest.raises(NotImplementedError):
        y.sum().backward()


@pytest.mark.parametrize("widths", [[8, 64, 64, 2944], [256, 64, 64, 1]])
def test_gpu_mlp_silu_inside_gemm_equals_composed(cuda_device, widths):
    """The radial / readout MLP with each SiLU applied inside the next layer's GEMM (its
    splitter warps) and SiLU' in the input gradient's epilogue (first-order evaluation,
    frozen weights) equals the composed SiLU passes: output and input gradient within
    float32 rounding of the 3xTF32 GEMMs."""
    from flashcart_b200 import ops
    from flashcart_b200.nn.layers import _mlp

    torch.manual_seed(len(widths) + widths[0])
    mlp = _mlp(widths).to(cuda_device)
    for p in mlp.parameters():
        p.requires_grad_(False)
    x = torch.randn(20000, widths[0], device=cuda_device)
    go = torch.randn(20000, widths[-1], device=cuda_device)
    xa = x.clone().requires_grad_(True)
    ya = mlp(xa)
    (ga,) = torch.autograd.grad(ya, xa, go)
    xb = x.clone().requires_grad_(True)
    timer = ops.KernelTimer()
    ops.set_kernel_timer(timer)
    try:
        with ops.first_order_only():
            yb = mlp(xb)
            (gb,) = torch.autograd.grad(yb, xb, go)
    finally:
        ops.set_kernel_timer(None)
    names = [r[0] for r in timer.records]
    assert names.count("linear_fwd") == 3 and names.count("linear_bwd") == 3
    fused = sum(1 for m in mlp if hasattr(m, "silu_input_fusable") and m.out_features % 4 == 0) - 1
    assert fused >= 1
    assert float((ya - yb).abs().max() / ya.abs().max()) < 2e-5
    assert float((ga - gb).abs().max() / ga.abs().max()) < 2e-5
    check_device_status(cuda_device)
