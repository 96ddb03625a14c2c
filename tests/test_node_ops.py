"""Fused node-level operators: RMS layer norm (fc_rms_norm_*, flashcart::rms_norm_*) and
the equivariant gate (fc_gate_*, flashcart::gate_*).

The fused kernels replace compositions of the reference when the graph is
differentiated once: RMSLayerNorm (nn/layers.py:413-540: symmetric scalar tensor
product of the features with themselves, per-rank weights 1/((2l+1)(l_max+1)), channel
mean, (mean_sq + eps)^-1/2, per-rank gains) and the per-rank gating products of
EquivariantGatedLayer (nn/layers.py:609-635). The oracles are those compositions (on the
oracle tensor product), differentiated by autograd.
"""

import ctypes

import pytest
import torch

import abi_calls as A
from flashcart_b200 import _native as N
from oracle import stf_oracle as O


def _composed(x, gains, l_max, C, eps):
    """RMSLayerNorm.forward of the reference, on the oracle tensor product (float64)."""
    n = x.shape[0]
    npaths = l_max + 1
    ones = torch.ones(npaths * C, dtype=x.dtype)
    inv = O.tensor_product(x, x, ones, None, None, l_max, l_max, 0, C, C, True, True, False).view(n, l_max + 1, C)
    lw = torch.tensor([1.0 / ((2 * l + 1) * (l_max + 1)) for l in range(l_max + 1)], dtype=torch.float64)
    mean_sq = (inv * lw.to(inv.dtype).view(1, -1, 1)).sum(1).mean(-1, keepdim=True)
    scaled = x * torch.pow(mean_sq + eps, -0.5)
    g = torch.cat([gains[l].repeat(2 * l + 1) for l in range(l_max + 1)])
    return scaled * g, lw


@pytest.mark.parametrize("l_max,C", [(0, 8), (1, 5), (2, 32), (3, 16)])
def test_emu_rms_norm_matches_composed_oracle(emu_lib, l_max, C):
    g = torch.Generator().manual_seed(7 + l_max)
    n, eps = 9, 1e-6
    x = torch.randn(n, (l_max + 1) ** 2 * C, generator=g, dtype=torch.float64)
    gains = 1.0 + 0.3 * torch.randn(l_max + 1, C, generator=g, dtype=torch.float64)
    xr = x.clone().requires_grad_(True)
    ref, lw = _composed(xr, gains, l_max, C, eps)
    gy = torch.randn_like(ref)
    (ref_gx,) = torch.autograd.grad(ref, [xr], gy)

    y = torch.empty_like(x)
    rstd = torch.empty(n, dtype=torch.float64)
    rc = emu_lib.fc_rms_norm_fwd(l_max, C, N.FC_F64, A.p(x), A.p(gains), A.p(lw), eps, n, A.p(y), A.p(rstd), None)
    N.check(emu_lib, rc, "fc_rms_norm_fwd")
    gx = torch.empty_like(x)
    rc = emu_lib.fc_rms_norm_bwd(l_max, C, N.FC_F64, A.p(gy), A.p(x), A.p(gains), A.p(lw), A.p(rstd), n, A.p(gx),
                                 None)
    N.check(emu_lib, rc, "fc_rms_norm_bwd")
    assert (y - ref.detach()).abs().max().item() < 1e-12 * max(1.0, ref.abs().max().item())
    assert (gx - ref_gx).abs().max().item() < 1e-12 * max(1.0, ref_gx.abs().max().item())


def test_emu_rms_norm_rejects_bad_arguments(emu_lib):
    x = torch.zeros(2, 16 * 4, dtype=torch.float64)
    rc = emu_lib.fc_rms_norm_fwd(4, 4, N.FC_F64, A.p(x), A.p(x), A.p(x), 1e-6, 2, A.p(x), A.p(x), None)
    assert rc == N.FC_ERR_UNSUPPORTED
    rc = emu_lib.fc_rms_norm_fwd(3, 4, 7, A.p(x), A.p(x), A.p(x), 1e-6, 2, A.p(x), A.p(x), None)
    assert rc == N.FC_ERR_INVALID
    rc = emu_lib.fc_rms_norm_bwd(3, 4, N.FC_F64, None, A.p(x), A.p(x), A.p(x), A.p(x), 2, A.p(x), None)
    assert rc == N.FC_ERR_INVALID
    assert b"null" in emu_lib.fc_last_error()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-12), (torch.float32, 2e-6)])
@pytest.mark.parametrize("l_max,C", [(3, 128), (2, 64), (1, 96)])
def test_gpu_fused_rms_norm_matches_composed(cuda_device, dtype, tol, l_max, C):
    """RMSLayerNorm inside first_order_only (fused kernels) against the same module outside
    it (composed tensor-product path), forward and input gradient."""
    from flashcart_b200 import ops
    from flashcart_b200.nn.layers import RMSLayerNorm

    torch.manual_seed(3)
    norm = RMSLayerNorm(l_max, C, eps=1e-6).to(cuda_device, dtype)
    with torch.no_grad():
        for w in norm.weights:
            w.add_(0.3 * torch.randn_like(w))
    for p in norm.parameters():
        p.requires_grad_(False)
    x = torch.randn(1000, (l_max + 1) ** 2 * C, device=cuda_device, dtype=dtype, requires_grad=True)
    gy = torch.randn_like(x)
    ref = norm(x)
    (ref_gx,) = torch.autograd.grad(ref, [x], gy)
    with ops.first_order_only():
        assert norm._fused_ok(x)
        out = norm(x)
        (gx,) = torch.autograd.grad(out, [x], gy)
    ops.check_device_status(cuda_device)
    assert (out - ref).abs().max().item() < tol * ref.abs().max().item()
    assert (gx - ref_gx).abs().max().item() < tol * ref_gx.abs().max().item()


@pytest.mark.gpu
def test_gpu_fused_rms_norm_refuses_second_derivative(cuda_device):
    from flashcart_b200 import ops
    from flashcart_b200.nn.layers import RMSLayerNorm

    norm = RMSLayerNorm(2, 32).to(cuda_device)
    for p in norm.parameters():
        p.requires_grad_(False)
    x = torch.randn(10, 9 * 32, device=cuda_device, requires_grad=True)
    with ops.first_order_only():
        y = norm(x)
        with pytest.raises(RuntimeError, match="second derivative"):
            torch.autograd.grad(y.square().sum(), [x], create_graph=True)


def _gate_composed(values, gates, l_max, H):
    n = values.shape[0]
    parts, a = [], 0
    for l in range(l_max + 1):
        b = a + (2 * l + 1) * H
        parts.append((values[:, a:b].view(n, 2 * l + 1, H) * gates[:, l].unsqueeze(1)).flatten(1))
        a = b
    return torch.cat(parts, dim=-1)


@pytest.mark.parametrize("l_max,H", [(0, 4), (2, 7), (3, 16)])
def test_emu_gate_matches_composition(emu_lib, l_max, H):
    g = torch.Generator().manual_seed(11 + l_max)
    n = 6
    v = torch.randn(n, (l_max + 1) ** 2 * H, generator=g, dtype=torch.float64)
    gt = torch.randn(n, l_max + 1, H, generator=g, dtype=torch.float64)
    vr, gr = v.clone().requires_grad_(True), gt.clone().requires_grad_(True)
    ref = _gate_composed(vr, gr, l_max, H)
    gy = torch.randn_like(ref)
    ref_gv, ref_gg = torch.autograd.grad(ref, [vr, gr], gy)
    y = torch.empty_like(v)
    N.check(emu_lib, emu_lib.fc_gate_fwd(l_max, H, N.FC_F64, A.p(v), A.p(gt), n, A.p(y), None), "fc_gate_fwd")
    gv, gg = torch.empty_like(v), torch.empty_like(gt)
    N.check(emu_lib, emu_lib.fc_gate_bwd(l_max, H, N.FC_F64, A.p(gy), A.p(v), A.p(gt), n, A.p(gv), A.p(gg), None),
            "fc_gate_bwd")
    assert torch.equal(y, ref.detach())
    assert (gv - ref_gv).abs().max().item() < 1e-14 * ref_gv.abs().max().item()
    assert (gg - ref_gg).abs().max().item() < 1e-12 * ref_gg.abs().max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-12), (torch.float32, 2e-6)])
def test_gpu_fused_gated_layer_matches_composed(cuda_device, dtype, tol):
    """EquivariantGatedLayer inside first_order_only (fused gate) against the same layer
    outside it, forward and input gradient."""
    from flashcart_b200 import ops
    from flashcart_b200.nn.layers import EquivariantGatedLayer

    torch.manual_seed(5)
    layer = EquivariantGatedLayer(3, 128, gate_activation="sigmoid").to(cuda_device, dtype)
    with torch.no_grad():
        for w in layer.output_linear.weight:
            w.normal_()
    for p in layer.parameters():
        p.requires_grad_(False)
    x = torch.randn(700, 16 * 128, device=cuda_device, dtype=dtype, requires_grad=True)
    gy = torch.randn_like(x)
    ref = layer(x)
    (ref_gx,) = torch.autograd.grad(ref, [x], gy)
    with ops.first_order_only():
        out = layer(x)
        (gx,) = torch.autograd.grad(out, [x], gy)
    ops.check_device_status(cuda_device)
    assert (out - ref).abs().max().item() < tol * ref.abs().max().item()
    assert (gx - ref_gx).abs().max().item() < tol * ref_gx.abs().max().item()


def _expand_ref(T, h, l_max, C, per_rank):
    blocks, off = [], 0
    for l in range(l_max + 1):
        n = 2 * l + 1
        hl = h[:, l] if per_rank else h
        blocks.append((T[:, off:off + n].unsqueeze(-1) * hl.unsqueeze(1)).reshape(T.shape[0], n * C))
        off += n
    return torch.cat(blocks, dim=-1)


@pytest.mark.parametrize("l_max,C,per_rank", [(3, 8, False), (3, 5, True), (2, 33, True), (0, 4, False)])
def test_emu_edge_expand_matches_composition(emu_lib, l_max, C, per_rank):
    g = torch.Generator().manual_seed(21 + l_max)
    n, nc = 7, (l_max + 1) ** 2
    T = torch.randn(n, nc, generator=g, dtype=torch.float64)
    h = torch.randn(*((n, l_max + 1, C) if per_rank else (n, C)), generator=g, dtype=torch.float64)
    Tr, hr = T.clone().requires_grad_(True), h.clone().requires_grad_(True)
    ref = _expand_ref(Tr, hr, l_max, C, per_rank)
    gy = torch.randn_like(ref)
    ref_gt, ref_gh = torch.autograd.grad(ref, [Tr, hr], gy)
    out = torch.empty_like(ref)
    N.check(emu_lib, emu_lib.fc_edge_expand_fwd(l_max, C, int(per_rank), N.FC_F64, A.p(T), A.p(h), n, A.p(out), None),
            "fc_edge_expand_fwd")
    gt, gh = torch.empty_like(T), torch.empty_like(h)
    N.check(emu_lib, emu_lib.fc_edge_expand_bwd(l_max, C, int(per_rank), N.FC_F64, A.p(gy), A.p(T), A.p(h), n, A.p(gt),
                                                A.p(gh), None), "fc_edge_expand_bwd")
    assert torch.equal(out, ref.detach())
    assert (gt - ref_gt).abs().max().item() < 1e-12 * ref_gt.abs().max().item()
    assert (gh - ref_gh).abs().max().item() < 1e-12 * ref_gh.abs().max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("per_rank", [False, True])
@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-12), (torch.float32, 1e-5)])
def test_gpu_edge_expand_matches_composition(cuda_device, per_rank, dtype, tol):
    """Forward, first derivative (kernels) and second derivative (composed backward)."""
    from flashcart_b200 import ops

    g = torch.Generator(device=cuda_device).manual_seed(4)
    n, L, C = 5000, 3, 128
    T = torch.randn(n, 16, device=cuda_device, dtype=dtype, generator=g, requires_grad=True)
    h = torch.randn(*((n, L + 1, C) if per_rank else (n, C)), device=cuda_device, dtype=dtype, generator=g,
                    requires_grad=True)
    ref = _expand_ref(T, h, L, C, per_rank)
    out = ops.edge_expand_fwd(T, h, L, C, per_rank)
    assert torch.equal(out, ref)
    gy = torch.randn_like(ref)
    r_gt, r_gh = torch.autograd.grad(ref, [T, h], gy, create_graph=True)
    gt, gh = torch.autograd.grad(out, [T, h], gy, create_graph=True)
    assert (gt - r_gt).abs().max().item() < tol * r_gt.abs().max().item()
    assert (gh - r_gh).abs().max().item() < tol * r_gh.abs().max().item()
    (a,) = torch.autograd.grad((gt.square().sum() + gh.square().sum()), [T])
    (b,) = torch.autograd.grad((r_gt.square().sum() + r_gh.square().sum()), [T])
    assert (a - b).abs().max().item() < 10 * tol * b.abs().max().item()
    with torch.no_grad():
        gt1, gh1 = torch.ops.flashcart.edge_expand_bwd(gy, T, h, L, C, per_rank)
    assert (gt1 - r_gt).abs().max().item() < tol * r_gt.abs().max().item()
    assert (gh1 - r_gh).abs().max().item() < tol * r_gh.abs().max().item()
    ops.check_device_status(cuda_device)
