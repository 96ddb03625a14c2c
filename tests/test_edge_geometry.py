"""Fused edge geometry (fc_edge_geometry_fwd / _bwd, flashcart::edge_geometry_fwd) against the
composed chain it replaces.

The reference computes, before its interaction layers (``model/flashcart.py:264-286``):
edge vectors with periodic shifts (``utils/geometry.py:25-53``), distances, directions
``v / max(|v|, 1e-4)``, ``Irreps.forward_normalized`` (``o3/irreps.py:54-72``), the
Chebyshev basis (``nn/radial.py:98-128``) and the polynomial-cutoff envelope
(``nn/radial.py:181-245``), multiplied into the radial-MLP input
(``nn/layers.py:351-356``). The composed float64 reference here is built from this
repository's geometry and radial modules (pinned to the reference's golden values in
``tests/test_radial_golden.py``) and the oracle's direction tensors; gradients come from
autograd through it. Cases: periodic shifts, two cells of one batch, an edge shorter than
1e-4 (clamped direction), edges beyond the cutoff, both Chebyshev mappings.
"""

import ctypes

import pytest
import torch

from flashcart_b200 import _native as N
from flashcart_b200.model.flashcart import get_edge_vectors
from flashcart_b200.nn.radial import ChebyshevBasis, PolynomialCutoff
from oracle import stf_oracle as O

R_MAX = 5.0


def _structure(seed=0, n_per_cell=40, n_cells=2, close_pair=True):
    """Atoms of two periodic cells (a batch), all pairs within 1.3 r_max across 27 images,
    edges beyond the cutoff, and (close_pair) an almost-coincident pair (|v| < 1e-4: the
    direction's clamp; float32 positions of a 10 A cell cannot resolve such a vector, so
    only float64 cases include it)."""
    g = torch.Generator().manual_seed(seed)
    cells = torch.stack([torch.diag(torch.tensor([9.0, 10.0, 11.0], dtype=torch.float64)),
                         torch.tensor([[9.5, 0.3, 0.0], [0.2, 10.5, 0.4], [0.0, 0.5, 11.5]], dtype=torch.float64)])
    cells = cells[:n_cells]
    pos, batch = [], []
    for b in range(n_cells):
        frac = torch.rand(n_per_cell, 3, generator=g, dtype=torch.float64)
        p = frac @ cells[b]
        if b == 0 and close_pair:
            p[1] = p[0] + torch.tensor([3e-5, -2e-5, 1e-5], dtype=torch.float64)
        pos.append(p)
        batch.append(torch.full((n_per_cell,), b, dtype=torch.int64))
    pos, batch = torch.cat(pos), torch.cat(batch)
    rows_i, rows_j, shifts = [], [], []
    rng = torch.arange(-1, 2)
    images = torch.cartesian_prod(rng, rng, rng).to(torch.float64)
    for b in range(n_cells):
        idx = torch.nonzero(batch == b).flatten()
        for i in idx.tolist():
            for j in idx.tolist():
                v = pos[j] - pos[i] + images @ cells[b]
                d = v.norm(dim=-1)
                keep = (d < 1.3 * R_MAX) & ~((i == j) & (d < 1e-12))
                for k in torch.nonzero(keep).flatten().tolist():
                    rows_i.append(i)
                    rows_j.append(j)
                    shifts.append(images[k].to(torch.int32))
    ei = torch.tensor([rows_i, rows_j], dtype=torch.int64)
    return pos, cells, torch.stack(shifts), ei, batch


def _composed(pos, cells, shifts, ei, batch, l_max, n_radial, mapping, p=6, use_shifts=True):
    """The composed chain on the inputs' device; the direction tensors from the oracle (host)."""
    vec = get_edge_vectors(pos, cells, shifts, ei, batch, use_shifts=use_shifts)
    r = vec.norm(dim=-1)
    d = vec / r.clamp_min(1.0e-4).unsqueeze(-1)
    attrs = O.irreps(d.cpu(), l_max)
    basis = ChebyshevBasis(n_radial, r_max=R_MAX, mapping=mapping).to(device=r.device, dtype=pos.dtype)(r)
    env = PolynomialCutoff(R_MAX, poly_order=p).to(device=r.device, dtype=pos.dtype)(r)
    return attrs, (basis * env.unsqueeze(-1)).cpu()


def _desc(l_max, n_radial, mapping, dtype, p=6, use_shifts=True):
    return N.EdgeGeometryDesc(l_max, n_radial, int(mapping == "cosine"), p, int(use_shifts),
                              N.FC_F64 if dtype == torch.float64 else N.FC_F32, 0.0, R_MAX, R_MAX)


def _vp(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None and t.numel() else None


@pytest.mark.parametrize("mapping", ["cosine", "affine"])
@pytest.mark.parametrize("l_max", [2, 3])
def test_emu_edge_geometry_matches_composed_chain(emu_lib, l_max, mapping):
    """Host-emulation build of the kernels' per-edge code through the C ABI, float64."""
    pos, cells, shifts, ei, batch = _structure()
    n_radial = 8
    d = _desc(l_max, n_radial, mapping, torch.float64)
    e = ei.shape[1]
    attrs = torch.empty(e, (l_max + 1) ** 2, dtype=torch.float64)
    radial = torch.empty(e, n_radial, dtype=torch.float64)
    status = torch.zeros(1, dtype=torch.int32)
    rc = emu_lib.fc_edge_geometry_fwd(ctypes.byref(d), _vp(pos), pos.shape[0], _vp(cells), cells.shape[0], _vp(shifts),
                                      _vp(ei), _vp(batch), e, _vp(attrs), _vp(radial), _vp(status), None)
    N.check(emu_lib, rc, "fc_edge_geometry_fwd")
    assert int(status) == 0
    p_ = pos.clone().requires_grad_(True)
    c_ = cells.clone().requires_grad_(True)
    ra, rr = _composed(p_, c_, shifts, ei, batch, l_max, n_radial, mapping)
    assert (attrs - ra).abs().max().item() < 1e-12
    assert (radial - rr).abs().max().item() < 1e-12
    ga = torch.randn(ra.shape, dtype=torch.float64, generator=torch.Generator().manual_seed(1))
    gr = torch.randn(rr.shape, dtype=torch.float64, generator=torch.Generator().manual_seed(2))
    want_p, want_c = torch.autograd.grad((ra * ga).sum() + (rr * gr).sum(), [p_, c_])
    g_pos = torch.full_like(pos, float("nan"))
    g_cells = torch.full_like(cells, float("nan"))
    rc = emu_lib.fc_edge_geometry_bwd(ctypes.byref(d), _vp(pos), pos.shape[0], _vp(cells), cells.shape[0],
                                      _vp(shifts), _vp(ei), _vp(batch), e, _vp(ga), _vp(gr), _vp(g_pos),
                                      _vp(g_cells), _vp(status), None)
    N.check(emu_lib, rc, "fc_edge_geometry_bwd")
    scale = max(1.0, want_p.abs().max().item())
    assert (g_pos - want_p).abs().max().item() < 1e-10 * scale
    assert (g_cells - want_c).abs().max().item() < 1e-10 * max(1.0, want_c.abs().max().item())


def test_emu_edge_geometry_flags_bad_index(emu_lib):
    pos, cells, shifts, ei, batch = _structure(n_cells=1)
    ei = ei.clone()
    ei[1, 5] = pos.shape[0]
    d = _desc(3, 8, "cosine", torch.float64)
    e = ei.shape[1]
    attrs = torch.full((e, 16), float("nan"), dtype=torch.float64)
    radial = torch.full((e, 8), float("nan"), dtype=torch.float64)
    status = torch.zeros(1, dtype=torch.int32)
    rc = emu_lib.fc_edge_geometry_fwd(ctypes.byref(d), _vp(pos), pos.shape[0], _vp(cells), 1, _vp(shifts), _vp(ei),
                                      _vp(batch), e, _vp(attrs), _vp(radial), _vp(status), None)
    N.check(emu_lib, rc, "fc_edge_geometry_fwd")
    assert int(status) & N.FC_DEV_BAD_INDEX
    assert (attrs[5] == 0).all() and (radial[5] == 0).all()
    assert torch.isfinite(attrs).all() and torch.isfinite(radial).all()


@pytest.mark.gpu
@pytest.mark.parametrize("shuffle", [False, True])
@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-11), (torch.float32, 2e-5)])
@pytest.mark.parametrize("mapping", ["cosine", "affine"])
def test_gpu_edge_geometry_matches_composed_chain(cuda_device, dtype, tol, mapping, shuffle):
    """Receiver-sorted edges (the model's order: runs of equal receivers are reduced in the
    warp before the atomics) and a random edge order."""
    from flashcart_b200 import ops

    pos, cells, shifts, ei, batch = _structure(seed=3, close_pair=dtype == torch.float64)
    if shuffle:
        perm = torch.randperm(ei.shape[1], generator=torch.Generator().manual_seed(9))
        ei, shifts = ei[:, perm].contiguous(), shifts[perm].contiguous()
    l_max, n_radial = 3, 8
    dev = cuda_device
    p_ = pos.to(dev, dtype).requires_grad_(True)
    c_ = cells.to(dev, dtype).requires_grad_(True)
    with ops.first_order_only():
        attrs, radial = ops.edge_geometry(p_, c_, shifts.to(dev), ei.to(dev), batch.to(dev), l_max, n_radial,
                                          mapping == "cosine", 6, 0.0, R_MAX, R_MAX)
    # the composed chain runs on the GPU in float64 (torch's device kernels). Run on the host,
    # it disagreed with the kernel by up to 7.3e-8 in the radial features in two full-suite
    # runs on some boxes, while the kernel's output was reproducible and the two agreed to
    # 7e-15 when the same case ran alone on such a box.
    rp = pos.to(dev).requires_grad_(True)
    rc_ = cells.to(dev).requires_grad_(True)
    ra, rr = _composed(rp.to(dtype).double(), rc_.to(dtype).double(), shifts.to(dev), ei.to(dev), batch.to(dev),
                       l_max, n_radial, mapping)
    for got, want, name in ((attrs, ra, "attrs"), (radial, rr, "radial")):
        err = (got.double().cpu() - want).abs().amax(dim=1)
        if err.max().item() >= tol:  # report the worst edges and whether a second launch repeats the values
            with ops.first_order_only():
                again = ops.edge_geometry(p_, c_, shifts.to(dev), ei.to(dev), batch.to(dev), l_max, n_radial,
                                          mapping == "cosine", 6, 0.0, R_MAX, R_MAX)[name == "radial"]
            worst = torch.topk(err, min(3, err.numel())).indices.tolist()
            # the worst edge's vector length recomputed in plain Python float64 arithmetic
            k0 = worst[0]
            i0, j0 = int(ei[0, k0]), int(ei[1, k0])
            cell0 = cells[int(batch[i0])].tolist()
            sh0 = [float(v) for v in shifts[k0]]
            v0 = [float(pos[j0, c]) - float(pos[i0, c]) + sum(sh0[a] * cell0[a][c] for a in range(3)) for c in range(3)]
            r0 = sum(c * c for c in v0) ** 0.5
            raise AssertionError(f"{name}: max |diff| {err.max().item():.3e} at edges {worst}; edge {k0}: |v| python "
                                 f"{r0!r}, kernel row {got[k0].double().cpu().tolist()}, composed row "
                                 f"{want[k0].detach().tolist()}; second launch bitwise equal: "
                                 f"{bool(torch.equal(again, got))}")
    g = torch.Generator().manual_seed(4)
    ga = torch.randn(ra.shape, dtype=torch.float64, generator=g)
    gr = torch.randn(rr.shape, dtype=torch.float64, generator=g)
    got_p, got_c = torch.autograd.grad((attrs * ga.to(dev, dtype)).sum() + (radial * gr.to(dev, dtype)).sum(),
                                       [p_, c_])
    want_p, want_c = torch.autograd.grad((ra * ga).sum() + (rr * gr).sum(), [rp, rc_])
    want_p, want_c = want_p.cpu(), want_c.cpu()
    # the almost-coincident pair divides by 1e-4: compare relative to the largest gradient
    assert (got_p.double().cpu() - want_p).abs().max().item() < tol * max(1.0, want_p.abs().max().item())
    assert (got_c.double().cpu() - want_c).abs().max().item() < tol * max(1.0, want_c.abs().max().item())
    ops.check_device_status(dev)


@pytest.mark.gpu
def test_gpu_fused_geometry_potential_matches_composed(cuda_device):
    """E/F/S of the potential with the fused edge geometry (first-order evaluation) equal the
    composed chain's (the model's path when a second derivative is requested), float64."""
    from test_model_parity import _build, _graph

    import os
    root = os.path.dirname(os.path.abspath(__file__))
    golden = torch.load(os.path.join(root, "golden", "model_golden.pt"), map_location="cpu", weights_only=True)
    model = _build("cfg3arch", golden).to(cuda_device, torch.float64)
    graph = _graph(golden, torch.float64, cuda_device)
    fused = model.predict(graph, compute_forces=True, compute_stress=True)
    orig = type(model)._geometry_fusable
    type(model)._geometry_fusable = lambda self, g: False
    try:
        composed = model.predict(graph, compute_forces=True, compute_stress=True)
    finally:
        type(model)._geometry_fusable = orig
    for k in ("energy", "forces", "stress"):
        ref = composed[k]
        assert (fused[k] - ref).abs().max().item() <= 1e-10 * max(1.0, ref.abs().max().item()), k
