"""The generated kernel bodies and the C ABI, executed on the CPU (host-emulation build).

The host-emulation library compiles the exact per-thread code of the sm_100a
kernels (generated tensor-product bodies, direction-tensor polynomials, linear-map
GEMMs, receiver CSR) with the host compiler; this suite drives it through the same
C entry points and checks every output against the reference's golden vectors.
"""

import ctypes

import pytest
import torch

import abi_calls as A
from flashcart_b200 import _native as N

TOL = 1e-11


def _tp_keys(golden):
    return sorted({k.rsplit("/", 1)[0] for k in golden if k.startswith("tp/")})


def _case(golden, key):
    m = [int(v) for v in golden[key + "/meta"]]
    idx_i = golden.get(key + "/idx_i")
    idx_j = golden.get(key + "/idx_j")
    return m, idx_i, idx_j


def test_emu_tp_forward(golden, emu_lib):
    for key in _tp_keys(golden):
        m, idx_i, idx_j = _case(golden, key)
        in1 = golden[key + "/in1"]
        in2 = in1 if m[5] else golden[key + "/in2"]
        out = A.tp_fwd(emu_lib, m, in1, in2, golden[key + "/w"], idx_i, idx_j)
        assert (out - golden[key + "/out"]).abs().max() < TOL, key


def test_emu_tp_backward(golden, emu_lib):
    for key in _tp_keys(golden):
        m, idx_i, idx_j = _case(golden, key)
        in1 = golden[key + "/in1"]
        sym = bool(m[5])
        in2 = in1 if sym else golden[key + "/in2"]
        g1, g2, gw = A.tp_bwd(emu_lib, m, golden[key + "/g"], in1, in2, golden[key + "/w"], idx_i, idx_j)
        if sym:
            assert (g1 + g2 - golden[key + "/grad_in1"]).abs().max() < TOL, key
        else:
            assert (g1 - golden[key + "/grad_in1"]).abs().max() < TOL, key
            assert (g2 - golden[key + "/grad_in2"]).abs().max() < TOL, key
        assert (gw - golden[key + "/grad_w"]).abs().max() < TOL, key


def test_emu_tp_backward_partial_requests(golden, emu_lib):
    key = "tp/l3x3to3_f21/conv"
    m, idx_i, idx_j = _case(golden, key)
    args = (golden[key + "/g"], golden[key + "/in1"], golden[key + "/in2"], golden[key + "/w"], idx_i, idx_j)
    for need in [(True, False, False), (False, True, False), (False, False, True)]:
        g = A.tp_bwd(emu_lib, m, *args, need=need)
        for got, want, n in zip(g, ("grad_in1", "grad_in2", "grad_w"), need):
            if n:
                assert (got - golden[f"{key}/{want}"]).abs().max() < TOL
            else:
                assert got is None


def test_emu_tp_double_backward(golden, emu_lib):
    for key in _tp_keys(golden):
        m, idx_i, idx_j = _case(golden, key)
        in1 = golden[key + "/in1"]
        sym = bool(m[5])
        in2 = in1 if sym else golden[key + "/in2"]
        v1 = golden[key + "/tan_in1"]
        v2 = v1 if sym else golden[key + "/tan_in2"]
        vw = golden[key + "/tan_w"]
        dg, d1, d2, dw = A.tp_dbwd(emu_lib, m, golden[key + "/g"], in1, in2, golden[key + "/w"], v1, v2, vw,
                                   idx_i, idx_j)
        assert (dg - golden[key + "/dd_g"]).abs().max() < TOL, (key, "g")
        if sym:
            assert (d1 + d2 - golden[key + "/dd_in1"]).abs().max() < TOL, (key, "in1")
        else:
            assert (d1 - golden[key + "/dd_in1"]).abs().max() < TOL, (key, "in1")
            assert (d2 - golden[key + "/dd_in2"]).abs().max() < TOL, (key, "in2")
        assert (dw - golden[key + "/dd_w"]).abs().max() < TOL, (key, "w")


@pytest.mark.parametrize("l", range(4))
def test_emu_irreps(golden, emu_lib, l):
    k = f"irreps/l{l}"
    x, g, v = golden[k + "/x"], golden[k + "/g"], golden[k + "/tan_x"]
    assert (A.irreps_fwd(emu_lib, x, l) - golden[k + "/out"]).abs().max() < TOL
    assert (A.irreps_bwd(emu_lib, g, x, l) - golden[k + "/grad_x"]).abs().max() < TOL
    dg, dx = A.irreps_dbwd(emu_lib, g, x, v, l)
    assert (dg - golden[k + "/dd_g"]).abs().max() < TOL
    assert (dx - golden[k + "/dd_x"]).abs().max() < TOL


def test_emu_linear(golden, emu_lib):
    names = sorted({k.split("/")[1] for k in golden if k.startswith("linear/")})
    for name in names:
        k = f"linear/{name}"
        meta = [int(v) for v in golden[k + "/meta"]]
        li, lo, fi, fo, has_ws = meta[:5]
        paths = meta[5:]
        common = min(li, lo)
        ws = [golden[f"{k}/w{l}"] for l in range(common + 1)]
        scale = torch.tensor([1.0 if has_ws == 1 else (fi * paths[l]) ** -0.5 for l in range(common + 1)],
                             dtype=torch.float64)
        d = A.linear_desc(li, lo, fi, fo, paths, torch.float64)
        out = A.linear_fwd(emu_lib, d, golden[k + "/x"], ws, scale)
        assert (out - golden[k + "/out"]).abs().max() < TOL, name
        gx, gws = A.linear_bwd(emu_lib, d, golden[k + "/g"], golden[k + "/x"], ws, scale)
        assert (gx - golden[k + "/grad_x"]).abs().max() < TOL, name
        for l in range(common + 1):
            assert (gws[l] - golden[f"{k}/grad_w{l}"]).abs().max() < TOL, (name, l)


def test_emu_rowptr_and_status_flags(emu_lib):
    idx = torch.tensor([0, 0, 1, 3, 3, 3], dtype=torch.int64)
    status = torch.zeros(1, dtype=torch.int32)
    rp = A.rowptr(emu_lib, idx, 5, status)
    assert rp.tolist() == [0, 2, 3, 3, 6, 6]
    assert int(status) == 0
    bad = torch.tensor([0, 2, 1, 7], dtype=torch.int64)
    A.rowptr(emu_lib, bad, 5, status)
    assert int(status) & N.FC_DEV_UNSORTED
    assert int(status) & N.FC_DEV_BAD_INDEX


def test_emu_tp_out_of_range_sender_is_flagged_not_read(emu_lib):
    m = [1, 1, 1, 2, 1, 0, 0, 0]
    in1 = torch.randn(3, 4 * 2, dtype=torch.float64)
    in2 = torch.randn(2, 4, dtype=torch.float64)
    w = torch.randn(2, 3 * 2, dtype=torch.float64)
    idx_i = torch.tensor([0, 1])
    idx_j = torch.tensor([1, 99])
    status = torch.zeros(1, dtype=torch.int32)
    out = A.tp_fwd(emu_lib, m, in1, in2, w, idx_i, idx_j, status)
    assert int(status) & N.FC_DEV_BAD_INDEX
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("sig", [(2, 2, 2, 4), (1, 1, 1, 3), (0, 3, 3, 2)])
def test_emu_tp_convolution_without_edges(emu_lib, sig):
    """A graph with no edges (isolated atoms only): every receiver sums nothing, the
    per-edge gradients have no rows, and nothing is read through the empty index arrays
    (the reference's gather / scatter_sum gives zeros the same way)."""
    l1, l2, lo, C = sig
    m = [l1, l2, lo, C, 1, 0, 0, 0]
    n = 5
    n_paths = emu_lib.fc_tp_num_paths(ctypes.byref(A.desc(m, torch.float64)))
    in1 = torch.randn(n, (l1 + 1) ** 2 * C, dtype=torch.float64)
    in2 = torch.zeros(0, (l2 + 1) ** 2, dtype=torch.float64)
    w = torch.zeros(0, n_paths * C, dtype=torch.float64)
    idx = torch.zeros(0, dtype=torch.int64)
    status = torch.zeros(1, dtype=torch.int32)
    out = A.tp_fwd(emu_lib, m, in1, in2, w, idx, idx, status)
    assert out.shape[0] == n and out.shape[1] > 0 and (out == 0).all()
    g = torch.randn_like(out)
    g1, g2, gw = A.tp_bwd(emu_lib, m, g, in1, in2, w, idx, idx, status=status)
    assert (g1 == 0).all() and g2.shape == in2.shape and gw.shape == w.shape
    v1 = torch.randn_like(in1)
    dg, d1, d2, dw = A.tp_dbwd(emu_lib, m, g, in1, in2, w, v1, in2, w, idx, idx, status)
    assert (dg == 0).all() and (d1 == 0).all() and d2.shape == in2.shape and dw.shape == w.shape
    assert int(status) == 0


def _ragged_receivers(n_nodes, degrees, seed):
    """Receiver-sorted idx_i with the given per-node degree (zeros allowed) and random senders."""
    g = torch.Generator().manual_seed(seed)
    idx_i = torch.repeat_interleave(torch.arange(n_nodes), torch.tensor(degrees))
    idx_j = torch.randint(0, n_nodes, (idx_i.numel(),), generator=g)
    return idx_i, idx_j, g


@pytest.mark.parametrize("sig", [(2, 2, 2, 4), (3, 3, 3, 2), (0, 3, 3, 3)])
def test_emu_tp_ragged_degrees_vs_oracle(emu_lib, sig):
    """Isolated receivers at both ends and in the middle, one receiver with many edges
    (several edge chunks), the rest of degree 1-3: forward and all three gradients
    against the oracle in float64."""
    from oracle import stf_oracle as O

    l1, l2, lo, C = sig
    m = [l1, l2, lo, C, 1, 0, 0, 0]
    degrees = [0, 0, 3, 137, 0, 1, 2, 0, 3, 1, 0, 0]
    n = len(degrees)
    idx_i, idx_j, g = _ragged_receivers(n, degrees, 5)
    e = idx_i.numel()
    n_paths = emu_lib.fc_tp_num_paths(ctypes.byref(A.desc(m, torch.float64)))
    in1 = torch.randn(n, (l1 + 1) ** 2 * C, generator=g, dtype=torch.float64)
    r = torch.nn.functional.normalize(torch.randn(e, 3, generator=g, dtype=torch.float64), dim=-1)
    in2 = O.irreps(r, l2)
    w = torch.randn(e, n_paths * C, generator=g, dtype=torch.float64)
    out = A.tp_fwd(emu_lib, m, in1, in2, w, idx_i, idx_j)
    leaves = [t.clone().requires_grad_(True) for t in (in1, in2, w)]
    ref = O.tensor_product(*leaves, idx_i, idx_j, l1, l2, lo, C, 1)
    assert (out - ref.detach()).abs().max() < TOL * max(1.0, ref.abs().max().item())
    for node, deg in enumerate(degrees):
        if deg == 0:
            assert (out[node] == 0).all()
    gout = torch.randn_like(out)
    grads = A.tp_bwd(emu_lib, m, gout, in1, in2, w, idx_i, idx_j)
    ref_grads = torch.autograd.grad(ref, leaves, gout)
    for a, b in zip(grads, ref_grads):
        assert (a - b).abs().max() < TOL * max(1.0, b.abs().max().item())


def test_emu_linear_without_rows(golden, emu_lib):
    """A map applied to zero rows (e.g. the radial layers of a graph with no edges):
    empty output, and weight gradients that are zero rather than left unwritten."""
    name = sorted({k.split("/")[1] for k in golden if k.startswith("linear/")})[0]
    k = f"linear/{name}"
    meta = [int(v) for v in golden[k + "/meta"]]
    li, lo, fi, fo = meta[:4]
    paths = meta[5:]
    common = min(li, lo)
    ws = [golden[f"{k}/w{l}"] for l in range(common + 1)]
    scale = torch.ones(common + 1, dtype=torch.float64)
    d = A.linear_desc(li, lo, fi, fo, paths, torch.float64)
    x = golden[k + "/x"][:0]
    out = A.linear_fwd(emu_lib, d, x, ws, scale)
    assert out.shape == (0, d.out_dim)
    gx, gws = A.linear_bwd(emu_lib, d, out, x, ws, scale)
    assert gx.shape == x.shape
    assert all((gw == 0).all() for gw in gws)


def test_emu_linear_double_backward(golden, emu_lib):
    """fc_linear_dbwd against the reference's VJP-of-VJP (tangents on grad_x and grad_w),
    plus the one-tangent forms against the two-tangent result split by linearity."""
    names = sorted({k.split("/")[1] for k in golden if k.startswith("linear/")})
    for name in names:
        k = f"linear/{name}"
        meta = [int(v) for v in golden[k + "/meta"]]
        li, lo, fi, fo, has_ws = meta[:5]
        paths = meta[5:]
        common = min(li, lo)
        ws = [golden[f"{k}/w{l}"] for l in range(common + 1)]
        vws = [golden[f"{k}/tan_w{l}"] for l in range(common + 1)]
        scale = torch.tensor([1.0 if has_ws == 1 else (fi * paths[l]) ** -0.5 for l in range(common + 1)],
                             dtype=torch.float64)
        d = A.linear_desc(li, lo, fi, fo, paths, torch.float64)
        g, x, vx = golden[k + "/g"], golden[k + "/x"], golden[k + "/tan_x"]
        dg, dx, dws = A.linear_dbwd(emu_lib, d, g, x, ws, vx, vws, scale)
        assert (dg - golden[k + "/dd_g"]).abs().max() < TOL, name
        assert (dx - golden[k + "/dd_x"]).abs().max() < TOL, name
        for l in range(common + 1):
            assert (dws[l] - golden[f"{k}/dd_w{l}"]).abs().max() < TOL, (name, l)
        dg_x, dx_x, dws_x = A.linear_dbwd(emu_lib, d, g, x, ws, vx, None, scale)
        dg_w, dx_w, dws_w = A.linear_dbwd(emu_lib, d, g, x, ws, None, vws, scale)
        assert (dx_x == 0).all() and all((w == 0).all() for w in dws_w)
        assert (dg_x + dg_w - dg).abs().max() < TOL, name
        assert (dx_w - dx).abs().max() < TOL and all((a - b).abs().max() < TOL for a, b in zip(dws_x, dws))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_emu_halo_pack_and_unpack(emu_lib, dtype):
    """Pack = row gather, unpack = row copy or (with repeated indices) row sum, as the
    forward and reverse ghost exchanges need; a bad index is flagged and skipped."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(40, 36, generator=g).to(dtype)
    send = torch.tensor([5, 0, 39, 5, 17, 22], dtype=torch.int64)
    buf = A.halo_pack(emu_lib, x, send)
    assert torch.equal(buf, x.index_select(0, send))
    ghosts = torch.tensor([30, 31, 32, 33, 34, 35], dtype=torch.int64)
    y = x.clone()
    A.halo_unpack(emu_lib, buf, ghosts, y, accumulate=False)
    ref = x.clone()
    ref[ghosts] = buf
    assert torch.equal(y, ref)
    owners = torch.tensor([1, 2, 1, 1, 7, 2], dtype=torch.int64)
    acc = torch.zeros(10, 36, dtype=dtype)
    A.halo_unpack(emu_lib, buf, owners, acc, accumulate=True)
    ref = torch.zeros(10, 36, dtype=dtype).index_add_(0, owners, buf)
    assert (acc - ref).abs().max() < (1e-6 if dtype == torch.float32 else 1e-14)
    status = torch.zeros(1, dtype=torch.int32)
    bad = torch.tensor([3, 40, -1], dtype=torch.int64)
    out = A.halo_pack(emu_lib, x, bad, status)
    assert int(status) & N.FC_DEV_BAD_INDEX
    assert torch.equal(out[0], x[3]) and (out[1:] == 0).all()
    status.zero_()
    tgt = torch.zeros(4, 36, dtype=dtype)
    A.halo_unpack(emu_lib, out, torch.tensor([0, 4, 1]), tgt, accumulate=True, status=status)
    assert int(status) & N.FC_DEV_BAD_INDEX and torch.equal(tgt[0], x[3]) and (tgt[1:] == 0).all()
