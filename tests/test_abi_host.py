"""Host-side checks that need no GPU: the libraries load, the header's symbols are
exported, argument errors map to the reference's exception types, module metadata
matches the reference conventions."""

import ctypes
import os
import re

import pytest
import torch

import abi_calls as A
from flashcart_b200 import _native as N
from flashcart_b200 import build_ext, o3
from flashcart_b200.codegen import stf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(fc_[a-z0-9_]+)\s*\(", text))
    return names


def test_header_symbols_match_binding():
    assert _declared_symbols() == set(N.EXPORTED_SYMBOLS)


@pytest.mark.parametrize("which", ["cuda", "emu"])
def test_library_loads_and_exports_every_declared_symbol(which):
    path = build_ext.CUDA_LIB if which == "cuda" else build_ext.EMU_LIB
    if not os.path.exists(path):
        build_ext.build(cuda=which == "cuda", emu=which == "emu")
    lib = ctypes.CDLL(path)
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    bound = N.bind(path)
    assert bound.fc_version().decode().startswith("flashcart_b200")


def test_unsupported_rank_and_bad_features_map_to_reference_errors(emu_lib):
    x = torch.zeros(2, 25 * 2, dtype=torch.float64)
    with pytest.raises(NotImplementedError, match="l_max"):
        A.tp_fwd(emu_lib, [4, 4, 4, 2, 2, 0, 0, 0], x, x, torch.zeros(2, 100, dtype=torch.float64))
    with pytest.raises(ValueError, match="must match unless one of them is 1"):
        A.tp_fwd(emu_lib, [1, 1, 1, 2, 3, 0, 0, 0], x, x, x)


def test_num_paths_and_out_dim_agree_with_module(emu_lib):
    for l1 in range(4):
        for l2 in range(4):
            for lo in range(4):
                for sym in ([False, True] if l1 == l2 else [False]):
                    tp = o3.TensorProduct(l1, l2, lo, 3, 1 if not sym else 3, symmetric_product=sym)
                    d = A.desc([l1, l2, lo, 3, 1 if not sym else 3, int(sym), 0, 0], torch.float32)
                    assert emu_lib.fc_tp_num_paths(ctypes.byref(d)) == tp.n_total_paths
                    assert sum(tp.out_paths) == len(stf.enumerate_paths(l1, l2, lo, sym))


def test_module_metadata_matches_reference_conventions():
    tp = o3.TensorProduct(2, 2, 2, 64, 1)
    assert tp.out_paths == [3, 4, 4] and tp.n_total_paths == 11
    tp = o3.TensorProduct(3, 3, 3, 128, 1)
    assert tp.out_paths == [4, 6, 7, 6] and tp.n_total_paths == 23
    assert tp.in1_dim == 16 * 128 and tp.in2_dim == 16
    lin = o3.LinearLayer(3, 3, 128, 128, in_paths=[4, 6, 7, 6])
    assert [tuple(w.shape) for w in lin.weight] == [(128, 512), (128, 768), (128, 896), (128, 768)]
    assert set(lin.state_dict()) == {"weight.0", "weight.1", "weight.2", "weight.3"}
    torch.testing.assert_close(lin.scale, torch.tensor([512 ** -0.5, 768 ** -0.5, 896 ** -0.5, 768 ** -0.5]))


def test_module_shape_errors_match_reference():
    tp = o3.TensorProduct(1, 1, 1, 2, 1)
    with pytest.raises(RuntimeError, match="Incorrect last dimension for in1"):
        tp(torch.zeros(2, 3), torch.zeros(2, tp.in2_dim), torch.zeros(2, 6))
    with pytest.raises(ValueError, match="Non-shared weights must be 2D"):
        tp(torch.zeros(2, tp.in1_dim), torch.zeros(2, tp.in2_dim), torch.zeros(6))
    with pytest.raises(ValueError, match="Input dimensions must match"):
        o3.TensorProduct(1, 1, 1, 2, 3)
    lin = o3.LinearLayer(1, 1, 2, 2)
    with pytest.raises(RuntimeError, match="Incorrect last dimension for x"):
        lin(torch.zeros(2, 3))


def test_product_path_has_no_cpu_fallback():
    tp = o3.TensorProduct(1, 1, 1, 2, 1)
    with pytest.raises(RuntimeError, match="CUDA"):
        tp(torch.zeros(2, tp.in1_dim), torch.zeros(2, tp.in2_dim), torch.zeros(2, tp.n_total_paths * 2))
    ir = o3.Irreps(2)
    with pytest.raises(RuntimeError, match="CUDA"):
        ir(torch.randn(4, 3))


def test_rotation_helpers_match_oracle_full_tensors():
    from oracle import stf_oracle as O

    torch.manual_seed(0)
    x = torch.randn(5, 16 * 2, dtype=torch.float64)
    full = o3.utils.irreps_to_cartesian(x, 3)
    back = o3.utils.cartesian_to_irreps(full, 3)
    assert (back - x).abs().max() < 1e-12
    q, _ = torch.linalg.qr(torch.randn(3, 3, dtype=torch.float64))
    rot = o3.utils.rotate_irreps(x, q, 3)
    # rotating unit-vector tensors equals the tensors of the rotated vectors
    r = torch.nn.functional.normalize(torch.randn(7, 3, dtype=torch.float64), dim=-1)
    lhs = o3.utils.rotate_irreps(O.irreps(r, 3), q, 3)
    rhs = O.irreps(r @ q.T, 3)
    assert (lhs - rhs).abs().max() < 1e-12
    assert rot.shape == x.shape


def test_new_entry_points_reject_bad_arguments(emu_lib):
    """Validation of fc_linear_dbwd and fc_halo_pack / fc_halo_unpack: status codes map to
    ValueError with the entry point named, before anything is read or launched."""
    x = torch.zeros(4, 8, dtype=torch.float64)
    idx = torch.tensor([0, 1])
    P, I = ctypes.c_void_p, ctypes.c_int64
    rc = emu_lib.fc_halo_pack(P(x.data_ptr()), 4, 8, 7, P(idx.data_ptr()), 2, P(x.data_ptr()), None, None)
    with pytest.raises(ValueError, match="fc_halo_pack: dtype"):
        N.check(emu_lib, rc, "fc_halo_pack")
    rc = emu_lib.fc_halo_unpack(P(x.data_ptr()), -1, 8, N.FC_F64, P(idx.data_ptr()), P(x.data_ptr()), 4, 0, None,
                                None)
    with pytest.raises(ValueError, match="fc_halo_unpack: negative size"):
        N.check(emu_lib, rc, "fc_halo_unpack")
    rc = emu_lib.fc_halo_pack(None, 4, 8, N.FC_F64, P(idx.data_ptr()), 2, P(x.data_ptr()), None, None)
    with pytest.raises(ValueError, match="null tensor"):
        N.check(emu_lib, rc, "fc_halo_pack")
    assert emu_lib.fc_halo_pack(None, 0, 8, N.FC_F64, None, 0, None, None, None) == 0  # nothing to move
    d = A.linear_desc(1, 1, 2, 2, [1, 1], torch.float64)
    w = [torch.zeros(2, 2, dtype=torch.float64), torch.zeros(2, 2, dtype=torch.float64)]
    xl = torch.zeros(3, d.in_dim, dtype=torch.float64)
    g = torch.zeros(3, d.out_dim, dtype=torch.float64)
    sc = torch.ones(2, dtype=torch.float64)
    vws = (ctypes.c_void_p * 2)(w[0].data_ptr(), None)
    rc = emu_lib.fc_linear_dbwd(ctypes.byref(d), P(g.data_ptr()), P(xl.data_ptr()), A.ptr_array(w), None, vws,
                                P(sc.data_ptr()), I(3), P(g.data_ptr()), None, None, None, None)
    with pytest.raises(ValueError, match="null weight tangent for rank 1"):
        N.check(emu_lib, rc, "fc_linear_dbwd")


def test_residual_entry_points_reject_bad_arguments(emu_lib):
    """Validation of fc_tp_bwd_residual, fc_linear_fwd_residual and fc_linear_bwd_residual:
    every refusal is decided on the host, before anything is read or launched."""
    P, I = ctypes.c_void_p, ctypes.c_int64
    C, n = 128, 4
    d = N.TpDesc(3, 3, 3, C, C, 0, 1, 0, N.FC_F32)
    rows = torch.zeros(n, 16 * C)
    go = torch.zeros(n, 99 * C)
    w = torch.zeros(23 * C)

    def tp_res(desc, r1, ld, comps, base=rows):
        return emu_lib.fc_tp_bwd_residual(ctypes.byref(desc), P(go.data_ptr()), P(base.data_ptr()),
                                          P(rows.data_ptr()), P(w.data_ptr()), I(n), r1, I(ld), comps, None,
                                          P(rows.data_ptr()), P(rows.data_ptr()), None, None)

    r1 = P(rows.data_ptr())
    for ld, comps in ((4 * C + 1, 4), (2 * C, 4), (16 * C, 17), (16 * C, -1)):  # odd, short, too many, negative
        with pytest.raises(ValueError, match="residual_in1 layout"):
            N.check(emu_lib, tp_res(d, r1, ld, comps), "fc_tp_bwd_residual")
    for bad in (N.TpDesc(3, 3, 3, C, C, 0, 1, 0, N.FC_F64), N.TpDesc(3, 3, 3, 96, 96, 0, 1, 0, N.FC_F32),
                N.TpDesc(3, 3, 3, C, C, 0, 1, 1, N.FC_F32)):  # float64, 96 channels, reduced paths
        assert tp_res(bad, r1, 4 * C, 4) == N.FC_ERR_UNSUPPORTED
        assert b"float32 dense products" in emu_lib.fc_last_error()
    odd = P(rows.data_ptr() + 4)  # rows that are not 8-byte aligned
    assert tp_res(d, odd, 4 * C, 4) == N.FC_ERR_UNSUPPORTED
    with pytest.raises(ValueError, match="negative size"):
        N.check(emu_lib, emu_lib.fc_tp_bwd_residual(ctypes.byref(d), None, None, None, None, I(-1), None, I(0), 0,
                                                    None, None, None, None, None), "fc_tp_bwd_residual")

    ld = A.linear_desc(1, 1, 8, 8, [1, 1], torch.float32)
    x = torch.zeros(n, ld.in_dim)
    ws = [torch.zeros(8, 8), torch.zeros(8, 8)]
    sc = torch.ones(2)
    for name in ("fc_linear_fwd_residual", "fc_linear_bwd_residual"):
        fn = getattr(emu_lib, name)
        assert fn(ctypes.byref(ld), P(x.data_ptr()), A.ptr_array(ws), None, P(sc.data_ptr()), I(0), None, None,
                  None, None) == 0  # no rows: nothing to do
        with pytest.raises(ValueError, match="null tensor"):
            N.check(emu_lib, fn(ctypes.byref(ld), P(x.data_ptr()), A.ptr_array(ws), None, P(sc.data_ptr()), I(n),
                                None, P(x.data_ptr()), None, None), name)
        part = A.linear_desc(1, 1, 8, 8, [1, 1], torch.float32)
        part.n_active = 1  # rank 1 of the output row left to nobody
        assert fn(ctypes.byref(part), P(x.data_ptr()), A.ptr_array(ws), None, P(sc.data_ptr()), I(n),
                  P(x.data_ptr()), P(x.data_ptr()), None, None) == N.FC_ERR_UNSUPPORTED
        assert b"cover the output row" in emu_lib.fc_last_error()
        xd = A.linear_desc(1, 1, 8, 8, [1, 1], torch.float64)
        assert fn(ctypes.byref(xd), P(x.data_ptr()), A.ptr_array(ws), None, P(sc.data_ptr()), I(n),
                  P(x.data_ptr()), P(x.data_ptr()), None, None) == N.FC_ERR_UNSUPPORTED
