"""Direct C-ABI calls (include/flashcart_b200.h) on torch tensors.

Used by the tests with two libraries: the host-emulation build (CPU tensors, host
pointers) and the sm_100a build (CUDA tensors). Mirrors what a reference-side
ctypes binding would do, without the torch operator layer.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch

from flashcart_b200 import _native as N
from flashcart_b200.ops import tp_out_dim


def p(t: Optional[torch.Tensor]):
    return None if t is None or t.numel() == 0 else ctypes.c_void_p(t.data_ptr())


def desc(meta, dtype) -> N.TpDesc:
    l1, l2, lo, f1, f2, sym, shared, red = [int(v) for v in meta[:8]]
    return N.TpDesc(l1, l2, lo, f1, f2, sym, shared, red, N.FC_F64 if dtype == torch.float64 else N.FC_F32)


def stream_of(t: torch.Tensor):
    if t.is_cuda:
        return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)
    return None


def rowptr(lib, idx_i, n_nodes, status=None):
    rp = torch.empty(n_nodes + 1, dtype=torch.int64, device=idx_i.device)
    rc = lib.fc_build_rowptr(p(idx_i), idx_i.numel(), n_nodes, p(rp), p(status), stream_of(idx_i))
    N.check(lib, rc, "fc_build_rowptr")
    return rp


def tp_fwd(lib, meta, in1, in2, w, idx_i=None, idx_j=None, status=None):
    d = desc(meta, in1.dtype)
    odim = tp_out_dim(d.in1_l_max, d.in2_l_max, d.out_l_max, d.in1_features, d.in2_features,
                      d.symmetric_product, d.reduce_paths)
    n = in1.shape[0]
    out = torch.full((n, odim), float("nan"), dtype=in1.dtype, device=in1.device)
    rp = rowptr(lib, idx_i, n, status) if idx_i is not None else None
    rc = lib.fc_tp_fwd(ctypes.byref(d), p(in1), p(in2), p(w), p(rp), p(idx_j), n, n, in2.shape[0], p(out), p(status),
                       stream_of(in1))
    N.check(lib, rc, "fc_tp_fwd")
    return out


def tp_bwd(lib, meta, g, in1, in2, w, idx_i=None, idx_j=None, need=(True, True, True), status=None):
    d = desc(meta, in1.dtype)
    n = in1.shape[0]
    g1 = torch.full_like(in1, float("nan")) if need[0] else None
    g2 = torch.full_like(in2, float("nan")) if need[1] else None
    gw = torch.full_like(w, float("nan")) if need[2] else None
    rp = rowptr(lib, idx_i, n, status) if idx_i is not None else None
    rc = lib.fc_tp_bwd(ctypes.byref(d), p(g), p(in1), p(in2), p(w), p(rp), p(idx_j), n, n, in2.shape[0],
                       p(g1), p(g2), p(gw), p(status), stream_of(in1))
    N.check(lib, rc, "fc_tp_bwd")
    return g1, g2, gw


def tp_dbwd(lib, meta, g, in1, in2, w, v1, v2, vw, idx_i=None, idx_j=None, status=None):
    d = desc(meta, in1.dtype)
    n = in1.shape[0]
    dg = torch.full_like(g, float("nan"))
    d1 = torch.full_like(in1, float("nan"))
    d2 = torch.full_like(in2, float("nan"))
    dw = torch.full_like(w, float("nan"))
    rp = rowptr(lib, idx_i, n, status) if idx_i is not None else None
    rc = lib.fc_tp_dbwd(ctypes.byref(d), p(g), p(in1), p(in2), p(w), p(v1), p(v2), p(vw), p(rp), p(idx_j), n, n,
                        in2.shape[0], p(dg), p(d1), p(d2), p(dw), p(status), stream_of(in1))
    N.check(lib, rc, "fc_tp_dbwd")
    return dg, d1, d2, dw


def irreps_fwd(lib, x, l):
    out = torch.full((x.shape[0], (l + 1) ** 2), float("nan"), dtype=x.dtype, device=x.device)
    code = N.FC_F64 if x.dtype == torch.float64 else N.FC_F32
    N.check(lib, lib.fc_irreps_fwd(p(x), x.shape[0], l, code, p(out), stream_of(x)), "fc_irreps_fwd")
    return out


def irreps_bwd(lib, g, x, l):
    gx = torch.full_like(x, float("nan"))
    code = N.FC_F64 if x.dtype == torch.float64 else N.FC_F32
    N.check(lib, lib.fc_irreps_bwd(p(g), p(x), x.shape[0], l, code, p(gx), stream_of(x)), "fc_irreps_bwd")
    return gx


def irreps_dbwd(lib, g, x, v, l):
    dg = torch.full_like(g, float("nan"))
    dx = torch.full_like(x, float("nan"))
    code = N.FC_F64 if x.dtype == torch.float64 else N.FC_F32
    N.check(lib, lib.fc_irreps_dbwd(p(g), p(x), p(v), x.shape[0], l, code, p(dg), p(dx), stream_of(x)),
            "fc_irreps_dbwd")
    return dg, dx


def linear_desc(li, lo, fi, fo, paths, dtype):
    common = min(li, lo)
    d = N.LinearDesc()
    d.n_active = common + 1
    d.dtype = N.FC_F64 if dtype == torch.float64 else N.FC_F32
    d.precision = N.FC_PREC_IEEE
    off = 0
    in_offs = []
    for l in range(li + 1):
        in_offs.append(off)
        off += (2 * l + 1) * fi * paths[l]
    d.in_dim = off
    d.out_dim = sum((2 * l + 1) * fo for l in range(lo + 1))
    o = 0
    for l in range(common + 1):
        d.in_offsets[l] = in_offs[l]
        d.out_offsets[l] = o
        o += (2 * l + 1) * fo
        d.m_values[l] = 2 * l + 1
        d.f_in_values[l] = fi * paths[l]
        d.f_out_values[l] = fo
    return d


def ptr_array(ts):
    arr = (ctypes.c_void_p * max(1, len(ts)))()
    for i, t in enumerate(ts):
        arr[i] = None if t is None else t.data_ptr()
    return arr


def linear_fwd(lib, d, x, ws, scale):
    out = torch.full((x.shape[0], d.out_dim), float("nan"), dtype=x.dtype, device=x.device)
    N.check(lib, lib.fc_linear_fwd(ctypes.byref(d), p(x), ptr_array(ws), p(scale), x.shape[0], p(out), None,
                                   stream_of(x)), "fc_linear_fwd")
    return out


def linear_bwd(lib, d, g, x, ws, scale):
    gx = torch.full_like(x, float("nan"))
    gws = [torch.full_like(w, float("nan")) for w in ws]
    N.check(lib, lib.fc_linear_bwd(ctypes.byref(d), p(g), p(x), ptr_array(ws), p(scale), x.shape[0], p(gx),
                                   ptr_array(gws), None, stream_of(x)), "fc_linear_bwd")
    return gx, gws


def linear_dbwd(lib, d, g, x, ws, vx, vws, scale):
    dg = torch.full_like(g, float("nan"))
    dx = torch.full_like(x, float("nan"))
    dws = [torch.full_like(w, float("nan")) for w in ws]
    N.check(lib, lib.fc_linear_dbwd(ctypes.byref(d), p(g), p(x), ptr_array(ws), p(vx),
                                    ptr_array(vws) if vws is not None else None, p(scale), x.shape[0], p(dg),
                                    p(dx), ptr_array(dws), None, stream_of(x)), "fc_linear_dbwd")
    return dg, dx, dws


def _dtype_code(t):
    return N.FC_F64 if t.dtype == torch.float64 else N.FC_F32


def halo_pack(lib, x, idx, status=None):
    buf = torch.full((idx.numel(), x.shape[1]), float("nan"), dtype=x.dtype, device=x.device)
    N.check(lib, lib.fc_halo_pack(p(x), x.shape[0], x.shape[1], _dtype_code(x), p(idx), idx.numel(), p(buf),
                                  p(status), stream_of(x)), "fc_halo_pack")
    return buf


def halo_unpack(lib, buf, idx, x, accumulate, status=None):
    N.check(lib, lib.fc_halo_unpack(p(buf), idx.numel(), buf.shape[1], _dtype_code(buf), p(idx), p(x), x.shape[0],
                                    int(accumulate), p(status), stream_of(x)), "fc_halo_unpack")
    return x
