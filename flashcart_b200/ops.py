"""``torch.ops.flashcart.*`` operators backed by the sm_100a kernels.

Same operator names, schemas and autograd chains as the reference runtimes
(``o3/_tensor_product.py:332-1096``, ``o3/_irreps.py:84-202``,
``o3/_linear.py:328-778``), so compiled graphs and exported programs that call
``flashcart::tp_fwd`` and friends resolve to these kernels. One addition,
``flashcart::tp_dbwd``, is the second derivative that the reference launches
inside the autograd of ``tp_bwd``; here it is an operator of its own so that it
is visible to ``torch.compile``.

Every operator requires CUDA tensors and calls the C ABI (``include/flashcart_b200.h``)
on the current stream. There is no CPU path: a CPU tensor raises.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
import threading
import weakref
from typing import Dict, List, Optional, Sequence, Tuple

import torch
from torch import Tensor

from flashcart_b200 import _native as N

__all__ = ["check_device_status", "status_word", "KernelTimer", "set_kernel_timer", "first_order_only", "rms_norm"]

_DEBUG_CHECK = os.environ.get("FLASHCART_B200_CHECK", "0") not in ("", "0", "false", "False")


# ----------------------------------------------------------------------------- plumbing


def _require_cuda(*tensors: Optional[Tensor]) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                "flashcart_b200 operators run only on CUDA tensors (sm_100a kernels); there is no CPU path.")


def _code(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return N.FC_F32
    if dtype == torch.float64:
        return N.FC_F64
    raise TypeError(f"flashcart_b200 kernels support float32 and float64, got {dtype}")


def _p(t: Optional[Tensor]):
    if t is None or t.numel() == 0:
        return None
    return ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


_STATUS: Dict[int, Tensor] = {}


def status_word(device: torch.device) -> Tensor:
    """Per-device int32 word into which kernels OR data-error bits (FC_DEV_*)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _STATUS.get(idx)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = w
    return w


# status bits raised by host-composed checks (above the kernels' FC_DEV_* bits)
DEV_NOT_UNIT = 1 << 8
DEV_NOT_SYMMETRIC = 1 << 9


def flag_if(cond: Tensor, bit: int, device: torch.device) -> None:
    """OR ``bit`` into the device status word where the 0-d bool ``cond`` holds, without a
    host synchronisation (the check surfaces at the next :func:`check_device_status`)."""
    w = status_word(device)
    w.bitwise_or_(cond.to(torch.int32) * bit)


def check_device_status(device: Optional[torch.device] = None, clear: bool = True) -> None:
    """Synchronise and raise if a kernel flagged bad data since the last check.

    Mirrors the reference's ``torch._assert_async`` guards (unsorted receivers,
    ``o3/_tensor_product.py:397-401``; unit-length directions, ``o3/irreps.py:66-69``;
    symmetric-product operands, ``o3/tensor_product.py:131``) and out-of-range edge
    indices, as error bits instead of device asserts: the CUDA context stays usable.
    """
    device = device or torch.device("cuda", torch.cuda.current_device())
    w = status_word(device)
    v = int(w.item())
    if clear and v:
        w.zero_()
    msgs = []
    if v & N.FC_DEV_UNSORTED:
        msgs.append("Scatter tensor product requires a receiver-sorted idx_i "
                    "(edges grouped by ascending destination index).")
    if v & N.FC_DEV_BAD_INDEX:
        msgs.append("An edge index points outside its node array.")
    if v & N.FC_DEV_TIMEOUT:
        msgs.append("A bounded device-side wait expired; the results of that call are invalid.")
    if v & DEV_NOT_UNIT:
        msgs.append("Irreps.forward_normalized requires unit-length input vectors.")
    if v & DEV_NOT_SYMMETRIC:
        msgs.append("Symmetric product requires in1 == in2.")
    if msgs:
        raise RuntimeError(" ".join(msgs))


def _after(lib, rc: int, what: str, device: torch.device) -> None:
    N.check(lib, rc, what)
    if _DEBUG_CHECK:
        check_device_status(device)


class KernelTimer:
    """Optional instrumentation: CUDA events around every C-ABI call on its stream.

    ``records`` collects (name, start_event, end_event); ``launches`` counts the
    kernels of this library enqueued while the timer is installed. Nothing is
    skipped or reordered; the events only bracket the calls.
    """

    def __init__(self):
        self.records = []
        self.launches = 0

    def durations_ms(self) -> Dict[str, List[float]]:
        out: Dict[str, List[float]] = {}
        for name, a, b, _ in self.records:
            out.setdefault(name, []).append(a.elapsed_time(b))
        return out

    def bytes_per_call(self) -> Dict[str, List[int]]:
        """Algorithmic bytes of each call: every tensor it reads or writes, counted once."""
        out: Dict[str, List[int]] = {}
        for name, _, _, nb in self.records:
            out.setdefault(name, []).append(nb)
        return out


_TIMER: Optional[KernelTimer] = None


def set_kernel_timer(timer: Optional[KernelTimer]) -> None:
    global _TIMER
    _TIMER = timer


class _timed:
    def __init__(self, name: str, kernels: int, nbytes: int = 0):
        self.name, self.kernels, self.nbytes = name, kernels, nbytes

    def __enter__(self):
        t = _TIMER
        if t is not None:
            t.launches += self.kernels
            self.a = torch.cuda.Event(enable_timing=True)
            self.a.record()
        return self

    def __exit__(self, *exc):
        t = _TIMER
        if t is not None and exc[0] is None:
            b = torch.cuda.Event(enable_timing=True)
            b.record()
            t.records.append((self.name, self.a, b, self.nbytes))
        return False


def _nbytes(*ts: Optional[Tensor]) -> int:
    return sum(t.numel() * t.element_size() for t in ts if t is not None)


def _idx(t: Optional[Tensor]) -> Optional[Tensor]:
    if t is None:
        return None
    if t.dtype != torch.int64:
        t = t.to(torch.int64)
    return t.contiguous()


# ----------------------------------------------------------------------------- tensor product


def _paths_per_l(in1_l_max: int, in2_l_max: int, out_l_max: int, sym: bool) -> List[int]:
    lmax = max(in1_l_max, in2_l_max)
    out = []
    for lo in range(out_l_max + 1):
        c = 0
        for l1 in range(lmax + 1):
            for l2 in range(l1 + 1):
                ok = abs(l1 - l2) <= lo <= l1 + l2 and (l1 + l2 + lo) % 2 == 0
                if ok and l1 <= in1_l_max and l2 <= in2_l_max:
                    c += 1
                if ok and not sym and l2 < l1 and l1 <= in2_l_max and l2 <= in1_l_max:
                    c += 1
        out.append(c)
    return out


def tp_out_dim(in1_l_max, in2_l_max, out_l_max, in1_features, in2_features, symmetric_product, reduce_paths) -> int:
    F = max(in1_features, in2_features)
    npl = _paths_per_l(in1_l_max, in2_l_max, out_l_max, symmetric_product)
    if reduce_paths:
        return sum((2 * l + 1) * F for l in range(out_l_max + 1) if npl[l])
    return sum(npl[l] * (2 * l + 1) * F for l in range(out_l_max + 1))


def _tp_desc(in1_l_max, in2_l_max, out_l_max, in1_features, in2_features, symmetric_product, shared_weights,
             reduce_paths, dtype) -> N.TpDesc:
    return N.TpDesc(int(in1_l_max), int(in2_l_max), int(out_l_max), int(in1_features), int(in2_features),
                    int(bool(symmetric_product)), int(bool(shared_weights)), int(bool(reduce_paths)), _code(dtype))


def _rowptr(lib, idx_i: Tensor, n_nodes: int, device, stream, status) -> Tensor:
    rowptr = torch.empty(n_nodes + 1, dtype=torch.int64, device=device)
    if _TIMER is not None:
        _TIMER.launches += 1
    rc = lib.fc_build_rowptr(_p(idx_i), idx_i.numel(), n_nodes, ctypes.c_void_p(rowptr.data_ptr()), status, stream)
    N.check(lib, rc, "fc_build_rowptr")
    return rowptr


def _conv(idx_i, idx_j) -> bool:
    return idx_i is not None and idx_j is not None


@torch.library.custom_op("flashcart::tp_fwd", mutates_args=())
def tp_fwd(in1: Tensor, in2: Tensor, weights: Tensor, idx_i: Optional[Tensor], idx_j: Optional[Tensor],
           in1_l_max: int, in2_l_max: int, out_l_max: int, in1_features: int, in2_features: int,
           symmetric_product: bool, shared_weights: bool, in1_offs: List[int], in2_offs: List[int],
           out_sizes: List[int], n_paths_per_l: List[int], n_total_paths: int,
           reduce_paths: bool = False) -> Tensor:
    _require_cuda(in1, in2, weights, idx_i, idx_j)
    lib = N.lib()
    dev = in1.device
    in1, in2, weights = in1.contiguous(), in2.contiguous(), weights.contiguous()
    desc = _tp_desc(in1_l_max, in2_l_max, out_l_max, in1_features, in2_features, symmetric_product,
                    shared_weights, reduce_paths, in1.dtype)
    out_dim = tp_out_dim(in1_l_max, in2_l_max, out_l_max, in1_features, in2_features, symmetric_product,
                         reduce_paths)
    n_out = in1.shape[0]
    out = torch.empty((n_out, out_dim), device=dev, dtype=in1.dtype)
    stream = _stream(dev)
    status = ctypes.c_void_p(status_word(dev).data_ptr())
    if _conv(idx_i, idx_j):
        idx_i, idx_j = _idx(idx_i), _idx(idx_j)
        rowptr = _rowptr(lib, idx_i, n_out, dev, stream, status)
        nb = _nbytes(in1, in2, weights, out, idx_j, rowptr)
        with _timed(f"tp_fwd_conv_{in1_l_max}{in2_l_max}{out_l_max}", 1, nb):
            rc = lib.fc_tp_fwd(ctypes.byref(desc), _p(in1), _p(in2), _p(weights),
                               ctypes.c_void_p(rowptr.data_ptr()), _p(idx_j), n_out, n_out, in2.shape[0], _p(out),
                               status, stream)
    else:
        if in1.shape[0] != in2.shape[0]:
            raise ValueError("idx_i and idx_j must be provided when in1 and in2 have different batch sizes. "
                             f"Got in1_batch={in1.shape[0]}, in2_batch={in2.shape[0]}.")
        with _timed(f"tp_fwd_dense_{in1_l_max}{in2_l_max}{out_l_max}", 1, _nbytes(in1, in2, weights, out)):
            rc = lib.fc_tp_fwd(ctypes.byref(desc), _p(in1), _p(in2), _p(weights), None, None, n_out, n_out,
                               n_out, _p(out), status, stream)
    _after(lib, rc, "fc_tp_fwd", dev)
    return out


@tp_fwd.register_fake
def _(in1, in2, weights, idx_i, idx_j, in1_l_max, in2_l_max, out_l_max, in1_features, in2_features,
      symmetric_product, shared_weights, in1_offs, in2_offs, out_sizes, n_paths_per_l, n_total_paths,
      reduce_paths=False):
    d = tp_out_dim(in1_l_max, in2_l_max, out_l_max, in1_features, in2_features, symmetric_product, reduce_paths)
    return in1.new_empty((in1.shape[0], d))


@torch.library.custom_op("flashcart::tp_bwd", mutates_args=())
def tp_bwd(grad_out: Tensor, in1: Tensor, in2: Tensor, weights: Tensor, idx_i: Optional[Tensor],
           idx_j: Optional[Tensor], in1_l_max: int, in2_l_max: int, out_l_max: int, in1_features: int,
           in2_features: int, symmetric_product: bool, shared_weights: bool, in1_offs: List[int],
           in2_offs: List[int], out_sizes: List[int], n_paths_per_l: List[int], n_total_paths: int,
           reduce_paths: bool, need_grad_in1: bool, need_grad_in2: bool,
           need_grad_weights: bool) -> Tuple[Tensor, Tensor, Tensor]:
    _require_cuda(grad_out, in1, in2, weights, idx_i, idx_j)
    lib = N.lib()
    dev = in1.device
    grad_out = grad_out.contiguous()
    in1, in2, weights = in1.contiguous(), in2.contiguous(), weights.contiguous()
    desc = _tp_desc(in1_l_max, in2_l_max, out_l_max, in1_features, in2_features, symmetric_product,
                    shared_weights, reduce_paths, in1.dtype)
    empty = in1.new_empty((0,))
    g1 = torch.empty_like(in1) if need_grad_in1 else empty
    g2 = torch.empty_like(in2) if need_grad_in2 else in2.new_empty((0,))
    gw = torch.empty_like(weights) if need_grad_weights else weights.new_empty((0,))
    if not (need_grad_in1 or need_grad_in2 or need_grad_weights):
        return g1, g2, gw
    stream = _stream(dev)
    status = ctypes.c_void_p(status_word(dev).data_ptr())
    if _conv(idx_i, idx_j):
        idx_i, idx_j = _idx(idx_i), _idx(idx_j)
        n_out = in1.shape[0]
        rowptr = _rowptr(lib, idx_i, n_out, dev, stream, status)
        nb = _nbytes(grad_out, in1, in2, weights, g1, g2, gw, idx_j, rowptr)
        with _timed(f"tp_bwd_conv_{in1_l_max}{in2_l_max}{out_l_max}", 1, nb):
            rc = lib.fc_tp_bwd(ctypes.byref(desc), _p(grad_out), _p(in1), _p(in2), _p(weights),
                               ctypes.c_void_p(rowptr.data_ptr()), _p(idx_j), n_out, n_out, in2.shape[0],
                               _p(g1), _p(g2), _p(gw), status, stream)
    else:
        n = in1.shape[0]
        with _timed(f"tp_bwd_dense_{in1_l_max}{in2_l_max}{out_l_max}", 1,
                    _nbytes(grad_out, in1, in2, weights, g1, g2, gw)):
            rc = lib.fc_tp_bwd(ctypes.byref(desc), _p(grad_out), _p(in1), _p(in2), _p(weights), None, None, n, n,
                               n, _p(g1), _p(g2), _p(gw), status, stream)
    _after(lib, rc, "fc_tp_bwd", dev)
    return g1, g2, gw


@tp_bwd.register_fake
def _(grad_out, in1, in2, weights, idx_i, idx_j, in1_l_max, in2_l_max, out_l_max, in1_features, in2_features,
      symmetric_product, shared_weights, in1_offs, in2_offs, out_sizes, n_paths_per_l, n_total_paths, reduce_paths,
      need_grad_in1, need_grad_in2, need_grad_weights):
    return (torch.empty_like(in1) if need_grad_in1 else in1.new_empty((0,)),
            torch.empty_like(in2) if need_grad_in2 else in2.new_empty((0,)),
            torch.empty_like(weights) if need_grad_weights else weights.new_empty((0,)))


@torch.library.custom_op("flashcart::tp_dbwd", mutates_args=())
def tp_dbwd(grad_out: Tensor, in1: Tensor, in2: Tensor, weights: Tensor, v_in1: Optional[Tensor],
            v_in2: Optional[Tensor], v_weights: Optional[Tensor], idx_i: Optional[Tensor], idx_j: Optional[Tensor],
            in1_l_max: int, in2_l_max: int, out_l_max: int, in1_features: int, in2_features: int,
            symmetric_product: bool, shared_weights: bool, reduce_paths: bool, need_d_grad_out: bool,
            need_d_in1: bool, need_d_in2: bool, need_d_weights: bool) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    _require_cuda(grad_out, in1, in2, weights, v_in1, v_in2, v_weights, idx_i, idx_j)
    lib = N.lib()
    dev = in1.device
    grad_out = grad_out.contiguous()
    in1, in2, weights = in1.contiguous(), in2.contiguous(), weights.contiguous()
    v_in1 = v_in1.contiguous() if v_in1 is not None and v_in1.numel() else None
    v_in2 = v_in2.contiguous() if v_in2 is not None and v_in2.numel() else None
    v_weights = v_weights.contiguous() if v_weights is not None and v_weights.numel() else None
    desc = _tp_desc(in1_l_max, in2_l_max, out_l_max, in1_features, in2_features, symmetric_product,
                    shared_weights, reduce_paths, in1.dtype)
    dg = torch.empty_like(grad_out) if need_d_grad_out else grad_out.new_empty((0,))
    d1 = torch.empty_like(in1) if need_d_in1 else in1.new_empty((0,))
    d2 = torch.empty_like(in2) if need_d_in2 else in2.new_empty((0,))
    dw = torch.empty_like(weights) if need_d_weights else weights.new_empty((0,))
    if not (need_d_grad_out or need_d_in1 or need_d_in2 or need_d_weights):
        return dg, d1, d2, dw
    stream = _stream(dev)
    status = ctypes.c_void_p(status_word(dev).data_ptr())
    if _conv(idx_i, idx_j):
        idx_i, idx_j = _idx(idx_i), _idx(idx_j)
        n_out = in1.shape[0]
        rowptr = _rowptr(lib, idx_i, n_out, dev, stream, status)
        rc = lib.fc_tp_dbwd(ctypes.byref(desc), _p(grad_out), _p(in1), _p(in2), _p(weights), _p(v_in1), _p(v_in2),
                            _p(v_weights), ctypes.c_void_p(rowptr.data_ptr()), _p(idx_j), n_out, n_out,
                            in2.shape[0], _p(dg), _p(d1), _p(d2), _p(dw), status, stream)
    else:
        n = in1.shape[0]
        rc = lib.fc_tp_dbwd(ctypes.byref(desc), _p(grad_out), _p(in1), _p(in2), _p(weights), _p(v_in1), _p(v_in2),
                            _p(v_weights), None, None, n, n, n, _p(dg), _p(d1), _p(d2), _p(dw), status, stream)
    _after(lib, rc, "fc_tp_dbwd", dev)
    return dg, d1, d2, dw


@tp_dbwd.register_fake
def _(grad_out, in1, in2, weights, v_in1, v_in2, v_weights, idx_i, idx_j, in1_l_max, in2_l_max, out_l_max,
      in1_features, in2_features, symmetric_product, shared_weights, reduce_paths, need_d_grad_out, need_d_in1,
      need_d_in2, need_d_weights):
    return (torch.empty_like(grad_out) if need_d_grad_out else grad_out.new_empty((0,)),
            torch.empty_like(in1) if need_d_in1 else in1.new_empty((0,)),
            torch.empty_like(in2) if need_d_in2 else in2.new_empty((0,)),
            torch.empty_like(weights) if need_d_weights else weights.new_empty((0,)))


_TP_SCALARS = 13  # in1_l_max ... reduce_paths


def _tp_fwd_setup(ctx, inputs, output):
    in1, in2, weights, idx_i, idx_j = inputs[:5]
    ctx.save_for_backward(in1, in2, weights, idx_i, idx_j)
    ctx.scalars = tuple(inputs[5:])


def _tp_fwd_backward(ctx, grad_out):
    n_extra = len(ctx.needs_input_grad) - 3
    need1, need2, needw = (bool(ctx.needs_input_grad[i]) for i in range(3))
    if grad_out is None or not (need1 or need2 or needw):
        return (None, None, None) + (None,) * n_extra
    in1, in2, weights, idx_i, idx_j = ctx.saved_tensors
    s = ctx.scalars
    reduce_paths = s[12] if len(s) > 12 else False
    g1, g2, gw = torch.ops.flashcart.tp_bwd(grad_out, in1, in2, weights, idx_i, idx_j, *s[:12], reduce_paths,
                                            need1, need2, needw)
    return (g1 if need1 else None, g2 if need2 else None, gw if needw else None) + (None,) * n_extra


tp_fwd.register_autograd(_tp_fwd_backward, setup_context=_tp_fwd_setup)


def _tp_bwd_setup(ctx, inputs, output):
    grad_out, in1, in2, weights, idx_i, idx_j = inputs[:6]
    ctx.save_for_backward(grad_out, in1, in2, weights, idx_i, idx_j)
    s = inputs[6:]
    # (in1_l_max, in2_l_max, out_l_max, in1_features, in2_features, symmetric, shared, ..., reduce, needs...)
    ctx.desc_args = (s[0], s[1], s[2], s[3], s[4], s[5], s[6], s[12])
    ctx.made = (bool(s[13]), bool(s[14]), bool(s[15]))
    if hasattr(ctx, "set_materialize_grads"):
        ctx.set_materialize_grads(False)


def _tp_bwd_backward(ctx, v1, v2, vw):
    n_extra = len(ctx.needs_input_grad) - 4
    need = [bool(ctx.needs_input_grad[i]) for i in range(4)]
    made1, made2, madew = ctx.made
    v1 = v1 if (made1 and v1 is not None and v1.numel()) else None
    v2 = v2 if (made2 and v2 is not None and v2.numel()) else None
    vw = vw if (madew and vw is not None and vw.numel()) else None
    if not any(need) or (v1 is None and v2 is None and vw is None):
        return (None,) * (4 + n_extra)
    grad_out, in1, in2, weights, idx_i, idx_j = ctx.saved_tensors
    a = ctx.desc_args
    dg, d1, d2, dw = torch.ops.flashcart.tp_dbwd(grad_out, in1, in2, weights, v1, v2, vw, idx_i, idx_j, a[0], a[1],
                                                 a[2], a[3], a[4], a[5], a[6], a[7], need[0], need[1], need[2],
                                                 need[3])
    return (dg if need[0] else None, d1 if need[1] else None, d2 if need[2] else None,
            dw if need[3] else None) + (None,) * n_extra


tp_bwd.register_autograd(_tp_bwd_backward, setup_context=_tp_bwd_setup)


# ----------------------------------------------------------------------------- direction tensors


@torch.library.custom_op("flashcart::irreps_fwd", mutates_args=())
def irreps_fwd(x: Tensor, l_max: int) -> Tensor:
    _require_cuda(x)
    lib = N.lib()
    x = x.contiguous()
    out = x.new_empty((x.shape[0], (l_max + 1) ** 2))
    if _TIMER is not None:
        _TIMER.launches += 1
    rc = lib.fc_irreps_fwd(_p(x), x.shape[0], int(l_max), _code(x.dtype), _p(out), _stream(x.device))
    _after(lib, rc, "fc_irreps_fwd", x.device)
    return out


@irreps_fwd.register_fake
def _(x, l_max):
    return x.new_empty((x.shape[0], (l_max + 1) ** 2))


@torch.library.custom_op("flashcart::irreps_bwd", mutates_args=())
def irreps_bwd(grad_output: Tensor, x: Tensor, l_max: int) -> Tensor:
    _require_cuda(grad_output, x)
    lib = N.lib()
    g, x = grad_output.contiguous(), x.contiguous()
    gx = torch.empty_like(x)
    if _TIMER is not None:
        _TIMER.launches += 1
    rc = lib.fc_irreps_bwd(_p(g), _p(x), x.shape[0], int(l_max), _code(x.dtype), _p(gx), _stream(x.device))
    _after(lib, rc, "fc_irreps_bwd", x.device)
    return gx


@irreps_bwd.register_fake
def _(grad_output, x, l_max):
    return torch.empty_like(x)


@torch.library.custom_op("flashcart::irreps_dbwd", mutates_args=())
def irreps_dbwd(grad_output: Tensor, x: Tensor, v: Tensor, l_max: int) -> Tuple[Tensor, Tensor]:
    _require_cuda(grad_output, x, v)
    lib = N.lib()
    g, x, v = grad_output.contiguous(), x.contiguous(), v.contiguous()
    dg = x.new_empty((x.shape[0], (l_max + 1) ** 2))
    dx = torch.empty_like(x)
    rc = lib.fc_irreps_dbwd(_p(g), _p(x), _p(v), x.shape[0], int(l_max), _code(x.dtype), _p(dg), _p(dx),
                            _stream(x.device))
    _after(lib, rc, "fc_irreps_dbwd", x.device)
    return dg, dx


@irreps_dbwd.register_fake
def _(grad_output, x, v, l_max):
    return x.new_empty((x.shape[0], (l_max + 1) ** 2)), torch.empty_like(x)


def _irreps_setup(ctx, inputs, output):
    x, l_max = inputs
    ctx.save_for_backward(x)
    ctx.l_max = int(l_max)


def _irreps_backward(ctx, grad_output):
    if grad_output is None or not ctx.needs_input_grad[0]:
        return None, None
    (x,) = ctx.saved_tensors
    return torch.ops.flashcart.irreps_bwd(grad_output, x, ctx.l_max), None


def _irreps_bwd_setup(ctx, inputs, output):
    g, x, l_max = inputs
    if hasattr(ctx, "set_materialize_grads"):
        ctx.set_materialize_grads(False)
    ctx.save_for_backward(g, x)
    ctx.l_max = int(l_max)


def _irreps_bwd_backward(ctx, v):
    need_g, need_x = bool(ctx.needs_input_grad[0]), bool(ctx.needs_input_grad[1])
    if v is None or not (need_g or need_x):
        return None, None, None
    g, x = ctx.saved_tensors
    dg, dx = torch.ops.flashcart.irreps_dbwd(g, x, v, ctx.l_max)
    return dg if need_g else None, dx if need_x else None, None


irreps_fwd.register_autograd(_irreps_backward, setup_context=_irreps_setup)
irreps_bwd.register_autograd(_irreps_bwd_backward, setup_context=_irreps_bwd_setup)


# ----------------------------------------------------------------------------- linear maps


def _linear_desc(x: Tensor, out_dim: int, in_offsets, out_offsets, m_values, f_in_values, f_out_values,
                 precision: str, act: int = 0) -> N.LinearDesc:
    d = N.LinearDesc()
    d.act = int(act)
    n = len(in_offsets)
    if n > N.FC_MAX_L + 1:
        raise NotImplementedError(f"flashcart_b200 linear supports at most {N.FC_MAX_L + 1} ranks, got {n}")
    d.n_active = n
    # bfloat16: the forward's bf16 storage path (tensor cores, fp32 accumulation)
    d.dtype = N.FC_BF16 if x.dtype == torch.bfloat16 else _code(x.dtype)
    d.precision = N.FC_PREC_TF32 if (precision == "tf32" and x.dtype == torch.float32) else N.FC_PREC_IEEE
    d.in_dim = x.shape[1]
    d.out_dim = int(out_dim)
    for l in range(n):
        d.in_offsets[l] = int(in_offsets[l])
        d.out_offsets[l] = int(out_offsets[l])
        d.m_values[l] = int(m_values[l])
        d.f_in_values[l] = int(f_in_values[l])
        d.f_out_values[l] = int(f_out_values[l])
    return d


def _ptr_array(tensors: Sequence[Optional[Tensor]]):
    arr = (ctypes.c_void_p * max(1, len(tensors)))()
    for i, t in enumerate(tensors):
        arr[i] = None if t is None or t.numel() == 0 else t.data_ptr()
    return arr


class _Split:
    __slots__ = ("refs", "versions", "bufs", "arr")


_SPLITS: Dict[Tuple, _Split] = {}


def _split_weights(lib, d: N.LinearDesc, ws: Sequence[Tensor], backward: bool):
    """tf32 hi / lo splits of frozen float32 weights for the tensor-core maps (the
    parameters ``predict`` freezes), made once and kept while the same weight tensors are
    unchanged (tensor identity, storage and ``_version``: in-place updates through torch
    invalidate them; writes through ``.data`` bypass the version counter and are not
    seen), so a step does not re-split constant weights. ``None`` when not applicable
    (the call then splits on its own). Never created during stream capture: a captured
    step reuses the splits its warm-up made."""
    if not ws or ws[0].dtype != torch.float32 or not ws[0].is_cuda or any(w.requires_grad for w in ws):
        return None  # trainable weights change every step: they are split per call
    key = (bool(backward),) + tuple(id(w) for w in ws) + tuple(tuple(w.shape) for w in ws)
    vers = tuple((w._version, w.data_ptr()) for w in ws)
    ent = _SPLITS.get(key)
    if ent is not None and ent.versions == vers and all(r() is w for r, w in zip(ent.refs, ws)):
        return ent.arr
    if torch.cuda.is_current_stream_capturing():
        return None
    if len(_SPLITS) > 1024:
        _SPLITS.clear()
    bufs = []
    for l, w in enumerate(ws):
        k, n = (d.f_out_values[l], d.f_in_values[l]) if backward else (d.f_in_values[l], d.f_out_values[l])
        bufs.append(torch.empty(2 * int(n) * ((int(k) + 3) // 4 * 4), dtype=torch.float32, device=w.device))
    arr = _ptr_array(bufs)
    if _TIMER is not None:
        _TIMER.launches += len(ws)
    rc = lib.fc_linear_presplit(ctypes.byref(d), _ptr_array(ws), int(bool(backward)), arr, _stream(ws[0].device))
    _after(lib, rc, "fc_linear_presplit", ws[0].device)
    ent = _Split()
    ent.refs = [weakref.ref(w) for w in ws]
    ent.versions, ent.bufs, ent.arr = vers, bufs, arr
    _SPLITS[key] = ent
    return arr


def _linear_fwd_impl(x: Tensor, weights: Sequence[Tensor], out_dim: int, lists, precision: str,
                     scale: Tensor, act: int = 0) -> Tensor:
    lib = N.lib()
    x = x.contiguous()
    n_active = len(lists[0])
    ws = [w.to(x.dtype).contiguous() for w in weights[:n_active]]
    sc = scale.to(device=x.device, dtype=torch.float32 if x.dtype == torch.bfloat16 else x.dtype).contiguous()
    out = x.new_empty((x.shape[0], int(out_dim)))
    d = _linear_desc(x, out_dim, lists[0], lists[1], lists[3], lists[4], lists[5], precision, act)
    split = _split_weights(lib, d, ws, False)
    with _timed("linear_fwd", n_active, _nbytes(x, out, *ws)):
        if split is not None:
            rc = lib.fc_linear_fwd_presplit(ctypes.byref(d), _p(x), _ptr_array(ws), split, _p(sc), x.shape[0],
                                            _p(out), ctypes.c_void_p(status_word(x.device).data_ptr()),
                                            _stream(x.device))
        else:
            rc = lib.fc_linear_fwd(ctypes.byref(d), _p(x), _ptr_array(ws), _p(sc), x.shape[0], _p(out),
                                   ctypes.c_void_p(status_word(x.device).data_ptr()), _stream(x.device))
    _after(lib, rc, "fc_linear_fwd", x.device)
    return out


def _linear_bwd_impl(grad_out: Tensor, x: Tensor, weights: Sequence[Tensor], need_x: bool, need_w: bool,
                     lists, precision: str, scale: Tensor, act: int = 0) -> Tuple[Tensor, List[Tensor]]:
    lib = N.lib()
    g, x = grad_out.contiguous(), x.contiguous()
    n_active = len(lists[0])
    ws = [w.to(x.dtype).contiguous() for w in weights[:n_active]]
    sc = scale.to(device=x.device, dtype=x.dtype).contiguous()
    gx = torch.empty_like(x) if need_x else x.new_empty((0,))
    gws = [torch.empty_like(w) for w in ws] if need_w else [w.new_empty((0,)) for w in ws]
    if n_active == 0:
        if need_x:
            gx.zero_()
        return gx, gws
    d = _linear_desc(x, g.shape[1], lists[0], lists[1], lists[3], lists[4], lists[5], precision, act)
    split = _split_weights(lib, d, ws, True) if need_x else None
    with _timed("linear_bwd", n_active * (int(need_x) + int(need_w)), _nbytes(g, x, gx, *ws, *gws)):
        if split is not None:
            rc = lib.fc_linear_bwd_presplit(ctypes.byref(d), _p(g), _p(x), _ptr_array(ws), split, _p(sc),
                                            x.shape[0], _p(gx), _ptr_array(gws) if need_w else None,
                                            ctypes.c_void_p(status_word(x.device).data_ptr()), _stream(x.device))
        else:
            rc = lib.fc_linear_bwd(ctypes.byref(d), _p(g), _p(x), _ptr_array(ws), _p(sc), x.shape[0],
                                   _p(gx) if need_x else None, _ptr_array(gws) if need_w else None,
                                   ctypes.c_void_p(status_word(x.device).data_ptr()), _stream(x.device))
    _after(lib, rc, "fc_linear_bwd", x.device)
    return gx, gws


@torch.library.custom_op("flashcart::linear_fwd", mutates_args=())
def linear_fwd(x: Tensor, weights: List[Tensor], meta: Tensor, out_size: int, use_fp64: bool,
               dot_input_precision: str, in_offsets: List[int], out_offsets: List[int], weight_offsets: List[int],
               m_values: List[int], f_in_values: List[int], f_out_values: List[int], scale: Tensor) -> Tensor:
    _require_cuda(x, *weights)
    lists = (in_offsets, out_offsets, weight_offsets, m_values, f_in_values, f_out_values)
    return _linear_fwd_impl(x, weights, out_size, lists, dot_input_precision, scale)


@linear_fwd.register_fake
def _(x, weights, meta, out_size, use_fp64, dot_input_precision, in_offsets, out_offsets, weight_offsets, m_values,
      f_in_values, f_out_values, scale):
    return x.new_empty((x.shape[0], int(out_size)))


@torch.library.custom_op("flashcart::linear_bwd", mutates_args=())
def linear_bwd(grad_out: Tensor, x: Tensor, weights: List[Tensor], need_x: bool, need_weight: bool, use_fp64: bool,
               dot_input_precision: str, in_offsets: List[int], out_offsets: List[int], weight_offsets: List[int],
               m_values: List[int], f_in_values: List[int], f_out_values: List[int],
               scale: Tensor) -> Tuple[Tensor, List[Tensor]]:
    _require_cuda(grad_out, x, *weights)
    lists = (in_offsets, out_offsets, weight_offsets, m_values, f_in_values, f_out_values)
    return _linear_bwd_impl(grad_out, x, weights, need_x, need_weight, lists, dot_input_precision, scale)


@linear_bwd.register_fake
def _(grad_out, x, weights, need_x, need_weight, use_fp64, dot_input_precision, in_offsets, out_offsets,
      weight_offsets, m_values, f_in_values, f_out_values, scale):
    n = len(in_offsets)
    return (torch.empty_like(x) if need_x else x.new_empty((0,)),
            [torch.empty_like(w) if need_weight else w.new_empty((0,)) for w in weights[:n]])


@torch.library.custom_op("flashcart::linear_silu_fwd", mutates_args=())
def linear_silu_fwd(x: Tensor, weights: List[Tensor], out_size: int, dot_input_precision: str,
                    in_offsets: List[int], out_offsets: List[int], m_values: List[int], f_in_values: List[int],
                    f_out_values: List[int], scale: Tensor) -> Tensor:
    """``linear_fwd`` of silu(x): the SiLU between two layers of the radial MLP
    (reference ``nn/layers.py:12-44``) applied by the GEMM's splitter warps to its input
    tiles, so the activations are never written (``fc_linear_desc.act = FC_ACT_SILU``)."""
    _require_cuda(x, *weights)
    lists = (in_offsets, out_offsets, [0] * len(in_offsets), m_values, f_in_values, f_out_values)
    return _linear_fwd_impl(x, weights, out_size, lists, dot_input_precision, scale, N.FC_ACT_SILU)


@linear_silu_fwd.register_fake
def _(x, weights, out_size, dot_input_precision, in_offsets, out_offsets, m_values, f_in_values, f_out_values,
      scale):
    return x.new_empty((x.shape[0], int(out_size)))


@torch.library.custom_op("flashcart::linear_silu_bwd", mutates_args=())
def linear_silu_bwd(grad_out: Tensor, x: Tensor, weights: List[Tensor], dot_input_precision: str,
                    in_offsets: List[int], out_offsets: List[int], m_values: List[int], f_in_values: List[int],
                    f_out_values: List[int], scale: Tensor) -> Tensor:
    """Input gradient of :func:`linear_silu_fwd`: silu'(x) * (grad_out (sW)) with the factor
    applied in the GEMM's epilogue (frozen weights: no weight gradient)."""
    _require_cuda(grad_out, x, *weights)
    lists = (in_offsets, out_offsets, [0] * len(in_offsets), m_values, f_in_values, f_out_values)
    gx, _ = _linear_bwd_impl(grad_out, x, weights, True, False, lists, dot_input_precision, scale, N.FC_ACT_SILU)
    return gx


@linear_silu_bwd.register_fake
def _(grad_out, x, weights, dot_input_precision, in_offsets, out_offsets, m_values, f_in_values, f_out_values,
      scale):
    return torch.empty_like(x)


def _lsilu_setup(ctx, inputs, output):
    x, weights = inputs[0], inputs[1]
    ctx.save_for_backward(x, inputs[-1], *weights)
    ctx.n_w = len(weights)
    ctx.meta = inputs[3:-1]


def _lsilu_backward(ctx, grad_out):
    if torch.is_grad_enabled():
        raise RuntimeError("flashcart::linear_silu_fwd was evaluated inside first_order_only(); its backward "
                           "cannot build a graph for a second derivative")
    x, scale, *weights = ctx.saved_tensors
    if any(w.requires_grad for w in weights):
        raise RuntimeError("flashcart::linear_silu_fwd has no weight gradient (frozen weights only)")
    gx = linear_silu_bwd(grad_out.contiguous(), x, weights, *ctx.meta, scale) if ctx.needs_input_grad[0] else None
    return (gx, [None] * len(weights), None) + (None,) * 7


linear_silu_fwd.register_autograd(_lsilu_backward, setup_context=_lsilu_setup)


# --------------------------------------------------------------------------- residual sums


def tp_dense_bwd_residual(tp, grad_out: Tensor, in1: Tensor, in2: Tensor, weights: Tensor,
                          residual_in1: Optional[Tensor], residual_in1_comps: int, residual_in2: Optional[Tensor],
                          out_in2: Optional[Tensor] = None) -> Tuple[Tensor, Tensor]:
    """Input gradients of the dense product ``tp(in1, in2, weights)`` (no edges) with other
    gradients of the same inputs added in the kernel (``fc_tp_bwd_residual``):
    grad_in1 = VJP + residual_in1 on the first ``residual_in1_comps`` components of each
    in1 row (``residual_in1`` holds just those, ``residual_in1_comps * F`` values per row),
    grad_in2 = VJP + residual_in2 (whole rows; ``out_in2`` may be ``residual_in2`` itself,
    which then accumulates). Frozen weights: no weight gradient."""
    _require_cuda(grad_out, in1, in2, weights)
    lib = N.lib()
    g, in1, in2, weights = grad_out.contiguous(), in1.contiguous(), in2.contiguous(), weights.contiguous()
    desc = _tp_desc(tp.in1_l_max, tp.in2_l_max, tp.out_l_max, tp.in1_features, tp.in2_features,
                    tp.symmetric_product, tp.shared_weights, tp.reduce_paths, in1.dtype)
    g1 = torch.empty_like(in1)
    g2 = torch.empty_like(in2) if out_in2 is None else out_in2
    r1 = residual_in1
    with _timed(f"tp_bwd_dense_{tp.in1_l_max}{tp.in2_l_max}{tp.out_l_max}", 1,
                _nbytes(g, in1, in2, weights, g1, g2, *([r1] if r1 is not None else []),
                        *([residual_in2] if residual_in2 is not None and residual_in2 is not g2 else []))):
        rc = lib.fc_tp_bwd_residual(ctypes.byref(desc), _p(g), _p(in1), _p(in2), _p(weights), in1.shape[0],
                                    _p(r1) if r1 is not None else None, r1.stride(0) if r1 is not None else 0,
                                    int(residual_in1_comps) if r1 is not None else 0,
                                    _p(residual_in2) if residual_in2 is not None else None, _p(g1), _p(g2),
                                    ctypes.c_void_p(status_word(in1.device).data_ptr()), _stream(in1.device))
    _after(lib, rc, "fc_tp_bwd_residual", in1.device)
    return g1, g2



def linear_residual_layout_ok(in_dim: int, out_dim: int, m_values: Sequence[int], f_in_values: Sequence[int],
                              f_out_values: Sequence[int], in_offsets: Sequence[int],
                              out_offsets: Sequence[int]) -> bool:
    """The rank layout the residual epilogue takes: active ranks covering both rows, at most
    128 channels per rank on both sides, in multiples of 4."""
    if not m_values:
        return False
    pi = po = 0
    for l in range(len(m_values)):
        if in_offsets[l] != pi or out_offsets[l] != po:
            return False
        if f_in_values[l] > 128 or f_out_values[l] > 128 or f_in_values[l] % 4 or f_out_values[l] % 4:
            return False
        pi += m_values[l] * f_in_values[l]
        po += m_values[l] * f_out_values[l]
    return pi == int(in_dim) and po == int(out_dim)


def linear_residual_fusable(x: Tensor, weights: Sequence[Tensor], out_dim: int, m_values: Sequence[int],
                            f_in_values: Sequence[int], f_out_values: Sequence[int], in_offsets: Sequence[int],
                            out_offsets: Sequence[int], residual: Tensor) -> bool:
    """``map(x) + residual`` (and its input gradient ``map^T(g) + residual``) can be one GEMM
    with the sum in its epilogue (``fc_linear_fwd_residual`` / ``fc_linear_bwd_residual``):
    first-order evaluation with frozen float32 weights on the GPU, active ranks covering the
    whole input and output rows, at most 128 channels per rank on both sides (the
    node-level maps) in multiples of 4, 16-byte aligned contiguous rows."""
    if not (first_order_only_active() and x.is_cuda and x.dtype == torch.float32 and x.dim() == 2
            and residual.dtype == torch.float32 and residual.device == x.device
            and tuple(residual.shape) == (x.shape[0], int(out_dim)) and residual.is_contiguous() and x.is_contiguous()
            and all(w.dtype == torch.float32 and not w.requires_grad for w in weights)):
        return False
    if x.data_ptr() % 16 or residual.data_ptr() % 16:
        return False
    return linear_residual_layout_ok(x.shape[1], out_dim, m_values, f_in_values, f_out_values, in_offsets,
                                     out_offsets)


def _linear_residual_impl(rows: Tensor, weights: Sequence[Tensor], out_dim: int, lists, precision: str,
                          scale: Tensor, residual: Tensor, backward: bool, out: Optional[Tensor] = None) -> Tensor:
    """out = map(rows) + residual (forward) or map^T(rows) + residual (backward: rows is the
    output gradient and out_dim the input row width); ``out`` may be ``residual`` itself."""
    lib = N.lib()
    rows = rows.contiguous()
    n_active = len(lists[0])
    ws = [w.to(rows.dtype).contiguous() for w in weights[:n_active]]
    sc = scale.to(device=rows.device, dtype=rows.dtype).contiguous()
    if out is None:
        out = rows.new_empty((rows.shape[0], int(out_dim)))
    in_dim, o_dim = (int(out_dim), rows.shape[1]) if backward else (rows.shape[1], int(out_dim))
    d = _linear_desc(rows.new_empty((0, in_dim)), o_dim, lists[0], lists[1], lists[3], lists[4], lists[5], precision, 0)
    split = _split_weights(lib, d, ws, backward)
    fn = lib.fc_linear_bwd_residual if backward else lib.fc_linear_fwd_residual
    name = "linear_bwd" if backward else "linear_fwd"
    with _timed(name, 1, _nbytes(rows, out, residual, *ws)):
        rc = fn(ctypes.byref(d), _p(rows), _ptr_array(ws), split, _p(sc), rows.shape[0], _p(residual), _p(out),
                ctypes.c_void_p(status_word(rows.device).data_ptr()), _stream(rows.device))
    _after(lib, rc, "fc_linear_bwd_residual" if backward else "fc_linear_fwd_residual", rows.device)
    return out


def _linear_input_grad(g: Tensor, in_size: int, weights: Sequence[Tensor], lists, precision: str,
                       scale: Tensor) -> Tensor:
    """grad_x = map^T(g) alone (frozen weights, no input activation): fc_linear_bwd reads its
    ``x`` argument only for weight gradients and activations, so the output buffer stands
    in for it."""
    lib = N.lib()
    n_active = len(lists[0])
    ws = [w.to(g.dtype).contiguous() for w in weights[:n_active]]
    sc = scale.to(device=g.device, dtype=g.dtype).contiguous()
    gx = g.new_empty((g.shape[0], int(in_size)))
    d = _linear_desc(gx, g.shape[1], lists[0], lists[1], lists[3], lists[4], lists[5], precision, 0)
    split = _split_weights(lib, d, ws, True)
    with _timed("linear_bwd", n_active, _nbytes(g, gx, *ws)):
        if split is not None:
            rc = lib.fc_linear_bwd_presplit(ctypes.byref(d), _p(g), _p(gx), _ptr_array(ws), split, _p(sc), g.shape[0],
                                            _p(gx), None, ctypes.c_void_p(status_word(g.device).data_ptr()),
                                            _stream(g.device))
        else:
            rc = lib.fc_linear_bwd(ctypes.byref(d), _p(g), _p(gx), _ptr_array(ws), _p(sc), g.shape[0], _p(gx), None,
                                   ctypes.c_void_p(status_word(g.device).data_ptr()), _stream(g.device))
    _after(lib, rc, "fc_linear_bwd", g.device)
    return gx


@torch.library.custom_op("flashcart::linear_residual_fwd", mutates_args=())
def linear_residual_fwd(x: Tensor, weights: List[Tensor], residual: Tensor, out_size: int, dot_input_precision: str,
                        in_offsets: List[int], out_offsets: List[int], m_values: List[int], f_in_values: List[int],
                        f_out_values: List[int], scale: Tensor) -> Tensor:
    """``linear_fwd(x) + residual`` with the sum done in the GEMM's epilogue: the residual
    connections around the node-level maps (the gate layer's ``node_feats +
    output_linear(...)``, reference ``nn/layers.py:609-635``; the interaction's skip sum,
    ``nn/layers.py:395-405``), without a separate pass over the rows. Frozen weights."""
    _require_cuda(x, residual, *weights)
    lists = (in_offsets, out_offsets, [0] * len(in_offsets), m_values, f_in_values, f_out_values)
    return _linear_residual_impl(x, weights, out_size, lists, dot_input_precision, scale, residual, False)


@linear_residual_fwd.register_fake
def _(x, weights, residual, out_size, dot_input_precision, in_offsets, out_offsets, m_values, f_in_values,
      f_out_values, scale):
    return x.new_empty((x.shape[0], int(out_size)))


@torch.library.custom_op("flashcart::linear_residual_bwd", mutates_args=())
def linear_residual_bwd(grad_out: Tensor, weights: List[Tensor], residual: Tensor, in_size: int,
                        dot_input_precision: str, in_offsets: List[int], out_offsets: List[int], m_values: List[int],
                        f_in_values: List[int], f_out_values: List[int], scale: Tensor) -> Tensor:
    """``map^T(grad_out) + residual``: an input gradient and the gradient that reaches the same
    tensor by another path, summed in the GEMM's epilogue. Frozen weights."""
    _require_cuda(grad_out, residual, *weights)
    lists = (in_offsets, out_offsets, [0] * len(in_offsets), m_values, f_in_values, f_out_values)
    return _linear_residual_impl(grad_out, weights, in_size, lists, dot_input_precision, scale, residual, True)


@linear_residual_bwd.register_fake
def _(grad_out, weights, residual, in_size, dot_input_precision, in_offsets, out_offsets, m_values, f_in_values,
      f_out_values, scale):
    return grad_out.new_empty((grad_out.shape[0], int(in_size)))


def _lres_setup(ctx, inputs, output):
    x, weights = inputs[0], inputs[1]
    ctx.save_for_backward(inputs[-1], *weights)
    ctx.n_w = len(weights)
    ctx.in_size = x.shape[1]
    ctx.meta = inputs[4:-1]


def _lres_backward(ctx, grad_out):
    if torch.is_grad_enabled():
        raise RuntimeError("flashcart::linear_residual_fwd was evaluated inside first_order_only(); its backward "
                           "cannot build a graph for a second derivative")
    scale, *weights = ctx.saved_tensors
    if any(w.requires_grad for w in weights):
        raise RuntimeError("flashcart::linear_residual_fwd has no weight gradient (frozen weights only)")
    g = grad_out.contiguous()
    gx = None
    if ctx.needs_input_grad[0]:
        prec, in_offs, out_offs, m, fi, fo = ctx.meta
        lists = (in_offs, out_offs, [0] * len(in_offs), m, fi, fo)
        gx = _linear_input_grad(g, ctx.in_size, weights, lists, prec, scale)
    return (gx, [None] * len(weights), g if ctx.needs_input_grad[2] else None) + (None,) * 8


linear_residual_fwd.register_autograd(_lres_backward, setup_context=_lres_setup)


@torch.library.custom_op("flashcart::linear_dbwd", mutates_args=())
def linear_dbwd(grad_out: Tensor, x: Tensor, weights: List[Tensor], v_grad_x: Tensor, v_grad_weight: List[Tensor],
                use_fp64: bool, dot_input_precision: str, need_d_grad_out: bool, need_d_x: bool,
                need_d_weight: bool, has_v_grad_x: bool, has_v_grad_weight: bool, in_offsets: List[int],
                out_offsets: List[int], weight_offsets: List[int], m_values: List[int], f_in_values: List[int],
                f_out_values: List[int], scale: Tensor) -> Tuple[Tensor, Tensor, List[Tensor]]:
    """VJP of linear_bwd, composed from the forward / backward kernels.

    With gx = g (sW) and gW = s g^T x (per rank), tangents (vx, vW) give
    d_g = vx (sW)^T + x (s vW)^T,  d_x = g (s vW),  d_W = s g^T vx.
    """
    _require_cuda(grad_out, x, *weights)
    lists = (in_offsets, out_offsets, weight_offsets, m_values, f_in_values, f_out_values)
    n = len(in_offsets)
    out_dim = grad_out.shape[1]
    d_g = grad_out.new_zeros(grad_out.shape) if need_d_grad_out else grad_out.new_empty((0,))
    d_x = torch.zeros_like(x) if need_d_x else x.new_empty((0,))
    d_w = [torch.zeros_like(w) if need_d_weight else w.new_empty((0,)) for w in weights[:n]]
    if need_d_grad_out:
        if has_v_grad_x:
            d_g = d_g + _linear_fwd_impl(v_grad_x, weights, out_dim, lists, dot_input_precision, scale)
        if has_v_grad_weight:
            d_g = d_g + _linear_fwd_impl(x, v_grad_weight, out_dim, lists, dot_input_precision, scale)
    if need_d_x and has_v_grad_weight:
        d_x, _ = _linear_bwd_impl(grad_out, x, v_grad_weight, True, False, lists, dot_input_precision, scale)
    if need_d_weight and has_v_grad_x:
        _, d_w = _linear_bwd_impl(grad_out, v_grad_x, weights, False, True, lists, dot_input_precision, scale)
    return d_g, d_x, d_w


@linear_dbwd.register_fake
def _(grad_out, x, weights, v_grad_x, v_grad_weight, use_fp64, dot_input_precision, need_d_grad_out, need_d_x,
      need_d_weight, has_v_grad_x, has_v_grad_weight, in_offsets, out_offsets, weight_offsets, m_values, f_in_values,
      f_out_values, scale):
    n = len(in_offsets)
    return (torch.empty_like(grad_out) if need_d_grad_out else grad_out.new_empty((0,)),
            torch.empty_like(x) if need_d_x else x.new_empty((0,)),
            [torch.empty_like(w) if need_d_weight else w.new_empty((0,)) for w in weights[:n]])


def _need(flag) -> bool:
    """needs_input_grad entry as a bool: list arguments report one flag per element."""
    if isinstance(flag, (list, tuple)):
        return any(bool(f) for f in flag)
    return bool(flag)


def _linear_setup(ctx, inputs, output):
    (x, weights, meta, out_size, use_fp64, prec, *lists, scale) = inputs
    ctx.save_for_backward(x, *weights, scale)
    ctx.n_w = len(weights)
    ctx.use_fp64 = bool(use_fp64)
    ctx.prec = prec
    ctx.lists = tuple(list(v) for v in lists)


def _linear_backward(ctx, grad_out):
    saved = ctx.saved_tensors
    x, weights, scale = saved[0], list(saved[1:1 + ctx.n_w]), saved[-1]
    need_x, need_w = _need(ctx.needs_input_grad[0]), _need(ctx.needs_input_grad[1])
    no_w = [None] * len(weights)
    if grad_out is None or not (need_x or need_w):
        return (None, no_w) + (None,) * 11
    gx, gws = torch.ops.flashcart.linear_bwd(grad_out, x, weights, need_x, need_w, ctx.use_fp64, ctx.prec,
                                             *ctx.lists, scale)
    if need_w:
        n = len(ctx.lists[0])
        gws = list(gws) + [torch.zeros_like(w) for w in weights[n:]]
    return (gx if need_x else None, gws if need_w else no_w) + (None,) * 11


def _linear_bwd_setup(ctx, inputs, output):
    (g, x, weights, need_x, need_w, use_fp64, prec, *lists, scale) = inputs
    ctx.save_for_backward(g, x, *weights, scale)
    ctx.n_w = len(weights)
    ctx.made = (bool(need_x), bool(need_w))
    ctx.use_fp64 = bool(use_fp64)
    ctx.prec = prec
    ctx.lists = tuple(list(v) for v in lists)
    if hasattr(ctx, "set_materialize_grads"):
        ctx.set_materialize_grads(False)


def _linear_bwd_backward(ctx, v_gx, v_gw):
    saved = ctx.saved_tensors
    g, x, weights, scale = saved[0], saved[1], list(saved[2:2 + ctx.n_w]), saved[-1]
    need_g, need_x, need_w = (_need(ctx.needs_input_grad[i]) for i in range(3))
    no_w = [None] * len(weights)
    if not (need_g or need_x or need_w):
        return (None, None, no_w) + (None,) * 11
    has_vx = v_gx is not None and v_gx.numel() != 0 and ctx.made[0]
    has_vw = (v_gw is not None and len(v_gw) > 0 and any(v is not None and v.numel() for v in v_gw)
              and ctx.made[1])
    vx = v_gx if has_vx else x.new_empty((0,))
    if has_vw:
        vw = [v if (v is not None and v.numel()) else torch.zeros_like(w) for v, w in zip(v_gw, weights)]
    else:
        vw = [w.new_empty((0,)) for w in weights]
    dg, dx, dw = torch.ops.flashcart.linear_dbwd(g, x, weights, vx, vw, ctx.use_fp64, ctx.prec, need_g, need_x,
                                                 need_w, has_vx, has_vw, *ctx.lists, scale)
    if need_w:
        n = len(ctx.lists[0])
        dw = list(dw) + [torch.zeros_like(w) for w in weights[n:]]
    return (dg if need_g else None, dx if need_x else None, dw if need_w else no_w) + (None,) * 11


linear_fwd.register_autograd(_linear_backward, setup_context=_linear_setup)
linear_bwd.register_autograd(_linear_bwd_backward, setup_context=_linear_bwd_setup)


# --------------------------------------------------------------------------- Muon Newton-Schulz

@torch.library.custom_op("flashcart::newton_schulz", mutates_args=())
def newton_schulz(update: Tensor, coeffs: List[float], steps: int, polish: List[float], polish_steps: int,
                  eps: float) -> Tensor:
    """Batched Newton-Schulz orthogonalisation in bf16 on the tensor cores
    (reference ``training/muon.py:27-61`` ``_batched_newtonschulz``): ``update`` is
    ``(batch, rows, cols)`` float32 or bfloat16; returns bfloat16 of the same shape."""
    _require_cuda(update)
    if update.dim() != 3:
        raise ValueError(f"update must be (batch, rows, cols), got shape {tuple(update.shape)}")
    if update.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError(f"update must be float32 or bfloat16, got {update.dtype}")
    lib = N.lib()
    u = update.contiguous()
    out = torch.empty(u.shape, dtype=torch.bfloat16, device=u.device)
    cf = (ctypes.c_float * 3)(*[float(v) for v in coeffs])
    pl = (ctypes.c_float * 3)(*[float(v) for v in (list(polish) + [0.0, 0.0, 0.0])[:3]])
    code = N.FC_F32 if u.dtype == torch.float32 else N.FC_BF16
    with _timed("newton_schulz", 4 * (int(steps) + int(polish_steps)) + 2, _nbytes(u, out)):
        rc = lib.fc_newton_schulz(_p(u), code, u.shape[0], u.shape[1], u.shape[2], cf, int(steps), pl,
                                  int(polish_steps), float(eps), _p(out),
                                  ctypes.c_void_p(status_word(u.device).data_ptr()), _stream(u.device))
    _after(lib, rc, "fc_newton_schulz", u.device)
    return out


@newton_schulz.register_fake
def _(update, coeffs, steps, polish, polish_steps, eps):
    return torch.empty(update.shape, dtype=torch.bfloat16, device=update.device)


# --------------------------------------------------------------------------- fused RMS layer norm

_FIRST_ORDER = threading.local()


@contextlib.contextmanager
def first_order_only():
    """Mark a region whose graph is differentiated at most once (energy -> forces and
    stress without ``create_graph``). Inside it, modules may use fused operators that
    have a first derivative but no second one (:func:`rms_norm`); a second derivative
    through them raises. ``FlashCartPotential.predict`` enters it when ``create_graph``
    is false."""
    prev = getattr(_FIRST_ORDER, "on", False)
    _FIRST_ORDER.on = True
    try:
        yield
    finally:
        _FIRST_ORDER.on = prev


def first_order_only_active() -> bool:
    return getattr(_FIRST_ORDER, "on", False)


def _rms_args(x: Tensor, gains: Tensor, l_weights: Tensor, l_max: int, features: int):
    if x.dim() != 2 or x.shape[1] != (l_max + 1) ** 2 * features:
        raise RuntimeError(f"Incorrect last dimension for node_feats. Expected {(l_max + 1) ** 2 * features}, "
                           f"got {x.shape[-1]}.")
    if x.dtype not in (torch.float32, torch.float64):
        raise ValueError(f"rms_norm supports float32 / float64, got {x.dtype}")
    g = gains.to(x.dtype).contiguous()
    lw = l_weights.to(device=x.device, dtype=x.dtype).contiguous()
    if g.numel() != (l_max + 1) * features or lw.numel() != l_max + 1:
        raise ValueError("rms_norm: gains must be (l_max+1, features) and l_weights (l_max+1,)")
    return x.contiguous(), g, lw


@torch.library.custom_op("flashcart::rms_norm_fwd", mutates_args=())
def rms_norm_fwd(x: Tensor, gains: Tensor, l_weights: Tensor, l_max: int, features: int,
                 eps: float) -> Tuple[Tensor, Tensor]:
    """Fused ``RMSLayerNorm`` forward (reference ``nn/layers.py:413-540``, affine, no
    centering): returns ``y`` and the per-row ``rstd = (mean_sq + eps)^-1/2``."""
    _require_cuda(x, gains, l_weights)
    x, g, lw = _rms_args(x, gains, l_weights, l_max, features)
    lib = N.lib()
    y = torch.empty_like(x)
    rstd = x.new_empty((x.shape[0],))
    with _timed("rms_norm_fwd", 1, _nbytes(x, y, rstd)):
        rc = lib.fc_rms_norm_fwd(int(l_max), int(features), _code(x.dtype), _p(x), _p(g), _p(lw), float(eps),
                                 x.shape[0], _p(y), _p(rstd), _stream(x.device))
    _after(lib, rc, "fc_rms_norm_fwd", x.device)
    return y, rstd


@rms_norm_fwd.register_fake
def _(x, gains, l_weights, l_max, features, eps):
    return torch.empty_like(x), x.new_empty((x.shape[0],))


@torch.library.custom_op("flashcart::rms_norm_bwd", mutates_args=())
def rms_norm_bwd(grad_y: Tensor, x: Tensor, gains: Tensor, l_weights: Tensor, rstd: Tensor, l_max: int,
                 features: int) -> Tensor:
    """First-order backward of :func:`rms_norm_fwd` with respect to ``x``."""
    _require_cuda(grad_y, x, gains, l_weights, rstd)
    x, g, lw = _rms_args(x, gains, l_weights, l_max, features)
    gy, r = grad_y.contiguous(), rstd.contiguous()
    lib = N.lib()
    gx = torch.empty_like(x)
    with _timed("rms_norm_bwd", 1, _nbytes(gy, x, r, gx)):
        rc = lib.fc_rms_norm_bwd(int(l_max), int(features), _code(x.dtype), _p(gy), _p(x), _p(g), _p(lw), _p(r),
                                 x.shape[0], _p(gx), _stream(x.device))
    _after(lib, rc, "fc_rms_norm_bwd", x.device)
    return gx


@rms_norm_bwd.register_fake
def _(grad_y, x, gains, l_weights, rstd, l_max, features):
    return torch.empty_like(x)


def _rms_setup(ctx, inputs, output):
    x, gains, l_weights, l_max, features, _ = inputs
    ctx.save_for_backward(x, gains, l_weights, output[1])
    ctx.l_max, ctx.features = l_max, features


def _rms_backward(ctx, grad_y, grad_rstd):
    if torch.is_grad_enabled():
        raise RuntimeError("flashcart::rms_norm_fwd was evaluated inside first_order_only(); its backward "
                           "cannot build a graph for a second derivative (use create_graph=False, or "
                           "evaluate the model outside first_order_only())")
    if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
        raise RuntimeError("flashcart::rms_norm_fwd: gradients of gains / l_weights are not provided")
    x, gains, l_weights, rstd = ctx.saved_tensors
    gx = None
    if ctx.needs_input_grad[0]:
        gx = rms_norm_bwd(grad_y.contiguous(), x, gains, l_weights, rstd, ctx.l_max, ctx.features)
    return gx, None, None, None, None, None


rms_norm_fwd.register_autograd(_rms_backward, setup_context=_rms_setup)


def rms_norm(x: Tensor, gains: Tensor, l_weights: Tensor, l_max: int, features: int, eps: float) -> Tensor:
    """``y = x * (mean_c sum_l l_weights[l] inv_l + eps)^-1/2 * gains[l, c]`` per row (first
    derivative only, see :func:`first_order_only`)."""
    return rms_norm_fwd(x, gains, l_weights, l_max, features, eps)[0]


# --------------------------------------------------------------------------- fused equivariant gate


@torch.library.custom_op("flashcart::gate_fwd", mutates_args=())
def gate_fwd(values: Tensor, gates: Tensor, l_max: int, features: int) -> Tensor:
    """``y[n, (l, m), c] = values[n, (l, m), c] * gates[n, l, c]`` over every rank block
    (the per-rank products and concatenation of ``EquivariantGatedLayer.forward``,
    reference ``nn/layers.py:609-635``)."""
    _require_cuda(values, gates)
    v, g = values.contiguous(), gates.contiguous()
    if v.dim() != 2 or v.shape[1] != (l_max + 1) ** 2 * features or g.numel() != v.shape[0] * (l_max + 1) * features:
        raise ValueError("gate: values must be (n, (l_max+1)^2 features) and gates (n, l_max+1, features)")
    if g.dtype != v.dtype or v.dtype not in (torch.float32, torch.float64):
        raise ValueError("gate: values and gates must share a float32 / float64 dtype")
    lib = N.lib()
    y = torch.empty_like(v)
    with _timed("gate_fwd", 1, _nbytes(v, g, y)):
        rc = lib.fc_gate_fwd(int(l_max), int(features), _code(v.dtype), _p(v), _p(g), v.shape[0], _p(y),
                             _stream(v.device))
    _after(lib, rc, "fc_gate_fwd", v.device)
    return y


@gate_fwd.register_fake
def _(values, gates, l_max, features):
    return torch.empty_like(values)


@torch.library.custom_op("flashcart::gate_bwd", mutates_args=())
def gate_bwd(grad_y: Tensor, values: Tensor, gates: Tensor, l_max: int, features: int) -> Tuple[Tensor, Tensor]:
    """First-order backward of :func:`gate_fwd`: (grad_values, grad_gates)."""
    _require_cuda(grad_y, values, gates)
    gy, v, g = grad_y.contiguous(), values.contiguous(), gates.contiguous()
    lib = N.lib()
    gv = torch.empty_like(v)
    gg = torch.empty(g.shape, dtype=g.dtype, device=g.device)
    with _timed("gate_bwd", 1, _nbytes(gy, v, g, gv, gg)):
        rc = lib.fc_gate_bwd(int(l_max), int(features), _code(v.dtype), _p(gy), _p(v), _p(g), v.shape[0], _p(gv),
                             _p(gg), _stream(v.device))
    _after(lib, rc, "fc_gate_bwd", v.device)
    return gv, gg


@gate_bwd.register_fake
def _(grad_y, values, gates, l_max, features):
    return torch.empty_like(values), torch.empty_like(gates)


def _gate_setup(ctx, inputs, output):
    values, gates, l_max, features = inputs
    ctx.save_for_backward(values, gates)
    ctx.l_max, ctx.features = l_max, features


def _gate_backward(ctx, grad_y):
    if torch.is_grad_enabled():
        raise RuntimeError("flashcart::gate_fwd was evaluated inside first_order_only(); its backward cannot "
                           "build a graph for a second derivative")
    values, gates = ctx.saved_tensors
    gv, gg = gate_bwd(grad_y.contiguous(), values, gates, ctx.l_max, ctx.features)
    return (gv if ctx.needs_input_grad[0] else None), (gg if ctx.needs_input_grad[1] else None), None, None


gate_fwd.register_autograd(_gate_backward, setup_context=_gate_setup)


# --------------------------------------------------------------------------- fused edge expansion


def _expand_index(l_max: int, device) -> Tensor:
    return torch.cat([torch.full((2 * l + 1,), l, dtype=torch.int64) for l in range(l_max + 1)]).to(device)


@torch.library.custom_op("flashcart::edge_expand_fwd", mutates_args=())
def edge_expand_fwd(moments: Tensor, h: Tensor, l_max: int, features: int, per_rank: bool) -> Tensor:
    """``out[e, k, c] = moments[e, k] * h[e, r, c]`` as rank-block rows (E, (l_max+1)^2 *
    features): ``h`` (E, features) shared by every rank, or (E, l_max+1, features) with
    ``per_rank`` (the factorised equivariant linear map of the expansion)."""
    _require_cuda(moments, h)
    t, hh = moments.contiguous(), h.contiguous()
    nc = (l_max + 1) ** 2
    if t.dim() != 2 or t.shape[1] != nc:
        raise ValueError(f"edge_expand: moments must be (E, {nc}), got {tuple(t.shape)}")
    if hh.numel() != t.shape[0] * (l_max + 1 if per_rank else 1) * features or hh.dtype != t.dtype:
        raise ValueError("edge_expand: h must be (E, features) or (E, l_max+1, features) with per_rank, same dtype")
    lib = N.lib()
    out = t.new_empty((t.shape[0], nc * features))
    with _timed("edge_expand_fwd", 1, _nbytes(t, hh, out)):
        rc = lib.fc_edge_expand_fwd(int(l_max), int(features), int(bool(per_rank)), _code(t.dtype), _p(t), _p(hh),
                                    t.shape[0], _p(out), _stream(t.device))
    _after(lib, rc, "fc_edge_expand_fwd", t.device)
    return out


@edge_expand_fwd.register_fake
def _(moments, h, l_max, features, per_rank):
    return moments.new_empty((moments.shape[0], (l_max + 1) ** 2 * features))


@torch.library.custom_op("flashcart::edge_expand_bwd", mutates_args=())
def edge_expand_bwd(grad_out: Tensor, moments: Tensor, h: Tensor, l_max: int, features: int,
                    per_rank: bool) -> Tuple[Tensor, Tensor]:
    """First-order backward of :func:`edge_expand_fwd`: (grad_moments, grad_h)."""
    _require_cuda(grad_out, moments, h)
    g, t, hh = grad_out.contiguous(), moments.contiguous(), h.contiguous()
    lib = N.lib()
    gt = torch.empty_like(t)
    gh = torch.empty_like(hh)
    with _timed("edge_expand_bwd", 1, _nbytes(g, t, hh, gt, gh)):
        rc = lib.fc_edge_expand_bwd(int(l_max), int(features), int(bool(per_rank)), _code(t.dtype), _p(g), _p(t),
                                    _p(hh), t.shape[0], _p(gt), _p(gh), _stream(t.device))
    _after(lib, rc, "fc_edge_expand_bwd", t.device)
    return gt, gh


@edge_expand_bwd.register_fake
def _(grad_out, moments, h, l_max, features, per_rank):
    return torch.empty_like(moments), torch.empty_like(h)


def _expand_setup(ctx, inputs, output):
    moments, h, l_max, features, per_rank = inputs
    ctx.save_for_backward(moments, h)
    ctx.l_max, ctx.features, ctx.per_rank = l_max, features, per_rank


def _expand_backward(ctx, grad_out):
    moments, h = ctx.saved_tensors
    L, F, pr = ctx.l_max, ctx.features, ctx.per_rank
    if torch.is_grad_enabled():
        # building a graph for a second derivative: the same gradient from differentiable ops
        e, nc = moments.shape
        g = grad_out.reshape(e, nc, F)
        hr = h.reshape(e, L + 1 if pr else 1, F)
        hx = hr.index_select(1, _expand_index(L, h.device)) if pr else hr
        gt = (g * hx).sum(-1)
        gm = g * moments.unsqueeze(-1)
        gh = (torch.zeros_like(hr).index_add(1, _expand_index(L, h.device), gm) if pr else gm.sum(1, keepdim=True))
        return gt, gh.reshape(h.shape), None, None, None
    gt, gh = edge_expand_bwd(grad_out.contiguous(), moments, h, L, F, pr)
    return (gt if ctx.needs_input_grad[0] else None), (gh if ctx.needs_input_grad[1] else None), None, None, None


edge_expand_fwd.register_autograd(_expand_backward, setup_context=_expand_setup)


# --------------------------------------------------------------------------- fused edge geometry


def _geom_desc(l_max: int, n_radial: int, cosine: bool, poly_order: int, use_shifts: bool, dtype: torch.dtype,
               r_min: float, r_max: float, r_cut: float) -> N.EdgeGeometryDesc:
    return N.EdgeGeometryDesc(int(l_max), int(n_radial), int(bool(cosine)), int(poly_order), int(bool(use_shifts)),
                              _code(dtype), float(r_min), float(r_max), float(r_cut))


def _geom_inputs(positions: Tensor, cells: Tensor, shifts: Tensor, edge_index: Tensor, batch: Tensor):
    if positions.dtype not in (torch.float32, torch.float64):
        raise ValueError(f"edge_geometry supports float32 / float64 positions, got {positions.dtype}")
    if positions.dim() != 2 or positions.shape[1] != 3:
        raise ValueError(f"edge_geometry: positions must be (n, 3), got {tuple(positions.shape)}")
    if edge_index.dim() != 2 or edge_index.shape[0] != 2:
        raise ValueError(f"edge_geometry: edge_index must be (2, E), got {tuple(edge_index.shape)}")
    c = cells.to(positions.dtype).reshape(-1, 3, 3).contiguous()
    s = shifts if shifts.dtype == torch.int32 else shifts.round().to(torch.int32)
    return (positions.contiguous(), c, s.contiguous(), edge_index.to(torch.int64).contiguous(),
            batch.to(torch.int64).contiguous())


@torch.library.custom_op("flashcart::edge_geometry_fwd", mutates_args=())
def edge_geometry_fwd(positions: Tensor, cells: Tensor, shifts: Tensor, edge_index: Tensor, batch: Tensor,
                      l_max: int, n_radial: int, cosine: bool, poly_order: int, r_min: float, r_max: float,
                      r_cut: float, use_shifts: bool) -> Tuple[Tensor, Tensor]:
    """Edge attributes T^l(v / |v|) (E, (l_max+1)^2) and radial features Chebyshev(|v|) *
    envelope(|v|) (E, n_radial) of the edges v = r_j - r_i + S . cell in one kernel
    (reference chain ``model/flashcart.py:264-286`` -> ``utils/geometry.py:25-53``,
    ``o3/irreps.py:54-72``, ``nn/radial.py:98-128, 181-245``)."""
    _require_cuda(positions, cells, edge_index)
    pos, c, s, ei, b = _geom_inputs(positions, cells, shifts, edge_index, batch)
    e = ei.shape[1]
    attrs = pos.new_empty((e, (l_max + 1) ** 2))
    radial = pos.new_empty((e, n_radial))
    lib = N.lib()
    d = _geom_desc(l_max, n_radial, cosine, poly_order, use_shifts, pos.dtype, r_min, r_max, r_cut)
    with _timed("edge_geometry_fwd", 1, _nbytes(pos, s, ei, attrs, radial)):
        rc = lib.fc_edge_geometry_fwd(ctypes.byref(d), _p(pos), pos.shape[0], _p(c), c.shape[0], _p(s), _p(ei), _p(b),
                                      e, _p(attrs), _p(radial), _p(status_word(pos.device)), _stream(pos.device))
    _after(lib, rc, "fc_edge_geometry_fwd", pos.device)
    return attrs, radial


@edge_geometry_fwd.register_fake
def _(positions, cells, shifts, edge_index, batch, l_max, n_radial, cosine, poly_order, r_min, r_max, r_cut,
      use_shifts):
    e = edge_index.shape[1]
    return positions.new_empty((e, (l_max + 1) ** 2)), positions.new_empty((e, n_radial))


@torch.library.custom_op("flashcart::edge_geometry_bwd", mutates_args=())
def edge_geometry_bwd(grad_attrs: Tensor, grad_radial: Tensor, positions: Tensor, cells: Tensor, shifts: Tensor,
                      edge_index: Tensor, batch: Tensor, l_max: int, n_radial: int, cosine: bool, poly_order: int,
                      r_min: float, r_max: float, r_cut: float, use_shifts: bool) -> Tuple[Tensor, Tensor]:
    """First derivative of :func:`edge_geometry_fwd`: (grad_positions (N, 3), grad_cells
    (G, 3, 3)); an empty gradient tensor stands for zero."""
    _require_cuda(positions, cells, edge_index)
    pos, c, s, ei, b = _geom_inputs(positions, cells, shifts, edge_index, batch)
    ga = grad_attrs.contiguous() if grad_attrs.numel() else None
    gr = grad_radial.contiguous() if grad_radial.numel() else None
    g_pos = torch.empty_like(pos)
    g_cells = torch.empty_like(c)
    lib = N.lib()
    d = _geom_desc(l_max, n_radial, cosine, poly_order, use_shifts, pos.dtype, r_min, r_max, r_cut)
    with _timed("edge_geometry_bwd", 1, _nbytes(pos, s, ei, ga, gr, g_pos)):
        rc = lib.fc_edge_geometry_bwd(ctypes.byref(d), _p(pos), pos.shape[0], _p(c), c.shape[0], _p(s), _p(ei), _p(b),
                                      ei.shape[1], _p(ga), _p(gr), _p(g_pos), _p(g_cells),
                                      _p(status_word(pos.device)), _stream(pos.device))
    _after(lib, rc, "fc_edge_geometry_bwd", pos.device)
    return g_pos, g_cells.reshape(cells.shape)


@edge_geometry_bwd.register_fake
def _(grad_attrs, grad_radial, positions, cells, shifts, edge_index, batch, l_max, n_radial, cosine, poly_order,
      r_min, r_max, r_cut, use_shifts):
    return torch.empty_like(positions), torch.empty_like(cells)


def _geom_setup(ctx, inputs, output):
    positions, cells, shifts, edge_index, batch = inputs[:5]
    ctx.save_for_backward(positions, cells, shifts, edge_index, batch)
    ctx.args = inputs[5:]


def _geom_backward(ctx, grad_attrs, grad_radial):
    if torch.is_grad_enabled():
        raise RuntimeError("flashcart::edge_geometry_fwd was evaluated inside first_order_only(); its backward "
                           "cannot build a graph for a second derivative")
    positions, cells, shifts, edge_index, batch = ctx.saved_tensors
    ga = grad_attrs if grad_attrs is not None else positions.new_zeros(0)
    gr = grad_radial if grad_radial is not None else positions.new_zeros(0)
    g_pos, g_cells = edge_geometry_bwd(ga, gr, positions, cells, shifts, edge_index, batch, *ctx.args)
    return ((g_pos if ctx.needs_input_grad[0] else None), (g_cells if ctx.needs_input_grad[1] else None),
            None, None, None) + (None,) * len(ctx.args)


edge_geometry_fwd.register_autograd(_geom_backward, setup_context=_geom_setup)


def edge_geometry(positions: Tensor, cells: Tensor, shifts: Tensor, edge_index: Tensor, batch: Tensor, l_max: int,
                  n_radial: int, cosine: bool, poly_order: int, r_min: float, r_max: float, r_cut: float,
                  use_shifts: bool = True) -> Tuple[Tensor, Tensor]:
    """(edge_attrs, radial) of :func:`edge_geometry_fwd`, differentiable once with respect to
    positions and cells (see :func:`first_order_only`)."""
    return edge_geometry_fwd(positions, cells, shifts, edge_index, batch, int(l_max), int(n_radial), bool(cosine),
                             int(poly_order), float(r_min), float(r_max), float(r_cut), bool(use_shifts))


def _vec_input(vectors: Tensor) -> Tensor:
    if vectors.dtype not in (torch.float32, torch.float64):
        raise ValueError(f"edge_geometry_vec supports float32 / float64 vectors, got {vectors.dtype}")
    if vectors.dim() != 2 or vectors.shape[1] != 3:
        raise ValueError(f"edge_geometry_vec: vectors must be (E, 3), got {tuple(vectors.shape)}")
    return vectors.contiguous()


@torch.library.custom_op("flashcart::edge_geometry_vec_fwd", mutates_args=())
def edge_geometry_vec_fwd(vectors: Tensor, l_max: int, n_radial: int, cosine: bool, poly_order: int, r_min: float,
                          r_max: float, r_cut: float) -> Tuple[Tensor, Tensor]:
    """:func:`edge_geometry_fwd` of edge vectors given per edge (the LAMMPS ML-IAP ``rij``,
    reference ``calculators/lammps_mliap.py:122-170``; the ``vectors`` branch of
    ``model/flashcart.py:264-286``)."""
    _require_cuda(vectors)
    v = _vec_input(vectors)
    e = v.shape[0]
    attrs = v.new_empty((e, (l_max + 1) ** 2))
    radial = v.new_empty((e, n_radial))
    lib = N.lib()
    d = _geom_desc(l_max, n_radial, cosine, poly_order, False, v.dtype, r_min, r_max, r_cut)
    with _timed("edge_geometry_fwd", 1, _nbytes(v, attrs, radial)):
        rc = lib.fc_edge_geometry_vec_fwd(ctypes.byref(d), _p(v), e, _p(attrs), _p(radial),
                                          _p(status_word(v.device)), _stream(v.device))
    _after(lib, rc, "fc_edge_geometry_vec_fwd", v.device)
    return attrs, radial


@edge_geometry_vec_fwd.register_fake
def _(vectors, l_max, n_radial, cosine, poly_order, r_min, r_max, r_cut):
    e = vectors.shape[0]
    return vectors.new_empty((e, (l_max + 1) ** 2)), vectors.new_empty((e, n_radial))


@torch.library.custom_op("flashcart::edge_geometry_vec_bwd", mutates_args=())
def edge_geometry_vec_bwd(grad_attrs: Tensor, grad_radial: Tensor, vectors: Tensor, l_max: int, n_radial: int,
                          cosine: bool, poly_order: int, r_min: float, r_max: float, r_cut: float) -> Tensor:
    """dE/dv per edge (E, 3) from the gradients of :func:`edge_geometry_vec_fwd`'s outputs
    (an empty gradient tensor stands for zero): the LAMMPS pair forces."""
    _require_cuda(vectors)
    v = _vec_input(vectors)
    ga = grad_attrs.contiguous() if grad_attrs.numel() else None
    gr = grad_radial.contiguous() if grad_radial.numel() else None
    g_v = torch.empty_like(v)
    lib = N.lib()
    d = _geom_desc(l_max, n_radial, cosine, poly_order, False, v.dtype, r_min, r_max, r_cut)
    with _timed("edge_geometry_bwd", 1, _nbytes(v, ga, gr, g_v)):
        rc = lib.fc_edge_geometry_vec_bwd(ctypes.byref(d), _p(v), v.shape[0], _p(ga), _p(gr), _p(g_v),
                                          _p(status_word(v.device)), _stream(v.device))
    _after(lib, rc, "fc_edge_geometry_vec_bwd", v.device)
    return g_v


@edge_geometry_vec_bwd.register_fake
def _(grad_attrs, grad_radial, vectors, l_max, n_radial, cosine, poly_order, r_min, r_max, r_cut):
    return torch.empty_like(vectors)


def _geom_vec_setup(ctx, inputs, output):
    ctx.save_for_backward(inputs[0])
    ctx.args = inputs[1:]


def _geom_vec_backward(ctx, grad_attrs, grad_radial):
    if torch.is_grad_enabled():
        raise RuntimeError("flashcart::edge_geometry_vec_fwd was evaluated inside first_order_only(); its backward "
                           "cannot build a graph for a second derivative")
    (vectors,) = ctx.saved_tensors
    ga = grad_attrs if grad_attrs is not None else vectors.new_zeros(0)
    gr = grad_radial if grad_radial is not None else vectors.new_zeros(0)
    return (edge_geometry_vec_bwd(ga, gr, vectors, *ctx.args),) + (None,) * len(ctx.args)


edge_geometry_vec_fwd.register_autograd(_geom_vec_backward, setup_context=_geom_vec_setup)


def edge_geometry_vec(vectors: Tensor, l_max: int, n_radial: int, cosine: bool, poly_order: int, r_min: float,
                      r_max: float, r_cut: float) -> Tuple[Tensor, Tensor]:
    """(edge_attrs, radial) of edge vectors given per edge, differentiable once with respect
    to the vectors (see :func:`first_order_only`)."""
    return edge_geometry_vec_fwd(vectors, int(l_max), int(n_radial), bool(cosine), int(poly_order), float(r_min),
                                 float(r_max), float(r_cut))


# --------------------------------------------------------------------------- halo exchange rows


def halo_pack(x: Tensor, idx: Tensor, out: Optional[Tensor] = None) -> Tensor:
    """``buf[k] = x[idx[k]]`` for rows of any width (``fc_halo_pack``): the send buffer of a
    halo exchange, one coalesced row copy per index (reference semantics: the owner rows
    that ``lammps_forward_exchange`` sends, ``utils/lammps.py:67-94``). ``out``, when
    given, is the contiguous (len(idx), ...) buffer written in place (e.g. the ghost rows
    of a feature matrix)."""
    _require_cuda(x, idx)
    xc = x.contiguous()
    re = 1
    for d in xc.shape[1:]:
        re *= int(d)
    if out is None:
        buf = xc.new_empty((idx.numel(),) + tuple(xc.shape[1:]))
    else:
        if (not out.is_contiguous() or out.dtype != xc.dtype or out.device != xc.device
                or tuple(out.shape) != (idx.numel(),) + tuple(xc.shape[1:])):
            raise ValueError("halo_pack: out must be a contiguous (len(idx), ...) tensor of x's dtype and device")
        buf = out
    if idx.numel() == 0:
        return buf
    lib = N.lib()
    with _timed("halo_pack", 1, _nbytes(buf) * 2):
        rc = lib.fc_halo_pack(_p(xc), xc.shape[0], re, _code(xc.dtype), _p(idx), idx.numel(), _p(buf),
                              _p(status_word(x.device)), _stream(x.device))
    _after(lib, rc, "fc_halo_pack", x.device)
    return buf


def halo_unpack_(x: Tensor, buf: Tensor, idx: Tensor, accumulate: bool) -> Tensor:
    """``x[idx[k]] = buf[k]`` (ghost rows receive their owners' features) or, with
    ``accumulate``, ``x[idx[k]] += buf[k]`` (ghost gradients added to their owners;
    ``lammps_reverse_exchange``, ``utils/lammps.py:96-118``), in place (``fc_halo_unpack``)."""
    _require_cuda(x, buf, idx)
    if idx.numel() == 0:
        return x
    if not x.is_contiguous():
        raise ValueError("halo_unpack_: x must be contiguous")
    b = buf.contiguous()
    lib = N.lib()
    re = 1
    for d in b.shape[1:]:
        re *= int(d)
    with _timed("halo_unpack", 1, _nbytes(b) * 2):
        rc = lib.fc_halo_unpack(_p(b), idx.numel(), re, _code(b.dtype), _p(idx), _p(x), x.shape[0],
                                int(bool(accumulate)), _p(status_word(x.device)), _stream(x.device))
    _after(lib, rc, "fc_halo_unpack", x.device)
    return x


class timed_region:
    """CUDA-event timing of a host region under the kernel timer (e.g. a collective); it
    counts no launch of this library."""

    def __init__(self, name: str, nbytes: int = 0):
        self._t = _timed(name, 0, nbytes)

    def __enter__(self):
        return self._t.__enter__()

    def __exit__(self, *exc):
        return self._t.__exit__(*exc)
