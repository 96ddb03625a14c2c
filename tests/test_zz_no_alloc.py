"""The allocation-free convolution entry point (fc_tp_conv_fwd_noalloc).

Some callers cannot allocate device memory themselves -- an MD engine plug-in whose
memory manager owns every device byte, or a time-step loop that may not call cudaMalloc
because it can synchronise the device. For them the library offers one convolution
forward that keeps its receiver-CSR workspace in a fixed array of its own device memory.
This file is collected last so that a failure here cannot hide the rest of the suite; it
passes both alone and after the other tests (the workspace keeps whatever the previous
call left, and the entry point rewrites all of it).

Checked here: the result against the float64 CPU oracle and against the allocating entry
points (fc_build_rowptr + fc_tp_fwd) on two calls in a row; senders beyond the receivers
(the ghost atoms of an MD plug-in); a graph at exactly the workspace capacity with edges
on its last receiver; an out-of-range sender reported through the status word; no device
memory taken by the calls; sizes beyond the capacity rejected before any launch.
"""

import ctypes

import pytest
import torch

import abi_calls as A
from flashcart_b200 import _native as N
from oracle import stf_oracle as O

pytestmark = pytest.mark.gpu

C = 64
META = [2, 2, 2, C, 1, 0, 0, 0]  # TensorProduct(2, 2, 2, C, 1): 11 paths, 35 output components


def _inputs(seed, n_recv, n_send, n_edges, dev, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    idx_i = torch.sort(torch.randint(0, n_recv, (n_edges,), generator=g)).values
    idx_j = torch.randint(0, n_send, (n_edges,), generator=g)
    in1 = torch.randn(n_send, 9 * C, generator=g, dtype=torch.float64)
    in2 = torch.randn(n_edges, 9, generator=g, dtype=torch.float64)
    w = torch.randn(n_edges, 11 * C, generator=g, dtype=torch.float64)
    host = (idx_i, idx_j, in1, in2, w)
    dev_t = (idx_i.to(dev), idx_j.to(dev), in1.to(dev, dtype), in2.to(dev, dtype), w.to(dev, dtype))
    return host, dev_t


def _noalloc(lib, in1, in2, w, idx_i, idx_j, n_recv, status):
    d = A.desc(META, in1.dtype)
    out = torch.full((n_recv, 35 * C), float("nan"), device=in1.device, dtype=in1.dtype)
    rc = lib.fc_tp_conv_fwd_noalloc(ctypes.byref(d), A.p(in1), A.p(in2), A.p(w), A.p(idx_i), A.p(idx_j),
                                    n_recv, in1.shape[0], idx_i.numel(), A.p(out), A.p(status), A.stream_of(in1))
    N.check(lib, rc, "fc_tp_conv_fwd_noalloc")
    return out


def _allocating(lib, in1, in2, w, idx_i, idx_j, n_recv, status):
    d = A.desc(META, in1.dtype)
    out = torch.full((n_recv, 35 * C), float("nan"), device=in1.device, dtype=in1.dtype)
    rp = A.rowptr(lib, idx_i, n_recv, status)
    rc = lib.fc_tp_fwd(ctypes.byref(d), A.p(in1), A.p(in2), A.p(w), A.p(rp), A.p(idx_j), n_recv, in1.shape[0],
                       in2.shape[0], A.p(out), A.p(status), A.stream_of(in1))
    N.check(lib, rc, "fc_tp_fwd")
    return out


def _oracle(host, n_recv):
    idx_i, idx_j, in1, in2, w = host
    return O.tensor_product(in1, in2, w, idx_i, idx_j, 2, 2, 2, C, 1)[:n_recv]


def _close(got, want, rel):
    err = (got.double().cpu() - want).abs().max().item()
    return err <= rel * max(1.0, want.abs().max().item()), err


def test_no_alloc_convolution_matches_oracle_and_allocating_entry_point(cuda_device):
    lib = N.lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    # two calls in a row with different graphs and sizes: the shared workspace is rebuilt each
    # time; the second graph has ghost senders (rows n_recv .. n_send-1 of in1 send, never receive)
    for seed, n_recv, n_send, n_edges in ((1, 3000, 3000, 40000), (2, 1700, 2300, 26000)):
        host, (idx_i, idx_j, in1, in2, w) = _inputs(seed, n_recv, n_send, n_edges, cuda_device)
        got = _noalloc(lib, in1, in2, w, idx_i, idx_j, n_recv, status)
        want = _allocating(lib, in1, in2, w, idx_i, idx_j, n_recv, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.isfinite(got).all()
        ok, err = _close(got, want.double().cpu(), 1e-6)
        assert ok, f"no-alloc vs fc_tp_fwd: {err:.3e}"
        ok, err = _close(got, _oracle(host, n_recv), 2e-5)
        assert ok, f"no-alloc vs float64 oracle: {err:.3e}"


def test_no_alloc_float64_matches_oracle_with_ghost_senders(cuda_device):
    lib = N.lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    host, (idx_i, idx_j, in1, in2, w) = _inputs(3, 500, 900, 7000, cuda_device, torch.float64)
    got = _noalloc(lib, in1, in2, w, idx_i, idx_j, 500, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ok, err = _close(got, _oracle(host, 500), 1e-12)
    assert ok, f"float64 no-alloc vs oracle: {err:.3e}"


def test_no_alloc_at_workspace_capacity(cuda_device):
    """n_nodes == FC_NOALLOC_MAX_NODES writes the workspace's last entry (rowptr[n_nodes]);
    edges sit on the first, a middle and the last receiver."""
    lib = N.lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    n = N.FC_NOALLOC_MAX_NODES
    g = torch.Generator().manual_seed(4)
    recv = torch.tensor([0, 0, n // 2, n - 1, n - 1, n - 1])
    send = torch.tensor([n - 1, 5, 0, n // 2, n - 1, 12345])
    dev = cuda_device
    in1 = torch.randn(n, 9 * C, generator=torch.Generator(device=dev).manual_seed(4), device=dev)
    in2 = torch.randn(recv.numel(), 9, generator=g, dtype=torch.float64)
    w = torch.randn(recv.numel(), 11 * C, generator=g, dtype=torch.float64)
    got = _noalloc(lib, in1, in2.to(dev, torch.float32), w.to(dev, torch.float32), recv.to(dev), send.to(dev), n,
                   status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # only the touched rows need the (small) oracle; every other row is an empty sum. The
    # oracle gets the sent rows only (its output has as many rows as its in1).
    touched = torch.unique(recv)
    sub_recv = torch.searchsorted(touched, recv)
    sent = in1[send.to(dev)].double().cpu()
    want_rows = O.tensor_product(sent, in2.float().double(), w.float().double(), sub_recv,
                                 torch.arange(send.numel()), 2, 2, 2, C, 1)[:touched.numel()]
    ok, err = _close(got[touched.to(dev)], want_rows, 2e-5)
    assert ok, f"touched rows vs oracle: {err:.3e}"
    row_abs = got.abs().sum(dim=1).cpu()
    mask = torch.ones(n, dtype=torch.bool)
    mask[touched] = False
    assert (row_abs[mask] == 0).all()


def test_no_alloc_flags_out_of_range_sender(cuda_device):
    lib = N.lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _, (idx_i, idx_j, in1, in2, w) = _inputs(5, 200, 200, 2000, cuda_device)
    idx_j[17] = 200  # one past the sender rows
    _noalloc(lib, in1, in2, w, idx_i, idx_j, 200, status)
    torch.cuda.synchronize()
    assert int(status.item()) & N.FC_DEV_BAD_INDEX


def test_no_alloc_calls_take_no_device_memory(cuda_device):
    lib = N.lib()
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _, (idx_i, idx_j, in1, in2, w) = _inputs(6, 3000, 3600, 40000, cuda_device)
    d = A.desc(META, in1.dtype)
    out = torch.empty((3000, 35 * C), device=cuda_device)
    args = (ctypes.byref(d), A.p(in1), A.p(in2), A.p(w), A.p(idx_i), A.p(idx_j), 3000, 3600, idx_i.numel(),
            A.p(out), A.p(status), A.stream_of(in1))
    N.check(lib, lib.fc_tp_conv_fwd_noalloc(*args), "fc_tp_conv_fwd_noalloc")  # first call: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda_device)
    torch_alloc0 = torch.cuda.memory_allocated(cuda_device)
    for _ in range(3):
        N.check(lib, lib.fc_tp_conv_fwd_noalloc(*args), "fc_tp_conv_fwd_noalloc")
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda_device)
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    assert torch.cuda.memory_allocated(cuda_device) == torch_alloc0
    assert int(status.item()) == 0


def test_no_alloc_rejects_graphs_beyond_its_workspace(cuda_device):
    lib = N.lib()
    d = A.desc([1, 1, 1, 32, 1, 0, 0, 0], torch.float32)
    too_many = N.FC_NOALLOC_MAX_NODES + 1
    rc = lib.fc_tp_conv_fwd_noalloc(ctypes.byref(d), None, None, None, None, None, too_many, too_many, 0, None, None,
                                    None)
    assert rc == N.FC_ERR_CAPACITY
    assert b"workspace" in lib.fc_last_error()
