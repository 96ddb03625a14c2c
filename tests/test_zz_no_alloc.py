"""The allocation-free convolution entry point (fc_tp_conv_fwd_noalloc).

Some callers cannot allocate device memory themselves -- an MD engine plug-in whose
memory manager owns every device byte, or a time-step loop that may not call cudaMalloc
because it can synchronise the device. For them the library offers one convolution forward that keeps its receiver-CSR
workspace in a fixed array of its own device memory. This file is collected last so
that a failure here cannot hide the rest of the suite; it passes both alone and after
the other tests (the workspace keeps whatever the previous call left, and the entry
point rewrites all of it).
"""

import ctypes

import pytest
import torch

import abi_calls as A
from flashcart_b200 import _native as N

pytestmark = pytest.mark.gpu


def _inputs(seed, n_nodes, n_edges, C, dev):
    g = torch.Generator().manual_seed(seed)
    idx_i = torch.sort(torch.randint(0, n_nodes, (n_edges,), generator=g)).values.to(dev)
    idx_j = torch.randint(0, n_nodes, (n_edges,), generator=g).to(dev)
    in1 = torch.randn(n_nodes, 9 * C, generator=g).to(dev)
    in2 = torch.randn(n_edges, 9, generator=g).to(dev)
    w = torch.randn(n_edges, 11 * C, generator=g).to(dev)
    return idx_i, idx_j, in1, in2, w


def _noalloc(lib, meta, in1, in2, w, idx_i, idx_j, status):
    d = A.desc(meta, in1.dtype)
    out = torch.full((in1.shape[0], 35 * meta[3]), float("nan"), device=in1.device)
    rc = lib.fc_tp_conv_fwd_noalloc(ctypes.byref(d), A.p(in1), A.p(in2), A.p(w), A.p(idx_i), A.p(idx_j),
                                    in1.shape[0], idx_i.numel(), A.p(out), A.p(status), A.stream_of(in1))
    N.check(lib, rc, "fc_tp_conv_fwd_noalloc")
    return out


def test_no_alloc_convolution_matches_the_allocating_entry_point(cuda_device):
    lib = N.lib()
    C = 64
    meta = [2, 2, 2, C, 1, 0, 0, 0]
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    # two calls in a row with different graphs and sizes: the shared workspace is rebuilt each time
    for seed, n_nodes, n_edges in ((1, 3000, 40000), (2, 1700, 26000)):
        idx_i, idx_j, in1, in2, w = _inputs(seed, n_nodes, n_edges, C, cuda_device)
        got = _noalloc(lib, meta, in1, in2, w, idx_i, idx_j, status)
        want = A.tp_fwd(lib, meta, in1, in2, w, idx_i, idx_j, status)
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        assert torch.isfinite(got).all()
        assert (got - want).abs().max().item() <= 1e-6 * max(1.0, want.abs().max().item())


def test_no_alloc_rejects_graphs_beyond_its_workspace(cuda_device):
    lib = N.lib()
    meta = [1, 1, 1, 32, 1, 0, 0, 0]
    d = A.desc(meta, torch.float32)
    too_many = N.FC_NOALLOC_MAX_NODES + 1
    rc = lib.fc_tp_conv_fwd_noalloc(ctypes.byref(d), None, None, None, None, None, too_many, 0, None, None, None)
    assert rc == N.FC_ERR_CAPACITY
    assert b"workspace" in lib.fc_last_error()
