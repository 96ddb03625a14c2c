"""Neighbour lists: the host cell list against the brute force (CPU), and the GPU cell
list (fc_neighbor_count / fc_neighbor_fill) against the host list, element for element.

The reference's list comes from matscipy (an unpinned, unvendored dependency, not
installed here), so parity for lists is exact agreement between independent searches in
the canonical (i, j, S) order, with the distance test in float64.
"""

import ctypes

import numpy as np
import pytest
import torch

from flashcart_b200 import _native as N
from flashcart_b200.data import neighbors, synthetic


def _random_box(n, L, seed):
    rng = np.random.default_rng(seed)
    pos = rng.uniform(0.0, 1.0, size=(n, 3)) * L
    pos[: n // 5] += rng.integers(-2, 3, size=(n // 5, 3)) * L  # some atoms outside the cell
    return pos, np.diag(L).astype(np.float64)


def test_host_cell_list_equals_bruteforce():
    s = synthetic.water_box(6, 6, 6, seed=3)
    a = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
    b = neighbors.neighbor_list_bruteforce(s["positions"], s["cell"], s["pbc"], 5.0)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    pos, cell = _random_box(400, np.array([16.0, 17.5, 15.2]), 1)
    a = neighbors.neighbor_list(pos, cell, [True] * 3, 4.9)
    b = neighbors.neighbor_list_bruteforce(pos, cell, [True] * 3, 4.9)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    assert (np.diff(a[0][0]) >= 0).all()


def test_neighbor_descriptor_validation(emu_lib):
    d = N.NlDesc()
    for k in range(3):
        d.lengths[k], d.inv_lengths[k], d.bin_widths[k], d.bins[k] = 12.0, 1 / 12.0, 6.0, 2
    d.r_max_sq = 25.0
    assert emu_lib.fc_neighbor_workspace_bytes(ctypes.byref(d), 10) == N.FC_ERR_UNSUPPORTED
    for k in range(3):
        d.lengths[k], d.inv_lengths[k], d.bin_widths[k], d.bins[k] = 18.0, 1 / 18.0, 6.0, 3
    assert emu_lib.fc_neighbor_workspace_bytes(ctypes.byref(d), 10) > 0
    d.r_max_sq = 49.0  # bin width 6 below r_max 7
    assert emu_lib.fc_neighbor_workspace_bytes(ctypes.byref(d), 10) == N.FC_ERR_INVALID


def _check_device_list(pos, cell, r_max, dev):
    ref_ei, ref_sh = neighbors.neighbor_list(pos, cell, [True] * 3, r_max, device="cpu")
    ei, sh = neighbors.neighbor_list_device(pos, cell, [True] * 3, r_max, device=dev)
    assert ei.is_cuda and ei.dtype == torch.int64 and sh.dtype == torch.int32
    assert torch.equal(ei.cpu(), torch.as_tensor(ref_ei))
    assert torch.equal(sh.cpu(), torch.as_tensor(ref_sh).to(torch.int32))
    return ei.shape[1]


@pytest.mark.gpu
def test_gpu_neighbor_list_equals_host_list(cuda_device):
    s = synthetic.water_box(6, 6, 6, seed=3)
    assert _check_device_list(s["positions"], s["cell"], 5.0, cuda_device) > 0
    pos, cell = _random_box(3000, np.array([21.0, 18.3, 30.7]), 2)
    assert _check_device_list(pos, cell, 5.5, cuda_device) > 0


@pytest.mark.gpu
def test_gpu_neighbor_list_config3_box(cuda_device):
    """The benchmark cell: 27,648 atoms, ~1.49 M edges, 14 x 14 x 9 bins."""
    s = synthetic.water_box(24, 24, 16, seed=0)
    n_edges = _check_device_list(s["positions"], s["cell"], 5.0, cuda_device)
    assert 1_400_000 < n_edges < 1_600_000
