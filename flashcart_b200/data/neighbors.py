"""Periodic neighbour lists in a canonical, receiver-sorted order.

The reference builds its lists with matscipy's ``neighbour_list("ijS")`` (reference
``data/neighbors.py:120-143``; matscipy is an unpinned, unvendored dependency): all
pairs (i, j, S) with |r_j - r_i + S . cell| < r_max, the self pair (i, i, 0) removed,
row 0 = receiver i, row 1 = sender j, edges grouped by ascending i (required by the
tensor-product convolution). Here the same set is produced in a fully canonical
order -- lexicographic in (i, j, S_x, S_y, S_z) -- with the distance test in float64:

* ``neighbor_list_bruteforce``: every (i, j) against every periodic image that can be
  within r_max (small systems, and the oracle of the cell list);
* ``neighbor_list``: a binned cell list for orthorhombic cells of at least three bins
  per periodic axis, falling back to the brute force otherwise;
* ``neighbor_list_device``: the same cell list as sm_100a kernels (``fc_neighbor_count``
  / ``fc_neighbor_fill``), the edges built and sorted on the GPU and returned as device
  tensors (``neighbor_list(device="cuda")`` uses it when the cell qualifies).
All evaluate the same float64 expressions for the wrap, the bins and the distance, so
their edge sets and orders agree exactly.
"""

from __future__ import annotations

import math
from typing import Tuple

import numpy as np
import torch


def _image_range(cell: np.ndarray, pbc, r_max: float) -> np.ndarray:
    """Number of periodic images per axis that can hold a neighbour within r_max."""
    inv = np.linalg.inv(cell)
    n = []
    for k in range(3):
        if not pbc[k]:
            n.append(0)
            continue
        spacing = 1.0 / np.linalg.norm(inv[:, k])  # distance between lattice planes
        n.append(int(math.ceil(r_max / spacing)))
    return np.array(n)


def _wrap(positions: np.ndarray, cell: np.ndarray, pbc) -> Tuple[np.ndarray, np.ndarray]:
    frac = positions @ np.linalg.inv(cell)
    wrap = np.where(np.asarray(pbc)[None, :], np.floor(frac), 0.0)
    return positions - wrap @ cell, wrap.astype(np.int64)


def _canonical(i, j, s):
    order = np.lexsort((s[:, 2], s[:, 1], s[:, 0], j, i))
    return np.stack([i[order], j[order]]).astype(np.int64), s[order].astype(np.int32)


def neighbor_list_bruteforce(positions, cell, pbc, r_max: float, chunk: int = 512):
    """All pairs within r_max over every relevant periodic image (float64)."""
    positions = np.asarray(positions, dtype=np.float64)
    cell = np.asarray(cell, dtype=np.float64)
    pw, wrap = _wrap(positions, cell, pbc)
    n = len(pw)
    nr = _image_range(cell, pbc, r_max)
    images = np.stack(np.meshgrid(*[np.arange(-k, k + 1) for k in nr], indexing="ij"), -1).reshape(-1, 3)
    offs = images @ cell
    I, J, S = [], [], []
    r2 = r_max * r_max
    for a in range(0, n, chunk):
        pi = pw[a:a + chunk]
        # v[i, j, s] = pw[j] - pw[i] + offs[s]
        v = pw[None, :, None, :] - pi[:, None, None, :] + offs[None, None, :, :]
        d2 = np.einsum("ijsk,ijsk->ijs", v, v)
        ii, jj, ss = np.nonzero(d2 < r2)
        ii = ii + a
        keep = ~((ii == jj) & np.all(images[ss] == 0, axis=1))
        I.append(ii[keep])
        J.append(jj[keep])
        S.append(images[ss[keep]])
    i = np.concatenate(I) if I else np.zeros(0, np.int64)
    j = np.concatenate(J) if J else np.zeros(0, np.int64)
    s = np.concatenate(S) if S else np.zeros((0, 3), np.int64)
    s = s - wrap[j] + wrap[i]
    return _canonical(i, j, s)


def _cell_list_geometry(cell: np.ndarray, pbc, r_max: float):
    """(lengths, bins) of the binned search, or None when the cell does not qualify
    (not orthorhombic, not periodic on every axis, fewer than three bins on an axis)."""
    lengths = np.diag(cell)
    ortho = np.allclose(cell, np.diag(lengths))
    nb = np.floor(lengths / r_max).astype(np.int64)
    if not ortho or not all(pbc) or (nb < 3).any():
        return None
    return lengths, nb


def neighbor_list_device(positions, cell, pbc, r_max: float, device="cuda"):
    """Cell list on the GPU: ``(edge_index (2, E) int64, shifts (E, 3) int32)`` as tensors on
    ``device``, equal to :func:`neighbor_list` element for element. ``positions`` may be a
    host array or a tensor (float64 is used). Raises ``NotImplementedError`` for cells the
    binned search does not cover (use :func:`neighbor_list`)."""
    import ctypes

    from flashcart_b200 import _native as N
    from flashcart_b200.ops import _after, _stream, status_word

    cell = np.asarray(cell, dtype=np.float64)
    geo = _cell_list_geometry(cell, pbc, r_max)
    if geo is None:
        raise NotImplementedError("neighbor_list_device needs an orthorhombic periodic cell with at least three "
                                  "bins of r_max per axis")
    lengths, nb = geo
    dev = torch.device(device)
    if dev.type != "cuda":
        raise RuntimeError("neighbor_list_device runs on CUDA devices only")
    pos = torch.as_tensor(positions, dtype=torch.float64).to(dev).contiguous()
    n = pos.shape[0]
    d = N.NlDesc()
    inv = np.linalg.inv(cell)
    width = lengths / nb
    for k in range(3):
        d.lengths[k] = float(lengths[k])
        d.inv_lengths[k] = float(inv[k, k])
        d.bin_widths[k] = float(width[k])
        d.bins[k] = int(nb[k])
    d.r_max_sq = float(r_max) * float(r_max)
    lib = N.lib()
    nbytes = lib.fc_neighbor_workspace_bytes(ctypes.byref(d), n)
    N.check(lib, int(nbytes) if nbytes < 0 else 0, "fc_neighbor_workspace_bytes")
    ws = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=dev)
    rowptr = torch.empty(n + 1, dtype=torch.int64, device=dev)
    status = ctypes.c_void_p(status_word(dev).data_ptr())
    stream = _stream(dev)
    rc = lib.fc_neighbor_count(ctypes.byref(d), ctypes.c_void_p(pos.data_ptr()), n, ctypes.c_void_p(ws.data_ptr()),
                               ctypes.c_void_p(rowptr.data_ptr()), status, stream)
    _after(lib, rc, "fc_neighbor_count", dev)
    n_edges = int(rowptr[-1].item())
    edge_index = torch.empty((2, n_edges), dtype=torch.int64, device=dev)
    shifts = torch.empty((n_edges, 3), dtype=torch.int32, device=dev)
    rc = lib.fc_neighbor_fill(ctypes.byref(d), n, ctypes.c_void_p(ws.data_ptr()), ctypes.c_void_p(rowptr.data_ptr()),
                              n_edges, ctypes.c_void_p(edge_index.data_ptr()) if n_edges else None,
                              ctypes.c_void_p(shifts.data_ptr()) if n_edges else None, status, stream)
    _after(lib, rc, "fc_neighbor_fill", dev)
    from flashcart_b200.ops import check_device_status

    check_device_status(dev)
    return edge_index, shifts


def neighbor_list(positions, cell, pbc, r_max: float, device: str = "cpu"):
    """Cell-list neighbour search (orthorhombic periodic cells), canonical order.

    Atoms are binned on the wrapped positions into >= r_max cubes; each bin is padded
    to the largest occupancy and compared with its 27 neighbouring bins in one batched
    float64 distance evaluation (torch on the host). With a CUDA ``device`` the list is
    built by the GPU kernels of :func:`neighbor_list_device` (same arithmetic, same
    order) and returned as host arrays.
    """
    positions = np.asarray(positions, dtype=np.float64)
    cell = np.asarray(cell, dtype=np.float64)
    geo = _cell_list_geometry(cell, pbc, r_max)
    if geo is None:
        return neighbor_list_bruteforce(positions, cell, pbc, r_max)
    if torch.device(device).type == "cuda":
        ei, sh = neighbor_list_device(positions, cell, pbc, r_max, device)
        return ei.cpu().numpy(), sh.cpu().numpy()
    lengths, nb = geo
    pw, wrap = _wrap(positions, cell, pbc)
    n = len(pw)
    b3 = np.minimum((pw / (lengths / nb)).astype(np.int64), nb - 1)
    bid = (b3[:, 0] * nb[1] + b3[:, 1]) * nb[2] + b3[:, 2]
    order = np.argsort(bid, kind="stable")
    counts = np.bincount(bid, minlength=int(nb.prod()))
    m = int(counts.max())
    start = np.concatenate([[0], np.cumsum(counts)[:-1]])
    slot = np.empty(n, np.int64)
    slot[order] = np.arange(n) - start[bid[order]]
    nbins = int(nb.prod())
    table = np.full((nbins, m), -1, np.int64)
    table[bid, slot] = np.arange(n)
    dev = torch.device(device)
    tab = torch.as_tensor(table, device=dev)
    pos_t = torch.as_tensor(pw, device=dev)
    L = torch.as_tensor(lengths, device=dev)
    bx = torch.arange(nbins, device=dev)
    coords = torch.stack([bx // (nb[1] * nb[2]), (bx // nb[2]) % nb[1], bx % nb[2]], -1)
    nb_t = torch.as_tensor(nb, device=dev)
    I, J, S = [], [], []
    r2 = r_max * r_max
    valid_i = tab >= 0
    pi = pos_t[tab.clamp_min(0)]  # (nbins, m, 3)
    for dx in (-1, 0, 1):
        for dy in (-1, 0, 1):
            for dz in (-1, 0, 1):
                d = torch.tensor([dx, dy, dz], device=dev)
                c = coords + d
                img = torch.div(c, nb_t, rounding_mode="floor")  # -1, 0 or +1 per axis
                c = c - img * nb_t
                other = (c[:, 0] * nb[1] + c[:, 1]) * nb[2] + c[:, 2]
                tj = tab[other]  # (nbins, m)
                pj = pos_t[tj.clamp_min(0)] + (img.to(pos_t.dtype) * L)[:, None, :]
                v = pj[:, None, :, :] - pi[:, :, None, :]
                d2 = (v * v).sum(-1)
                ok = (d2 < r2) & valid_i[:, :, None] & (tj >= 0)[:, None, :]
                bb, a, b = torch.nonzero(ok, as_tuple=True)
                ii = tab[bb, a]
                jj = tj[bb, b]
                ss = img[bb]
                keep = ~((ii == jj) & (ss == 0).all(-1))
                I.append(ii[keep].cpu().numpy())
                J.append(jj[keep].cpu().numpy())
                S.append(ss[keep].cpu().numpy())
    i = np.concatenate(I)
    j = np.concatenate(J)
    s = np.concatenate(S).astype(np.int64)
    s = s - wrap[j] + wrap[i]
    return _canonical(i, j, s)
