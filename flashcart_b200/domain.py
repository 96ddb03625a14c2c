"""Atom-domain decomposition of one periodic cell with halo exchange.

The single large cell is split into a grid of spatial domains, one per rank. A rank owns
the atoms whose fractional coordinates fall in its domain and evaluates every edge whose
receiver it owns; the senders of those edges that it does not own are its *ghosts*. The
periodic image shift stays on the edge (edge vector = r_j - r_i + S . cell), so a ghost is
simply a copy of another rank's atom, and a rank's own periodic images need no copy.

Two quantities cross ranks, both through :class:`HaloExchange` (forward: owners send the
rows their neighbours hold as ghosts; backward: the ghost gradients travel back and are
added into the owners' rows):

* positions (after the virtual strain), so that forces and the strain derivative of a
  ghost's contributions reach the rank that owns the atom;
* node features between interaction layers (the reference's LAMMPS ML-IAP forward /
  reverse exchange, ``utils/lammps.py:67-156``): layer k+1 reads its senders' layer-k
  outputs, which their owners computed.

Energies and the virial are summed over ranks at the end; every rank ends with the exact
forces of its own atoms. The plan is a pure function of the global structure, computed
identically on every rank (the structure is small next to the model's per-edge data).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Callable, List, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist


def domain_grid(world: int, cell_lengths: Sequence[float]) -> Tuple[int, int, int]:
    """Domains per axis: repeatedly halve the longest remaining domain edge (2 -> 2x1x1,
    4 -> 2x2x1, 8 -> 2x2x2 for the benchmark cell); a world size with an odd factor puts
    that factor on the longest axis."""
    grid = [1, 1, 1]
    n = world
    lengths = [float(x) for x in cell_lengths]
    f = 2
    factors = []
    while n > 1:
        while n % f == 0:
            factors.append(f)
            n //= f
        f += 1
    for f in sorted(factors, reverse=True):
        ax = max(range(3), key=lambda a: lengths[a] / grid[a])
        grid[ax] *= f
    return grid[0], grid[1], grid[2]


@dataclass
class DomainPlan:
    """What one rank evaluates and exchanges."""

    rank: int
    world: int
    grid: Tuple[int, int, int]
    owned: torch.Tensor                 # (n_own,) global atom ids, ascending
    ghosts: torch.Tensor                # (n_ghost,) global atom ids, ascending
    edge_index: torch.Tensor            # (2, E_loc) local ids: receivers in [0, n_own) ascending
    shifts: torch.Tensor                # (E_loc, 3) periodic image shifts of the local edges
    global_edges: torch.Tensor          # (E_loc,) ids of the local edges in the global list
    send_idx: List[torch.Tensor] = field(default_factory=list)   # per destination: owned-local rows
    recv_pos: List[torch.Tensor] = field(default_factory=list)   # per source: ghost rows

    @property
    def send_all(self) -> torch.Tensor:
        """Owned-local rows of every destination, concatenated in rank order (the send buffer)."""
        if getattr(self, "_send_all", None) is None or self._send_all.device != self.owned.device:
            self._send_all = torch.cat(self.send_idx) if self.send_idx else self.owned.new_zeros(0)
        return self._send_all

    @property
    def recv_all(self) -> torch.Tensor:
        """Ghost rows of every source, concatenated in rank order (the receive buffer)."""
        if getattr(self, "_recv_all", None) is None or self._recv_all.device != self.owned.device:
            self._recv_all = torch.cat(self.recv_pos) if self.recv_pos else self.owned.new_zeros(0)
        return self._recv_all

    @property
    def send_splits(self) -> List[int]:
        return [int(i.numel()) for i in self.send_idx]

    @property
    def recv_splits(self) -> List[int]:
        return [int(p.numel()) for p in self.recv_pos]

    @property
    def n_own(self) -> int:
        return int(self.owned.numel())

    @property
    def n_ghost(self) -> int:
        return int(self.ghosts.numel())

    @property
    def local_atoms(self) -> torch.Tensor:
        return torch.cat([self.owned, self.ghosts])

    def to(self, device) -> "DomainPlan":
        mv = lambda t: t.to(device)
        p = DomainPlan(self.rank, self.world, self.grid, mv(self.owned), mv(self.ghosts), mv(self.edge_index),
                       mv(self.shifts), mv(self.global_edges), [mv(t) for t in self.send_idx],
                       [mv(t) for t in self.recv_pos])
        p.send_all, p.recv_all  # concatenated index lists, built once on the device
        return p


def build_plans(positions, cell, edge_index, shifts, world: int) -> List[DomainPlan]:
    """Plans of all ranks for one periodic cell (host computation, numpy).

    ``edge_index`` (2, E): receivers (row 0, ascending) and senders; ``shifts`` (E, 3)
    integer image shifts; ``cell`` (3, 3) rows are the lattice vectors.
    """
    pos = np.asarray(torch.as_tensor(positions, dtype=torch.float64).cpu())
    cel = np.asarray(torch.as_tensor(cell, dtype=torch.float64).cpu()).reshape(3, 3)
    ei = np.asarray(torch.as_tensor(edge_index).cpu())
    sh = np.asarray(torch.as_tensor(shifts).cpu())
    n = pos.shape[0]
    grid = domain_grid(world, np.linalg.norm(cel, axis=1))
    frac = pos @ np.linalg.inv(cel)
    frac = frac - np.floor(frac)
    cidx = np.minimum((frac * np.asarray(grid)).astype(np.int64), np.asarray(grid) - 1)
    owner = cidx[:, 0] + grid[0] * (cidx[:, 1] + grid[1] * cidx[:, 2])
    recv, send = ei[0], ei[1]
    plans = []
    ghost_lists = []
    for r in range(world):
        owned = np.nonzero(owner == r)[0]
        local_of = np.full(n, -1, dtype=np.int64)
        local_of[owned] = np.arange(owned.size)
        emask = owner[recv] == r
        eids = np.nonzero(emask)[0]
        er, es = recv[eids], send[eids]
        foreign = np.unique(es[owner[es] != r])
        local_of_ghost = np.full(n, -1, dtype=np.int64)
        local_of_ghost[foreign] = owned.size + np.arange(foreign.size)
        lj = np.where(owner[es] == r, local_of[es], local_of_ghost[es])
        li = local_of[er]
        assert (li >= 0).all() and (lj >= 0).all()
        plans.append(DomainPlan(
            rank=r, world=world, grid=grid, owned=torch.as_tensor(owned), ghosts=torch.as_tensor(foreign),
            edge_index=torch.as_tensor(np.stack([li, lj])), shifts=torch.as_tensor(sh[eids]),
            global_edges=torch.as_tensor(eids)))
        ghost_lists.append(foreign)
    # exchange lists: rank s sends to rank d the atoms it owns that d holds as ghosts, in the
    # order of d's ghost list; d places source s's rows at those ghost positions
    for d in range(world):
        src = owner[ghost_lists[d]]
        plans[d].recv_pos = [torch.as_tensor(np.nonzero(src == s)[0]) for s in range(world)]
    for s in range(world):
        owned_local = np.full(n, -1, dtype=np.int64)
        owned_local[plans[s].owned.numpy()] = np.arange(plans[s].n_own)
        plans[s].send_idx = [torch.as_tensor(owned_local[ghost_lists[d][owner[ghost_lists[d]] == s]])
                             for d in range(world)]
    return plans


def _all_to_all(recv: torch.Tensor, send: torch.Tensor, out_splits, in_splits, group) -> None:
    """Uneven all-to-all; CUDA tensors are staged through host memory on a gloo group
    (the multi-process tests on one GPU), passed directly to NCCL otherwise."""
    if send.is_cuda and dist.get_backend(group) == "gloo":
        r = recv.new_empty(recv.shape, device="cpu")
        dist.all_to_all_single(r, send.cpu(), out_splits, in_splits, group=group)
        recv.copy_(r)
    else:
        dist.all_to_all_single(recv, send, out_splits, in_splits, group=group)


def _pack(x: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """Rows ``x[idx]`` as one contiguous send buffer: the device kernel (``fc_halo_pack``) for
    CUDA tensors, torch indexing for the CPU ranks of the host tests."""
    if x.is_cuda:
        from flashcart_b200 import ops

        return ops.halo_pack(x, idx)
    return x.index_select(0, idx).contiguous()


def _unpack(x: torch.Tensor, buf: torch.Tensor, idx: torch.Tensor, accumulate: bool) -> torch.Tensor:
    """``x[idx] = buf`` or ``x[idx] += buf`` in place (``fc_halo_unpack`` on the GPU)."""
    if x.is_cuda:
        from flashcart_b200 import ops

        return ops.halo_unpack_(x, buf, idx, accumulate)
    if accumulate:
        return x.index_add_(0, idx, buf)
    x[idx] = buf
    return x


def _exchange(send: torch.Tensor, recv_rows: int, out_splits, in_splits, group) -> torch.Tensor:
    recv = send.new_empty((recv_rows,) + tuple(send.shape[1:]))
    if send.is_cuda:
        from flashcart_b200 import ops

        with ops.timed_region("halo_all_to_all", 2 * send.numel() * send.element_size()):
            _all_to_all(recv, send, out_splits, in_splits, group)
    else:
        _all_to_all(recv, send, out_splits, in_splits, group)
    return recv


def ghost_rows_from_owners(x_owned: torch.Tensor, plan: DomainPlan, group=None,
                           out: torch.Tensor = None) -> torch.Tensor:
    """Forward exchange: this rank's ghost rows (``plan.ghosts`` order) from the owned rows
    of every rank; ``out`` (n_ghost, ...) contiguous is written in place when given."""
    x_owned = x_owned.contiguous()
    send = _pack(x_owned, plan.send_all)
    if plan.world == 1:
        recv = send
    else:
        recv = _exchange(send, sum(plan.recv_splits), plan.recv_splits, plan.send_splits, group)
    if out is None:
        out = x_owned.new_empty((plan.n_ghost,) + tuple(x_owned.shape[1:]))
    return _unpack(out, recv, plan.recv_all, accumulate=False)


def owners_from_ghost_rows(g_ghost: torch.Tensor, plan: DomainPlan, group=None,
                           out_owned: torch.Tensor = None) -> torch.Tensor:
    """Reverse exchange: ghost rows travel to their owners and are added into the owned
    rows (``out_owned`` (n_own, ...) contiguous, accumulated in place; zeros when None)."""
    g_ghost = g_ghost.contiguous()
    send = _pack(g_ghost, plan.recv_all)
    if plan.world == 1:
        recv = send
    else:
        recv = _exchange(send, sum(plan.send_splits), plan.send_splits, plan.recv_splits, group)
    if out_owned is None:
        out_owned = g_ghost.new_zeros((plan.n_own,) + tuple(g_ghost.shape[1:]))
    return _unpack(out_owned, recv, plan.send_all, accumulate=True)


class HaloExchange(torch.autograd.Function):
    """Owned rows -> this rank's ghost rows over a process group (all-to-all with uneven
    splits); backward sends the ghost gradients to their owners and adds them there. On
    the GPU the rows are packed and unpacked by this library's kernels
    (``fc_halo_pack`` / ``fc_halo_unpack``) and move over NCCL."""

    @staticmethod
    def forward(ctx, x_owned: torch.Tensor, plan: DomainPlan, group=None):
        ctx.plan, ctx.group = plan, group
        return ghost_rows_from_owners(x_owned, plan, group)

    @staticmethod
    def backward(ctx, g_ghost: torch.Tensor):
        return owners_from_ghost_rows(g_ghost, ctx.plan, ctx.group), None, None


def halo(plan: DomainPlan, group=None) -> Callable[[torch.Tensor], torch.Tensor]:
    """The exchange of one rank as a function ``x_owned -> x_ghost``."""
    return lambda x: HaloExchange.apply(x, plan, group)


def evaluate_domain(energy_fn, graph, plan: DomainPlan, group=None, compute_forces: bool = True,
                    compute_stress: bool = True):
    """One rank's share of a domain-decomposed energy / forces / stress evaluation.

    ``energy_fn(local_graph, n_out, halo_fn)`` returns the site energies of the ``n_out``
    owned atoms from a graph over owned + ghost atoms (receivers owned), calling
    ``halo_fn(owned_rows)`` wherever a layer needs its senders' outputs. Positions of the
    owned atoms are strained (symmetric virtual strain D, as in the serial predict) and
    sent to the ranks that hold them as ghosts; the backward returns the ghosts' gradients
    to their owners. ``energy`` and the strain derivative are summed over the group;
    ``forces`` are those of the owned atoms (``plan.owned`` order).
    """
    from flashcart_b200.model.flashcart import rows_times_3x3, to_voigt6

    g = dict(graph.to_dict() if hasattr(graph, "to_dict") else graph)
    cell = g["cell"].detach().reshape(1, 3, 3)
    pos_leaf = g["positions"].detach().index_select(0, plan.owned).requires_grad_(compute_forces)
    displacement = torch.zeros_like(cell).requires_grad_(compute_stress)
    sym = 0.5 * (displacement + displacement.transpose(-1, -2))
    scaling = torch.eye(3, device=cell.device, dtype=cell.dtype).unsqueeze(0) + sym
    pos_s = rows_times_3x3(pos_leaf, scaling[0])
    cell_s = cell @ scaling
    pos_local = torch.cat([pos_s, HaloExchange.apply(pos_s, plan, group)], dim=0)
    local = plan.local_atoms
    g_local = {"positions": pos_local, "cell": cell_s, "shifts": plan.shifts, "edge_index": plan.edge_index,
               "batch": torch.zeros(local.numel(), dtype=torch.long, device=cell.device),
               "atom_types": g["atom_types"].index_select(0, local), "use_shifts": True}
    node_energies = energy_fn(g_local, plan.n_own, halo(plan, group))
    e_local = node_energies.sum()
    inputs = ([pos_leaf] if compute_forces else []) + ([displacement] if compute_stress else [])
    grads = torch.autograd.grad(e_local, inputs) if inputs else ()
    tot = torch.cat([e_local.detach().reshape(1)] + ([grads[-1].reshape(9)] if compute_stress else []))
    if plan.world > 1:
        dist.all_reduce(tot, group=group)
    out = {"node_energies": node_energies.detach(), "energy": tot[:1]}
    if compute_forces:
        out["forces"] = -grads[0]
    if compute_stress:
        volume = torch.det(cell_s.detach())
        out["stress"] = to_voigt6(tot[1:].reshape(1, 3, 3) / volume.view(-1, 1, 1))
    return out
