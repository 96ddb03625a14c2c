"""LAMMPS ML-IAP interface of the potential, with ghost exchanges on the device halo kernels.

Counterpart of the reference's ``calculators/lammps_mliap.py`` and ``utils/lammps.py``:

* :func:`lammps_data_slot` and the custom operators ``flashcart::lammps_forward_exchange`` /
  ``flashcart::lammps_reverse_exchange`` (each the other's backward), through which the
  model refreshes ghost-atom features between interaction layers
  (``utils/lammps.py:17-194``);
* :func:`graph_from_mliap` / :func:`graph_dict_from_mliap`: the ML-IAP arrays (``pair_i``,
  ``pair_j``, ``rij``, ``elems``) as a graph over owned + ghost atoms whose edge vectors are
  LAMMPS's ``rij`` (``calculators/lammps_mliap.py:32-232``);
* :class:`FlashCartLAMMPSUnified`: ``compute_forces`` evaluates the owned atoms' site
  energies and the pair forces dE/d(rij) and hands them to ``data.update_pair_forces``
  (or accumulates them into ``data.f``) (``calculators/lammps_mliap.py:482-745``).

On the B200 the edge vectors go through the vectors-given form of the fused geometry
kernel (``fc_edge_geometry_vec_fwd/bwd``: its backward writes the pair forces directly),
and the exchange hooks that LAMMPS's KOKKOS build provides can be replaced by this
library's device halo kernels (``fc_halo_pack`` / ``fc_halo_unpack``):

* :class:`GhostImageExchange`: ghosts that are images of this rank's own atoms (one
  process, periodic cell) -- one gather kernel forward, one scatter-add kernel reverse;
* :class:`DomainGhostExchange` / :class:`DomainMLIAPData`: an atom-domain decomposition
  over a ``torch.distributed`` group (:mod:`flashcart_b200.domain`), the rows packed and
  unpacked on the device and moved by NCCL all-to-all.
"""

from __future__ import annotations

import logging
import os
import sys
from contextlib import contextmanager
from pathlib import Path
from typing import Any, Callable, Dict, Iterator, List, NoReturn, Optional, Union

import numpy as np
import torch

COMPILE_MODES = ("default", "max-autotune-no-cudagraphs")

# chemical symbols -> atomic numbers, Z = 1..118 (the element table of ``ase.data``)
_SYMBOLS = (
    "X H He Li Be B C N O F Ne Na Mg Al Si P S Cl Ar K Ca Sc Ti V Cr Mn Fe Co Ni Cu Zn Ga Ge As Se Br Kr "
    "Rb Sr Y Zr Nb Mo Tc Ru Rh Pd Ag Cd In Sn Sb Te I Xe Cs Ba La Ce Pr Nd Pm Sm Eu Gd Tb Dy Ho Er Tm Yb "
    "Lu Hf Ta W Re Os Ir Pt Au Hg Tl Pb Bi Po At Rn Fr Ra Ac Th Pa U Np Pu Am Cm Bk Cf Es Fm Md No Lr Rf "
    "Db Sg Bh Hs Mt Ds Rg Cn Nh Fl Mc Lv Ts Og").split()
ATOMIC_NUMBERS = {s: z for z, s in enumerate(_SYMBOLS)}


def _env_bool(name: str) -> bool:
    return os.environ.get(name, "").strip().lower() in ("1", "true", "yes", "on")


def _env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


# --------------------------------------------------------------------------- exchange operators

_LAMMPS_DATA: Optional[Any] = None


@contextmanager
def lammps_data_slot(lammps_data: Any) -> Iterator[None]:
    """Expose an ML-IAP data object (``forward_exchange`` / ``reverse_exchange``) to the
    exchange operators for the duration of an evaluation and its differentiation; the
    previous object is restored on exit (reference ``utils/lammps.py:17-35``)."""
    global _LAMMPS_DATA
    previous = _LAMMPS_DATA
    _LAMMPS_DATA = lammps_data
    try:
        yield
    finally:
        _LAMMPS_DATA = previous


def _require_lammps_data() -> Any:
    data = _LAMMPS_DATA
    if data is None or not hasattr(data, "forward_exchange") or not hasattr(data, "reverse_exchange"):
        raise RuntimeError(
            "LAMMPS ghost exchange requires an ML-IAP data object with forward_exchange/reverse_exchange. "
            "Evaluate the model inside flashcart_b200.lammps.lammps_data_slot(data).")
    return data


def _sync_stream(t: torch.Tensor) -> None:
    """Device synchronisation around a hook when torch runs on a non-default stream (the
    hook's own work, e.g. Kokkos, is ordered against the legacy default stream only;
    reference ``utils/lammps.py:47-64``)."""
    if t.is_cuda and torch.cuda.current_stream(t.device) != torch.cuda.default_stream(t.device):
        torch.cuda.synchronize(t.device)


@torch.library.custom_op("flashcart::lammps_forward_exchange", mutates_args=())
def lammps_forward_exchange(feats: torch.Tensor) -> torch.Tensor:
    """(ntotal, C) features, owned rows first -> a new tensor whose ghost rows hold their
    owners' features (reference ``utils/lammps.py:67-94``)."""
    data = _require_lammps_data()
    feats = feats.contiguous()
    out = torch.empty_like(feats)
    _sync_stream(feats)
    data.forward_exchange(feats, out, feats.shape[-1])
    _sync_stream(feats)
    return out


@torch.library.custom_op("flashcart::lammps_reverse_exchange", mutates_args=())
def lammps_reverse_exchange(grads: torch.Tensor) -> torch.Tensor:
    """(ntotal, C) gradients -> a new tensor with the ghost rows added into their owners'
    rows and the ghost rows zero (reference ``utils/lammps.py:96-118``)."""
    data = _require_lammps_data()
    grads = grads.contiguous()
    out = torch.empty_like(grads)
    _sync_stream(grads)
    data.reverse_exchange(grads, out, grads.shape[-1])
    _sync_stream(grads)
    return out


@lammps_forward_exchange.register_fake
def _(feats):
    return feats.new_empty(feats.shape)


@lammps_reverse_exchange.register_fake
def _(grads):
    return grads.new_empty(grads.shape)


def _forward_exchange_backward(ctx, grad_out):
    return torch.ops.flashcart.lammps_reverse_exchange(grad_out)


def _reverse_exchange_backward(ctx, grad_out):
    return torch.ops.flashcart.lammps_forward_exchange(grad_out)


lammps_forward_exchange.register_autograd(_forward_exchange_backward)
lammps_reverse_exchange.register_autograd(_reverse_exchange_backward)


def lammps_exchange_features(feats: torch.Tensor, nlocal: int, ntotal: int) -> torch.Tensor:
    """Owned features (nlocal, C) -- or (ntotal, C) -- -> (ntotal, C) with the ghost rows
    filled by the forward exchange; every rank takes part, ghosts or not (reference
    ``utils/lammps.py:159-194``)."""
    if feats.shape[0] == nlocal and ntotal > nlocal:
        feats = torch.cat([feats, feats.new_zeros((ntotal - nlocal,) + tuple(feats.shape[1:]))], dim=0)
    elif feats.shape[0] != ntotal:
        raise RuntimeError(f"LAMMPS feature exchange expected {nlocal} or {ntotal} rows, got {feats.shape[0]}.")
    return torch.ops.flashcart.lammps_forward_exchange(feats)


# --------------------------------------------------------------------------- device exchange hooks


def _gather_into(x: torch.Tensor, idx: torch.Tensor, out: torch.Tensor) -> None:
    """out[k] = x[idx[k]] in place: ``fc_halo_pack`` on the GPU; torch indexing for the CPU
    tensors of the host tests of the exchange plumbing."""
    if x.is_cuda:
        from flashcart_b200 import ops

        ops.halo_pack(x, idx, out=out)
    else:
        torch.index_select(x, 0, idx, out=out)


def _scatter_add_into(x: torch.Tensor, buf: torch.Tensor, idx: torch.Tensor) -> None:
    """x[idx[k]] += buf[k] in place (``fc_halo_unpack`` with accumulation on the GPU)."""
    if x.is_cuda:
        from flashcart_b200 import ops

        ops.halo_unpack_(x, buf, idx, accumulate=True)
    else:
        x.index_add_(0, idx, buf)


class _IdentityExchange:
    """Hooks for a layout without ghosts when the data object has none (reference
    ``calculators/lammps_mliap.py:419-451``)."""

    def forward_exchange(self, feats, out, vec_len: int) -> None:
        out.copy_(feats)

    def reverse_exchange(self, grads, out, vec_len: int) -> None:
        out.copy_(grads)


class GhostImageExchange:
    """ML-IAP exchange hooks for ghosts that are copies of this process's own atoms (a
    single rank with a periodic cell: LAMMPS's ghosts are then the owned atoms' periodic
    images). ``owner[k]`` is the owned row of ghost row ``nlocal + k``. Forward: owned rows
    copied, ghost rows gathered from their owners (one ``fc_halo_pack`` launch into the
    output's ghost rows). Reverse: owned rows copied, each ghost row added into its owner
    (``fc_halo_unpack`` with atomics: an atom may have several images), ghost rows zeroed.
    The same semantics as LAMMPS's forward / reverse communication."""

    def __init__(self, owner: torch.Tensor, nlocal: int):
        self.owner = torch.as_tensor(owner, dtype=torch.long)
        self.nlocal = int(nlocal)
        if self.owner.numel() and (int(self.owner.min()) < 0 or int(self.owner.max()) >= self.nlocal):
            raise ValueError(f"GhostImageExchange: owners must lie in [0, {self.nlocal})")
        self.forward_exchange_calls = 0
        self.reverse_exchange_calls = 0

    def _idx(self, t: torch.Tensor) -> torch.Tensor:
        if self.owner.device != t.device:
            self.owner = self.owner.to(t.device)
        return self.owner

    def forward_exchange(self, feats: torch.Tensor, out: torch.Tensor, vec_len: int) -> None:
        self.forward_exchange_calls += 1
        n = self.nlocal
        out[:n].copy_(feats[:n])
        if out.shape[0] > n:
            _gather_into(feats[:n], self._idx(feats), out[n:])

    def reverse_exchange(self, grads: torch.Tensor, out: torch.Tensor, vec_len: int) -> None:
        self.reverse_exchange_calls += 1
        n = self.nlocal
        out[:n].copy_(grads[:n])
        if out.shape[0] > n:
            _scatter_add_into(out[:n], grads[n:], self._idx(grads))
            out[n:].zero_()


class DomainGhostExchange:
    """ML-IAP exchange hooks of one rank of an atom-domain decomposition
    (:func:`flashcart_b200.domain.build_plans`): rows ``[0, n_own)`` are the rank's atoms,
    rows ``[n_own, n_own + n_ghost)`` its ghosts in ``plan.ghosts`` order. Forward: the
    owners' rows are packed on the device, sent by all-to-all over ``group`` (NCCL) and
    unpacked into the ghost rows; reverse: the ghost rows travel back and are added into
    their owners'. Every rank of the group must call each hook the same number of times."""

    def __init__(self, plan, group=None):
        self.plan = plan
        self.group = group
        self.forward_exchange_calls = 0
        self.reverse_exchange_calls = 0

    def _plan_on(self, t: torch.Tensor):
        if self.plan.owned.device != t.device:
            self.plan = self.plan.to(t.device)
        return self.plan

    def forward_exchange(self, feats: torch.Tensor, out: torch.Tensor, vec_len: int) -> None:
        from flashcart_b200.domain import ghost_rows_from_owners

        self.forward_exchange_calls += 1
        plan = self._plan_on(feats)
        n = plan.n_own
        out[:n].copy_(feats[:n])
        ghost_rows_from_owners(feats[:n], plan, self.group, out=out[n:])

    def reverse_exchange(self, grads: torch.Tensor, out: torch.Tensor, vec_len: int) -> None:
        from flashcart_b200.domain import owners_from_ghost_rows

        self.reverse_exchange_calls += 1
        plan = self._plan_on(grads)
        n = plan.n_own
        out[:n].copy_(grads[:n])
        owners_from_ghost_rows(grads[n:], plan, self.group, out_owned=out[:n])
        out[n:].zero_()


class DomainMLIAPData(DomainGhostExchange):
    """An ML-IAP data object for one rank of an atom-domain decomposition of a periodic
    cell, for engines other than LAMMPS (and the tests): owned atoms then ghosts, the
    rank's edges (receivers owned) with ``rij = r_j - r_i + S . cell``, element indices
    ``elems``, the exchange hooks of :class:`DomainGhostExchange`, and ``f`` / ``eatoms``
    buffers that :meth:`FlashCartLAMMPSUnified.compute_forces` fills. ``f`` holds the
    forces of owned and ghost rows (ghost rows: contributions to be returned to their
    owners, as LAMMPS's reverse communication does; :meth:`owned_forces` does it here)."""

    def __init__(self, plan, positions, cell, atom_types, group=None, dtype=torch.float64):
        device = positions.device
        plan = plan.to(device)
        super().__init__(plan, group)
        local = plan.local_atoms
        pos = positions.to(dtype).index_select(0, local)
        ei = plan.edge_index
        c = torch.as_tensor(cell, dtype=dtype, device=device).reshape(3, 3)
        rij = pos.index_select(0, ei[1]) - pos.index_select(0, ei[0]) + plan.shifts.to(dtype) @ c
        self.nlocal = plan.n_own
        self.ntotal = plan.n_own + plan.n_ghost
        self.nghosts = plan.n_ghost
        self.npairs = int(ei.shape[1])
        self.pair_i = ei[0].to(torch.int32)
        self.pair_j = ei[1].to(torch.int32)
        self.rij = rij
        self.elems = atom_types.index_select(0, local).to(torch.int32)
        self.f = torch.zeros(self.ntotal, 3, dtype=torch.float64, device=device)
        self.eatoms = torch.zeros(self.nlocal, dtype=torch.float64, device=device)
        self.energy = 0.0
        self.eflag = True

    def owned_forces(self) -> torch.Tensor:
        """Forces of the owned atoms with the ghost rows' contributions returned to their
        owners (reverse communication of ``f``)."""
        from flashcart_b200.domain import owners_from_ghost_rows

        out = self.f[:self.nlocal].contiguous().clone()
        return owners_from_ghost_rows(self.f[self.nlocal:], self.plan, self.group, out_owned=out)


# --------------------------------------------------------------------------- graphs from ML-IAP arrays


def _mliap_array(data, name: str):
    try:
        return getattr(data, name)
    except NameError as exc:  # KOKKOS ML-IAP exposes CUDA arrays through CuPy
        if "cupy" in str(exc):
            raise RuntimeError("LAMMPS Kokkos ML-IAP provided CUDA arrays, but CuPy is not available.") from exc
        raise


def _array_device(values, requested) -> torch.device:
    """CUDA arrays (``__cuda_array_interface__``) keep a requested CUDA device or take the
    current one; host arrays go to the requested device, CPU by default (reference
    ``calculators/lammps_mliap.py:256-285``)."""
    if any(hasattr(v, "__cuda_array_interface__") or (torch.is_tensor(v) and v.is_cuda) for v in values):
        requested = None if requested is None else torch.device(requested)
        if requested is not None and requested.type == "cuda":
            return requested
        if not torch.cuda.is_available() or _env_bool("FLASHCART_LAMMPS_CPU"):
            raise RuntimeError("LAMMPS provides CUDA ML-IAP arrays, but FlashCart is configured for CPU.")
        return torch.device("cuda")
    return torch.device("cpu") if requested is None else torch.device(requested)


def _validate_lammps_indices(name: str, idx: torch.Tensor, size: int) -> None:
    lo, hi = (0, -1) if idx.numel() == 0 else (int(idx.min()), int(idx.max()))
    if lo < 0 or hi >= size:
        raise ValueError(f"LAMMPS {name} contains indices in [{lo}, {hi}], expected [0, {size}).")


def _mliap_core_tensors(data, element_types: List[str], device, dtype, validate: bool):
    """(ntotal, nlocal, nghost, npairs, device, dtype, pair_i, pair_j, vectors, atom_types)
    restricted to the reported counts (reference ``calculators/lammps_mliap.py:176-232``)."""
    ntotal = int(data.ntotal)
    nlocal = int(data.nlocal)
    nghost = int(getattr(data, "nghosts", getattr(data, "nghost", ntotal - nlocal)))
    npairs = int(data.npairs)
    if npairs <= 0 or ntotal <= 0:
        raise ValueError(f"Empty ML-IAP layout: ntotal={ntotal}, npairs={npairs}.")
    dtype = torch.get_default_dtype() if dtype is None else dtype
    arrays = [_mliap_array(data, k) for k in ("pair_i", "pair_j", "rij", "elems")]
    device = _array_device(arrays, device)
    pair_i = torch.as_tensor(arrays[0], device=device).to(torch.long)[:npairs]
    pair_j = torch.as_tensor(arrays[1], device=device).to(torch.long)[:npairs]
    vectors = torch.as_tensor(arrays[2], device=device).to(dtype)[:npairs]
    elems = torch.as_tensor(arrays[3], device=device).to(torch.long)[:ntotal]
    if validate:
        _validate_lammps_indices("pair_i", pair_i, ntotal)
        _validate_lammps_indices("pair_j", pair_j, ntotal)
    if vectors.ndim != 2 or vectors.shape[-1] != 3:
        raise ValueError(f"LAMMPS rij must have shape (npairs, 3), got {tuple(vectors.shape)}.")
    if validate:
        _validate_lammps_indices("atom_types", elems, len(element_types))
    if validate or _env_bool("FLASHCART_LAMMPS_DEBUG"):
        if _env_bool("FLASHCART_LAMMPS_DEBUG"):
            logging.info("FlashCart LAMMPS graph: ntotal=%d nlocal=%d nghost=%d npairs=%d device=%s",
                         ntotal, nlocal, nghost, npairs, device)
    return ntotal, nlocal, nghost, npairs, device, dtype, pair_i, pair_j, vectors, elems


def _z_table(element_types: List[str], device) -> torch.Tensor:
    return torch.tensor([ATOMIC_NUMBERS[s] for s in element_types], dtype=torch.long, device=device)


def graph_from_mliap(data, element_types: List[str], r_max: float, device=None, dtype=None, cell=None, pbc=None,
                     validate: bool = False) -> Dict[str, Any]:
    """Graph over owned + ghost atoms with LAMMPS's edge vectors (``use_shifts=False``);
    ``batch`` and ``n_atoms`` cover the ``nlocal`` owned atoms only, so site energies are
    summed over owned atoms (reference ``calculators/lammps_mliap.py:32-119``). Returned
    as a dict with the reference ``Data``'s fields."""
    ntotal, nlocal, nghost, npairs, device, dtype, pair_i, pair_j, vectors, atom_types = _mliap_core_tensors(
        data, element_types, device, dtype, validate)
    cell_t = (torch.eye(3, dtype=dtype, device=device).unsqueeze(0) * 1.0e3 if cell is None
              else torch.as_tensor(cell, dtype=dtype, device=device).reshape(1, 3, 3))
    if pbc is None:
        pbc_t = torch.zeros(1, 3, dtype=torch.bool, device=device)
    else:
        pbc_t = torch.as_tensor(pbc, dtype=torch.bool, device=device)
        pbc_t = (pbc_t.expand(3) if pbc_t.ndim == 0 else pbc_t).reshape(1, 3)
    return {
        "num_nodes": ntotal, "n_atoms": torch.tensor([nlocal], dtype=torch.long, device=device),
        "atomic_numbers": _z_table(element_types, device)[atom_types],
        "positions": torch.zeros(ntotal, 3, dtype=dtype, device=device), "cell": cell_t, "pbc": pbc_t,
        "edge_index": torch.stack([pair_i, pair_j], dim=0),
        "shifts": torch.zeros(npairs, 3, dtype=torch.long, device=device), "atom_types": atom_types,
        "vectors": vectors, "batch": torch.zeros(nlocal, dtype=torch.long, device=device), "use_shifts": False,
        "lammps_exchange": True, "nlocal": nlocal, "ntotal": ntotal, "nghost": nghost, "r_max": float(r_max),
    }


def graph_dict_from_mliap(data, element_types: List[str], device=None, dtype=None,
                          validate: bool = False) -> Dict[str, Any]:
    """The tensors of :func:`graph_from_mliap` that energy and edge-force evaluation reads
    (no positions, cell or shifts; reference ``calculators/lammps_mliap.py:122-173``)."""
    _, nlocal, _, _, device, _, pair_i, pair_j, vectors, atom_types = _mliap_core_tensors(
        data, element_types, device, dtype, validate)
    return {
        "n_atoms": torch.tensor([nlocal], dtype=torch.long, device=device),
        "edge_index": torch.stack([pair_i, pair_j], dim=0),
        "atomic_numbers": _z_table(element_types, device)[atom_types], "atom_types": atom_types,
        "vectors": vectors, "batch": torch.zeros(nlocal, dtype=torch.long, device=device), "use_shifts": False,
        "lammps_exchange": True,
    }


def _exchange_object(data, nlocal: int, ntotal: int):
    """The data object when it has both exchange hooks; identity hooks without ghosts;
    otherwise an error (reference ``calculators/lammps_mliap.py:454-479``)."""
    if hasattr(data, "forward_exchange") and hasattr(data, "reverse_exchange"):
        return data
    if ntotal == nlocal:
        return _IdentityExchange()
    raise RuntimeError(
        "Ghost atoms require the ML-IAP communication hooks, which only the KOKKOS ML-IAP build provides "
        "(or pass hooks built on this library's halo kernels: GhostImageExchange / DomainGhostExchange). "
        "Build LAMMPS with PKG_KOKKOS and run with `-k on ... -sf kk`, or use a model with one interaction layer.")


def _has_mliap_attr(data, name: str) -> bool:
    return hasattr(type(data), name) or name in getattr(data, "__dict__", {})


# --------------------------------------------------------------------------- the ML-IAP unified class

try:  # LAMMPS's abstract base when LAMMPS's Python module is installed
    from lammps.mliap.mliap_unified_abc import MLIAPUnified
except ImportError:
    class MLIAPUnified:  # type: ignore[no-redef]
        def __init__(self, *args, **kwargs):
            pass


class FlashCartLAMMPSUnified(MLIAPUnified):
    """The potential behind LAMMPS's ``pair_style mliap unified`` (reference
    ``calculators/lammps_mliap.py:482-745``).

    ``compute_forces(data)`` builds the ML-IAP graph (owned atoms first, then ghosts, edge
    vectors ``rij``), evaluates the owned atoms' site energies with the model's CUDA
    operators and differentiates the energy with respect to the edge vectors: those pair
    forces go to ``data.update_pair_forces`` when LAMMPS offers it, else are accumulated
    into ``data.f`` (+f on the receiver, -f on the sender). With several interaction layers
    the ghost features are refreshed between layers by the data object's exchange hooks
    (KOKKOS ML-IAP, or :class:`GhostImageExchange` / :class:`DomainGhostExchange` on the
    device halo kernels), in reverse during the differentiation.

    ``compile_mode`` is accepted and validated for interface compatibility; evaluation runs
    this library's kernels eagerly either way (there is no tracing compiler on the path).
    """

    def __init__(self, model, add_atomic_offsets: bool = False, compile_mode: Optional[str] = None,
                 compile_fullgraph: bool = True):
        super().__init__()
        if compile_mode is not None and compile_mode not in COMPILE_MODES:
            raise ValueError(f"compile_mode must be one of {COMPILE_MODES} or None, got {compile_mode!r}.")
        self.model = model
        self.element_types = list(model.elements)
        self.r_max = float(model.r_max)
        self.rcutfac = 0.5 * self.r_max
        self.ndescriptors = 1
        self.nparams = 1
        self.dtype = next(model.parameters()).dtype
        self.add_atomic_offsets = bool(add_atomic_offsets)
        self.compile_mode = compile_mode
        self.compile_fullgraph = bool(compile_fullgraph)
        self._atomic_shifts = model.scale_shift.shifts.detach().to(torch.float64)
        self.device = torch.device("cpu")
        self.model = self.model.to(self.device).eval()
        self._initialized = False
        self._checked_lammps_graph = False
        self._step = 0
        self._freeze_model_parameters()

    def compute_descriptors(self, data) -> None:
        """ML-IAP descriptor hook: nothing to do (compute_forces evaluates the model)."""

    def compute_gradients(self, data) -> None:
        """ML-IAP gradient hook: nothing to do (compute_forces evaluates the forces)."""

    def _freeze_model_parameters(self) -> None:
        for p in self.model.parameters():
            p.requires_grad_(False)

    def _predict_fn(self) -> Callable[[Dict[str, Any]], Dict[str, torch.Tensor]]:
        return lambda graph: self.model._predict_impl(graph, compute_forces=False, compute_stress=False,
                                                      compute_edge_forces=True, create_graph=False)

    def _fail(self, message: str) -> NoReturn:
        """Exit an attached LAMMPS process (an exception inside the callback would leave the
        other ranks waiting in the next exchange); raise when standalone (reference
        ``calculators/lammps_mliap.py:614-633``)."""
        if getattr(self, "interface", None) is not None:
            try:
                print(f"FlashCart LAMMPS: {message}", file=sys.stderr, flush=True)
            finally:
                os._exit(1)
        raise RuntimeError(message)

    def compute_forces(self, data) -> None:
        """Energies and pair forces of one ML-IAP call (reference
        ``calculators/lammps_mliap.py:635-745``); every rank must own atoms with pairs."""
        nlocal = int(data.nlocal)
        ntotal = int(data.ntotal)
        npairs = int(data.npairs)
        if nlocal == 0 or npairs <= 0:
            self._fail(
                f"This rank owns {nlocal} atoms with {npairs} neighbor pairs. Every rank must own atoms with "
                "neighbor pairs. For empty regions, try the LAMMPS `balance` command or fewer ranks. "
                "Configurations with no neighbor pairs remain unsupported on one rank.")
        self._step += 1
        validate = (not self._checked_lammps_graph or _env_bool("FLASHCART_LAMMPS_VALIDATE")
                    or _env_bool("FLASHCART_LAMMPS_DEBUG"))
        graph = graph_dict_from_mliap(data, self.element_types, device=self.device, dtype=self.dtype,
                                      validate=validate)
        self._checked_lammps_graph = True
        graph_device = graph["vectors"].device
        if graph_device != self.device:
            self.device = graph_device
            self.model = self.model.to(self.device)
        if not self._initialized:
            self._freeze_model_parameters()
            self._initialized = True
            logging.info("FlashCart LAMMPS: model on %s, r_max=%.4f", self.device, self.r_max)

        # the convolution kernels take receiver-sorted edges (LAMMPS lists pairs atom by
        # atom, so this is normally a no-op check); the pair forces return in ML-IAP order
        edge_index = graph["edge_index"]
        perm = None
        if npairs > 1 and not bool((edge_index[0, 1:] >= edge_index[0, :-1]).all()):
            perm = torch.argsort(edge_index[0], stable=True)
            graph["edge_index"] = edge_index.index_select(1, perm)
            graph["vectors"] = graph["vectors"].index_select(0, perm)
        graph["vectors"] = graph["vectors"].detach().requires_grad_(True)
        exchange_data = data
        if self.model.n_interactions > 1:
            try:
                exchange_data = _exchange_object(data, nlocal, ntotal)
            except RuntimeError as exc:
                self._fail(str(exc))
        with lammps_data_slot(exchange_data):
            out = self._predict_fn()(graph)

        pair_forces = out["edge_forces"].detach().to(torch.float64)
        if perm is not None:
            pair_forces = torch.empty_like(pair_forces).index_copy_(0, perm, pair_forces)
        if bool(getattr(data, "eflag", True)):
            e_local = out["node_energies"].detach().to(torch.float64)[:nlocal]
            if self.add_atomic_offsets:
                e_local = e_local + self._atomic_shifts.to(e_local.device)[graph["atom_types"][:nlocal]]
            if _has_mliap_attr(data, "eatoms"):
                try:
                    buf = _mliap_array(data, "eatoms")
                except AttributeError:
                    data.eatoms = e_local.cpu().numpy()
                else:
                    if buf is not None:
                        t = torch.as_tensor(buf)
                        t[:nlocal].copy_(e_local.to(dtype=t.dtype, device=t.device))
            data.energy = float(e_local.sum().cpu())

        if hasattr(data, "update_pair_forces"):
            data.update_pair_forces(pair_forces if pair_forces.is_cuda else pair_forces.numpy())
            self._maybe_empty_cache()
            return
        f_view = data.f
        if f_view is None:
            raise RuntimeError("ML-IAP data.f is NULL: Cannot write forces.")
        pair_i, pair_j = edge_index[0], edge_index[1]
        forces = torch.zeros(ntotal, 3, dtype=pair_forces.dtype, device=pair_forces.device)
        forces.index_add_(0, pair_i, pair_forces)
        forces.index_add_(0, pair_j, -pair_forces)
        if torch.is_tensor(f_view):
            f_view[:ntotal].copy_(forces.to(dtype=f_view.dtype, device=f_view.device))
        else:
            np.asarray(f_view)[:ntotal, :] = forces.cpu().numpy()
        self._maybe_empty_cache()

    def _maybe_empty_cache(self) -> None:
        """Release cached CUDA blocks every FLASHCART_LAMMPS_EMPTY_CACHE_EVERY calls when
        FLASHCART_LAMMPS_EMPTY_CACHE is set (pair counts change during MD)."""
        if not _env_bool("FLASHCART_LAMMPS_EMPTY_CACHE") or self.device.type != "cuda":
            return
        if self._step % max(_env_int("FLASHCART_LAMMPS_EMPTY_CACHE_EVERY", 1), 1) == 0:
            torch.cuda.empty_cache()


def build_lammps_unified(checkpoint: Union[str, Path], compile_mode: Optional[str] = None) -> FlashCartLAMMPSUnified:
    """Load an inference checkpoint on the CPU and wrap it for LAMMPS (reference
    ``calculators/lammps_mliap.py:761-779``)."""
    from flashcart_b200.model.flashcart import FlashCartPotential

    model = FlashCartPotential.from_checkpoint(checkpoint, device=torch.device("cpu"), map_location="cpu")
    return FlashCartLAMMPSUnified(model, compile_mode=compile_mode)


def save_lammps_unified(unified: FlashCartLAMMPSUnified, path: Union[str, Path]) -> Path:
    """``torch.save`` of the interface and its model for ``pair_style mliap unified``
    (reference ``calculators/lammps_mliap.py:782-803``)."""
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    torch.save(unified, path)
    return path
