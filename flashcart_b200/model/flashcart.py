"""FlashCart potential and energy/force/stress prediction on the B200 operators.

``FlashCartPotential`` has the reference's constructor, submodules, state_dict keys
and ``to_model_config``/``from_config`` (reference ``model/flashcart.py:25-483``), so a
reference checkpoint (``model.pt`` + ``model_config.yaml``) loads unchanged.
``predict`` follows ``model/atomistic.py:75-340``: a symmetric virtual strain for the
stress, forces and stress from one ``torch.autograd.grad`` call, Voigt order
xx, yy, zz, yz, xz, xy and ``virials = -stress * volume``.
"""

from __future__ import annotations

import contextlib
from collections.abc import Mapping
from pathlib import Path
from typing import Callable, Any, Dict, List, Optional

import torch
import torch.nn as nn

from flashcart_b200 import o3, ops
from flashcart_b200.nn.layers import (EnergyReadoutLayer, EquivariantGatedLayer, InteractionLayer, ProductLayer,
                                      ScaleShiftEnergyLayer)
from flashcart_b200.nn.radial import ChebyshevBasis, PolynomialCutoff

MIN_EDGE_LENGTH = 1.0e-4


def rows_times_3x3(x, m):
    """``x @ m`` for rows x (R, 3) and one 3 x 3 matrix m, as a broadcast product summed
    over the inner index. Its gradient with respect to m is a reduction over the R rows;
    the GEMM form's gradient is an (3 x R) x (R x 3) product that cuBLAS runs as a
    single-tile SIMT kernel (0.2-0.35 ms at R = 1.5 M)."""
    return (x.unsqueeze(-1) * m).sum(-2)


def get_edge_vectors(positions, cell, shifts, edge_index, batch, use_shifts: bool = True):
    """v_e = r_j - r_i + S_e . cell (row 0 receivers i, row 1 senders j; reference ``utils/geometry.py:25-53``).

    Same value as the reference; the gathers use ``index_select`` (whose gradient is an
    atomic scatter-add) and a single-cell batch multiplies the shifts by the cell as one
    (E, 3) x (3, 3) product, so the position / cell gradients of forces and stress do
    not go through the sort-based backward of advanced indexing.
    """
    idx_i, idx_j = edge_index[0], edge_index[1]
    vec = positions.index_select(0, idx_j) - positions.index_select(0, idx_i)
    if not use_shifts:
        return vec
    s = shifts.to(cell.dtype)
    if cell.shape[0] == 1:
        return vec + rows_times_3x3(s, cell[0])
    per_edge_cell = cell.index_select(0, batch.index_select(0, idx_i))
    return vec + torch.bmm(s.unsqueeze(1), per_edge_cell).squeeze(1)


def to_voigt6(t: torch.Tensor) -> torch.Tensor:
    """(..., 3, 3) -> (..., 6) in xx, yy, zz, yz, xz, xy with averaged off-diagonals."""
    return torch.stack([t[..., 0, 0], t[..., 1, 1], t[..., 2, 2], (t[..., 1, 2] + t[..., 2, 1]) / 2,
                        (t[..., 0, 2] + t[..., 2, 0]) / 2, (t[..., 0, 1] + t[..., 1, 0]) / 2], dim=-1)


def _uses_shifts(pbc) -> bool:
    if pbc is None:
        return True
    if torch.is_tensor(pbc):
        return bool(torch.any(pbc).item())
    if isinstance(pbc, bool):
        return pbc
    return any(bool(v) for v in pbc)


class FlashCartPotential(nn.Module):
    """Equivariant interatomic potential (reference ``model/flashcart.py:25-317``)."""

    def __init__(self, elements: List[str], r_max: float, r_min: float = 0.0, n_hidden_feats: int = 32,
                 l_max_hidden_feats: int = 1, l_max_edge_attrs: int = 3, n_radial: int = 8,
                 n_interactions: int = 2, correlation: int = 3, path_reduced_product: bool = True,
                 element_agnostic_interaction: bool = True, element_agnostic_product: bool = True,
                 n_element_interaction_features: int = 16, nonlinearity: bool = False,
                 gate_activation: str = "silu", gate_bias: bool = True, layer_norm: bool = False,
                 hidden_radial: Optional[List[int]] = None, hidden_readout: Optional[List[int]] = None,
                 radial_mapping: str = "affine", cutoff_poly_order: int = 6, avg_neighbors: Optional[float] = None,
                 atomic_shifts: Optional[List[float]] = None, fit_atomic_shifts: bool = True,
                 recompute_radial: bool = False, use_triton: bool = False):
        super().__init__()
        self.elements = list(elements)
        self.r_min = r_min
        self.r_max = float(r_max)
        self.n_hidden_feats = n_hidden_feats
        self.l_max_hidden_feats = l_max_hidden_feats
        self.l_max_edge_attrs = l_max_edge_attrs
        self.n_radial = n_radial
        self.n_interactions = n_interactions
        self.correlation = correlation
        self.path_reduced_product = path_reduced_product
        self.hidden_radial = [64, 64] if hidden_radial is None else list(hidden_radial)
        self.hidden_readout = [64, 64] if hidden_readout is None else list(hidden_readout)
        self.radial_mapping = radial_mapping
        self.cutoff_poly_order = cutoff_poly_order
        self.atomic_shifts = None if atomic_shifts is None else list(atomic_shifts)
        self.fit_atomic_shifts = bool(fit_atomic_shifts)
        self.avg_neighbors = 1.0 if avg_neighbors is None else float(avg_neighbors)
        self.auto_avg_neighbors = avg_neighbors is None
        self.nonlinearity = nonlinearity
        self.gate_activation = gate_activation
        self.gate_bias = gate_bias
        self.layer_norm = layer_norm
        self.element_agnostic_interaction = element_agnostic_interaction
        self.element_agnostic_product = element_agnostic_product
        self.n_element_interaction_features = n_element_interaction_features
        self.recompute_radial = recompute_radial
        self.use_triton = use_triton
        self.node_dim = sum((2 * l + 1) * n_hidden_feats for l in range(l_max_hidden_feats + 1))

        self.embedding = nn.Embedding(len(elements), n_hidden_feats)
        self.radial_basis = ChebyshevBasis(n_radial, r_max=r_max, r_min=r_min, mapping=radial_mapping)
        self.cutoff_fn = PolynomialCutoff(r_max, poly_order=cutoff_poly_order)
        # constants of the fused edge-geometry kernel as host values (reading the modules'
        # device buffers would synchronise, which a captured step may not do)
        self._geometry_args = (int(n_radial), radial_mapping == "cosine", int(cutoff_poly_order), float(r_min),
                               float(r_max), float(r_max))
        self.irreps = o3.Irreps(l_max_edge_attrs, use_triton=use_triton)
        product_out = [l_max_hidden_feats if i < n_interactions - 1 else 0 for i in range(n_interactions)]
        inter_in = [0 if i == 0 else l_max_hidden_feats for i in range(n_interactions)]
        self.use_products = correlation > 1
        inter_out = [l_max_edge_attrs] * n_interactions if self.use_products else product_out
        self.interactions = nn.ModuleList([
            InteractionLayer(in1_l_max=li, in2_l_max=l_max_edge_attrs, out_l_max=lo, in1_features=n_hidden_feats,
                             out_features=n_hidden_feats, n_radial=n_radial, hidden_radial=self.hidden_radial,
                             n_elements=None if element_agnostic_interaction else len(elements),
                             element_features=n_element_interaction_features, avg_neighbors=self.avg_neighbors,
                             use_sc=True, use_layer_norm=layer_norm, use_triton=use_triton,
                             recompute_radial=recompute_radial)
            for li, lo in zip(inter_in, inter_out)])
        self.products = nn.ModuleList([
            ProductLayer(in_l_max=l_max_edge_attrs, out_l_max=po, in_features=n_hidden_feats,
                         n_elements=None if element_agnostic_product else len(elements), correlation=correlation,
                         path_reduced=path_reduced_product, use_sc=True, use_layer_norm=layer_norm,
                         use_triton=use_triton)
            for po in product_out] if self.use_products else [])
        if nonlinearity:
            self.nonlinearities = nn.ModuleList([
                EquivariantGatedLayer(l_max=lo, in_features=n_hidden_feats, hidden_features=n_hidden_feats,
                                      gate_activation=gate_activation, gate_bias=gate_bias, use_triton=use_triton)
                for lo in inter_out])
        self.readout = EnergyReadoutLayer(n_hidden_feats, n_interactions, hidden_readout=self.hidden_readout)
        self.scale_shift = ScaleShiftEnergyLayer(len(elements))

    # ------------------------------------------------------------------ forward

    def forward(self, graph: Dict[str, Any]) -> torch.Tensor:
        """Site energies of a graph dict (reference ``model/flashcart.py:223-317``).

        ``graph`` holds ``edge_index`` (2, E) with receivers in row 0 (ascending),
        ``batch``, ``atom_types`` and either ``vectors`` or ``positions``/``cell``/
        ``shifts`` (+ optional ``use_shifts``).
        """
        if not isinstance(graph, Mapping):
            raise TypeError(f"{self.__class__.__name__}.forward expects a tensor dictionary. Use predict() for Data.")
        return self._forward_impl(graph)

    def _forward_impl(self, graph: Dict[str, Any], n_out: Optional[int] = None,
                      halo_fn: Optional[Callable[[torch.Tensor], torch.Tensor]] = None) -> torch.Tensor:
        """Site energies; with ``n_out`` only the first ``n_out`` atoms are receivers (the
        atoms a domain owns, the rest are its ghosts) and ``halo_fn`` maps the owned rows of
        a layer's output to the ghost rows that the next layer reads."""
        edge_index = graph["edge_index"]
        batch = graph["batch"]
        atom_types = graph["atom_types"]
        vectors = graph.get("vectors")
        use_shifts = graph.get("use_shifts", True)
        if not isinstance(use_shifts, bool):
            use_shifts = _uses_shifts(use_shifts)
        # the next layer's senders: owned rows -> owned + ghost rows
        exchange: Optional[Callable[[torch.Tensor], torch.Tensor]] = None
        if bool(graph.get("lammps_exchange", False)):
            # LAMMPS ML-IAP layout (reference model/flashcart.py:255-301): owned atoms first,
            # then ghosts; batch covers the owned atoms, atom_types all of them, and the
            # ghost rows come from the ML-IAP forward exchange between layers
            from flashcart_b200.lammps import lammps_exchange_features

            n_out = int(batch.shape[0])
            n_total = int(atom_types.shape[0])
            exchange = lambda x: lammps_exchange_features(x, n_out, n_total)
        elif halo_fn is not None:
            exchange = lambda x: torch.cat([x, halo_fn(x)], dim=0)
        if vectors is not None and self._vectors_fusable(vectors):
            edge_attrs, edge_feats = ops.edge_geometry_vec(vectors, self.irreps.l_max, *self._geometry_args)
            envelope = None
        elif vectors is None and self._geometry_fusable(graph):
            # one kernel from positions to edge attributes and enveloped radial features
            # (same arithmetic as the chain below; first derivative only)
            edge_attrs, edge_feats = ops.edge_geometry(graph["positions"], graph["cell"], graph["shifts"], edge_index,
                                                       batch, self.irreps.l_max, *self._geometry_args,
                                                       use_shifts=use_shifts)
            envelope = None
        else:
            if vectors is None:
                vectors = get_edge_vectors(graph["positions"], graph["cell"], graph["shifts"], edge_index, batch,
                                           use_shifts=use_shifts)
            distances = vectors.norm(dim=-1)
            directions = vectors / distances.clamp_min(MIN_EDGE_LENGTH).unsqueeze(-1)
            edge_attrs = self.irreps.forward_normalized(directions)
            edge_feats = self.radial_basis(distances)
            envelope = self.cutoff_fn(distances)
        node_feats = self.embedding(atom_types)
        own_types = atom_types if n_out is None else atom_types[:n_out]
        outputs = []
        for i, interaction in enumerate(self.interactions):
            feats = interaction(node_feats, edge_attrs, edge_feats, edge_index, envelope,
                                atom_types=atom_types if not self.element_agnostic_interaction else None,
                                out_nodes=n_out)
            if self.nonlinearity:
                feats = self.nonlinearities[i](feats)
            if self.use_products:
                node_feats = self.products[i](feats, None if self.element_agnostic_product else own_types)
            else:
                node_feats = feats
            outputs.append(node_feats[:, :self.n_hidden_feats])
            if exchange is not None and i + 1 < len(self.interactions):
                node_feats = exchange(node_feats)
        energies = self.readout(outputs)
        return self.scale_shift(energies, own_types)

    def _geometry_fusable(self, graph) -> bool:
        """The fused edge-geometry kernel replaces the edge-vector -> attributes / radial
        chain when the graph is differentiated at most once (first_order_only), the data
        are on the GPU in float32 / float64, a cell tensor is given, and no interaction
        layer mixes element embeddings into its radial input (they need the envelope on
        its own)."""
        pos = graph.get("positions")
        cell = graph.get("cell")
        return (ops.first_order_only_active() and torch.is_tensor(pos) and pos.is_cuda
                and pos.dtype in (torch.float32, torch.float64) and torch.is_tensor(cell)
                and self.irreps.l_max <= 3 and all(inter.emb_i is None for inter in self.interactions))

    def _vectors_fusable(self, vectors) -> bool:
        """The vectors-given form of the fused geometry kernel (LAMMPS ``rij``) under the
        same conditions as :meth:`_geometry_fusable`."""
        return (ops.first_order_only_active() and torch.is_tensor(vectors) and vectors.is_cuda
                and vectors.dtype in (torch.float32, torch.float64) and self.irreps.l_max <= 3
                and all(inter.emb_i is None for inter in self.interactions))

    # ------------------------------------------------------------------ predict

    def predict(self, graph, compute_forces: bool = False, compute_stress: bool = False,
                create_graph: Optional[bool] = False, compute_edge_forces: bool = False) -> Dict[str, torch.Tensor]:
        """Energies and requested derivatives (reference ``model/atomistic.py:75-340``).

        Returns ``node_energies`` (N,), ``energy`` (G,), and when requested ``forces``
        (N, 3) = -dE/dR, ``stress`` (G, 6) = (dE/dD)/det(cell) in Voigt order,
        ``virials`` = -stress * volume, D being a symmetric virtual strain applied to
        positions and cell, and ``edge_forces`` (E, 3) = dE/dv of the graph's ``vectors``.
        """
        if create_graph is False and (compute_forces or compute_stress or compute_edge_forces):
            # Forces and stress need derivatives with respect to the geometry only; with the
            # parameters frozen the operators skip their weight gradients (identical results).
            frozen = [p for p in self.parameters() if p.requires_grad]
            for p in frozen:
                p.requires_grad_(False)
            try:
                return self.predict(graph, compute_forces, compute_stress, create_graph=None,
                                    compute_edge_forces=compute_edge_forces)
            finally:
                for p in frozen:
                    p.requires_grad_(True)
        create_graph = bool(create_graph)
        g = self._prepare_predict_graph(graph, compute_forces, compute_stress, compute_edge_forces)
        return self._predict_impl(g, compute_forces, compute_stress, compute_edge_forces, create_graph)

    def _prepare_predict_graph(self, graph, compute_forces: bool, compute_stress: bool,
                               compute_edge_forces: bool) -> Dict[str, Any]:
        """Graph fields for the requested derivatives (reference ``model/atomistic.py:158-240``):
        detached positions (strained for the stress, requiring grad for forces), the strain
        ``displacement``, and detached ``vectors`` requiring grad for edge forces."""
        g = dict(graph.to_dict() if hasattr(graph, "to_dict") else graph)
        g["use_shifts"] = _uses_shifts(g.get("use_shifts", g.get("pbc")))
        if compute_forces or compute_stress or torch.is_tensor(g.get("positions")):
            positions = g["positions"].detach()
            cell = g["cell"].detach() if torch.is_tensor(g.get("cell")) else None
            if compute_stress:
                if cell is None:
                    raise ValueError("Cannot compute stress without cell information.")
                displacement = torch.zeros_like(cell).requires_grad_(True)
                sym = 0.5 * (displacement + displacement.transpose(-1, -2))
                scaling = torch.eye(3, device=cell.device, dtype=cell.dtype).unsqueeze(0) + sym
                if scaling.shape[0] == 1:
                    positions = rows_times_3x3(positions, scaling[0])
                else:
                    per_atom = scaling.index_select(0, g["batch"])
                    positions = torch.bmm(positions.unsqueeze(-2), per_atom).squeeze(-2)
                cell = cell @ scaling
                g["displacement"] = displacement
            if compute_forces:
                positions.requires_grad_(True)
            g["positions"] = positions
            g["cell"] = cell
        if compute_edge_forces:
            vectors = g.get("vectors")
            if vectors is None:
                raise ValueError("Cannot compute edge forces without graph.vectors.")
            g["vectors"] = vectors.detach().requires_grad_(True)
        return g

    def _predict_impl(self, g: Dict[str, Any], compute_forces: bool, compute_stress: bool,
                      compute_edge_forces: bool, create_graph: bool) -> Dict[str, torch.Tensor]:
        """Energies and derivatives of a prepared graph (reference ``model/atomistic.py:276-340``);
        the LAMMPS interface calls it directly with differentiable ``vectors``."""
        # without create_graph the graph is differentiated once: fused first-order kernels
        # (RMS layer norm, edge geometry) may replace their composed, twice-differentiable forms
        with ops.first_order_only() if not create_graph else contextlib.nullcontext():
            node_energies = self(g)
            n_graphs = int(g["n_atoms"].shape[0]) if "n_atoms" in g else int(g["batch"].max().item()) + 1
            energy = torch.zeros(n_graphs, dtype=node_energies.dtype, device=node_energies.device)
            energy = energy.index_add(0, g["batch"], node_energies)
            out = {"node_energies": node_energies, "energy": energy}
            inputs = (([g["positions"]] if compute_forces else []) + ([g["displacement"]] if compute_stress else [])
                      + ([g["vectors"]] if compute_edge_forces else []))
            grads = (torch.autograd.grad(energy.sum(), inputs, create_graph=create_graph,
                                         allow_unused=compute_edge_forces) if inputs else None)
        if inputs:
            k = 0
            if compute_forces:
                out["forces"] = -grads[0]
                k = 1
            if compute_stress:
                volume = torch.det(g["cell"])
                stress = to_voigt6(grads[k] / volume.view(-1, 1, 1))
                out["stress"] = stress
                out["virials"] = -stress * volume.unsqueeze(-1)
                k += 1
            if compute_edge_forces:
                out["edge_forces"] = grads[k] if grads[k] is not None else torch.zeros_like(g["vectors"])
            if not create_graph:
                out["node_energies"] = out["node_energies"].detach()
                out["energy"] = out["energy"].detach()
        return out

    def predict_domain(self, graph, plan, group=None, compute_forces: bool = True,
                       compute_stress: bool = True) -> Dict[str, torch.Tensor]:
        """Energy, forces of the owned atoms and stress of one periodic cell evaluated by
        atom-domain decomposition (one rank's share; every rank of ``group`` calls this with
        its own ``plan`` from :func:`flashcart_b200.domain.build_plans`).

        Positions of the owned atoms go through the virtual strain, then to the ranks that
        hold them as ghosts (:class:`flashcart_b200.domain.HaloExchange`); the backward
        returns the ghosts' position and feature gradients to their owners, so ``forces``
        are complete for the owned atoms. ``energy`` and ``stress`` are summed over ranks.
        """
        from flashcart_b200.domain import evaluate_domain

        frozen = [p for p in self.parameters() if p.requires_grad]
        for p in frozen:
            p.requires_grad_(False)
        try:
            with ops.first_order_only():
                return evaluate_domain(self._forward_impl, graph, plan, group, compute_forces, compute_stress)
        finally:
            for p in frozen:
                p.requires_grad_(True)

    # ------------------------------------------------------------------ config

    def non_decayable_parameters(self):
        """Child-layer hooks and the element embedding (reference ``model/flashcart.py:366-382``)."""
        from flashcart_b200.nn.layers import iter_child_special_parameters

        yield from iter_child_special_parameters(self, "non_decayable_parameters")
        yield from self.embedding.parameters()

    def non_muon_parameters(self):
        from flashcart_b200.nn.layers import iter_child_special_parameters

        yield from iter_child_special_parameters(self, "non_muon_parameters")
        yield from self.embedding.parameters()

    def to_model_config(self) -> Dict[str, Any]:
        return {
            "elements": list(self.elements), "r_max": self.r_max, "r_min": self.r_min,
            "n_hidden_feats": self.n_hidden_feats, "l_max_hidden_feats": self.l_max_hidden_feats,
            "l_max_edge_attrs": self.l_max_edge_attrs, "n_radial": self.n_radial,
            "n_interactions": self.n_interactions, "correlation": self.correlation,
            "path_reduced_product": self.path_reduced_product,
            "element_agnostic_interaction": self.element_agnostic_interaction,
            "element_agnostic_product": self.element_agnostic_product,
            "n_element_interaction_features": self.n_element_interaction_features,
            "nonlinearity": self.nonlinearity, "gate_activation": self.gate_activation,
            "gate_bias": self.gate_bias, "layer_norm": self.layer_norm,
            "hidden_radial": list(self.hidden_radial), "hidden_readout": list(self.hidden_readout),
            "radial_mapping": self.radial_mapping, "cutoff_poly_order": self.cutoff_poly_order,
            "atomic_shifts": self.atomic_shifts, "fit_atomic_shifts": self.fit_atomic_shifts,
            "avg_neighbors": float(self.avg_neighbors), "use_triton": self.use_triton,
        }

    @classmethod
    def from_config(cls, cfg: Dict[str, Any]) -> "FlashCartPotential":
        defaults = dict(r_min=0.0, n_hidden_feats=32, l_max_hidden_feats=1, l_max_edge_attrs=3, n_radial=8,
                        n_interactions=2, correlation=3, path_reduced_product=True,
                        element_agnostic_interaction=True, element_agnostic_product=True,
                        n_element_interaction_features=16, nonlinearity=False, gate_activation="silu",
                        gate_bias=True, layer_norm=False, hidden_radial=[64, 64], hidden_readout=[64, 64],
                        radial_mapping="affine", cutoff_poly_order=6, atomic_shifts=None, fit_atomic_shifts=True,
                        avg_neighbors=None, use_triton=False, recompute_radial=False)
        kw = {k: cfg.get(k, v) for k, v in defaults.items()}
        return cls(elements=cfg["elements"], r_max=cfg["r_max"], **kw)

    # ------------------------------------------------------------------ checkpoints
    # Inference checkpoint directory of the reference (model/atomistic.py:15-47, 441-527):
    # ``model.pt`` (state dict), ``model_config.yaml`` (to_model_config), optional ``meta.yaml``.

    def save_weights(self, path, filename: str = "model.pt") -> None:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        torch.save(self.state_dict(), path / filename)

    def load_weights(self, path, filename: str = "model.pt", map_location="cpu") -> None:
        self.load_state_dict(torch.load(Path(path) / filename, weights_only=True, map_location=map_location))

    def save_inference_checkpoint(self, path, meta: Optional[Dict[str, Any]] = None) -> None:
        import yaml

        path = Path(path)
        self.save_weights(path)
        with open(path / "model_config.yaml", "w") as f:
            yaml.safe_dump(self.to_model_config(), f, sort_keys=False)
        if meta is not None:
            with open(path / "meta.yaml", "w") as f:
                yaml.safe_dump(meta, f, sort_keys=False)

    @classmethod
    def load_model_config(cls, ckpt_dir) -> Dict[str, Any]:
        import yaml

        cfg = Path(ckpt_dir) / "model_config.yaml"
        if not cfg.exists():
            raise FileNotFoundError(f"No model_config.yaml in {ckpt_dir}.")
        with open(cfg) as f:
            return yaml.safe_load(f)

    @classmethod
    def from_checkpoint(cls, ckpt_dir, device=None, map_location="cpu") -> "FlashCartPotential":
        model = cls.from_config(cls.load_model_config(ckpt_dir))
        model.load_weights(ckpt_dir, map_location=map_location)
        if device is not None:
            model = model.to(device)
        return model.eval()
