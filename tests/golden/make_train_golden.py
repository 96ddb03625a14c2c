"""Generate golden vectors of one data-parallel training step from the REFERENCE model.

Run where the reference source tree is available (never needed at test time)::

    PYTHONPATH=<reference>/src python tests/golden/make_train_golden.py [<reference>/src]

Config-4 setting at a test size: 4 seeded random-walk molecules
(``flashcart_b200.training.synthetic_molecules``, rank 0, step 0), elements H/C/N/O, the
config-0 architecture (64 channels, ranks <= 2, 2 layers, correlation 3); labels from a
teacher (``torch.manual_seed(1)``), student ``torch.manual_seed(0)``, both the reference's
``FlashCartPotential`` (PyTorch path) in float64 (built under the float32 default, as the
reference's float64 runs do). Records the teacher's energies / forces, the student's loss
(energy MSE per atom + force MSE, forces with ``create_graph=True``) and every parameter
gradient (as sum, sum of squares and first 64 entries), the reference optimizer routing (``make_optimizer(optimizer="muon")``: which
parameters go to Muon, which skip weight decay) and the parameters after one step of the
reference optimizers (lr 1e-2, weight decay 1e-3).

Output: ``tests/golden/train_golden.pt``.
"""

from __future__ import annotations

import os
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))


def _shims():
    """Import-time dependencies of the reference package that these calls do not use."""
    if "lightning" not in sys.modules:
        lightning = types.ModuleType("lightning")
        fabric = types.ModuleType("lightning.fabric")

        class Fabric:  # type hint only
            pass

        fabric.Fabric = Fabric
        lightning.fabric = fabric
        sys.modules["lightning"] = lightning
        sys.modules["lightning.fabric"] = fabric
    if "torch_ema" not in sys.modules:
        ema = types.ModuleType("torch_ema")

        class ExponentialMovingAverage:  # referenced by the training task module only
            pass

        ema.ExponentialMovingAverage = ExponentialMovingAverage
        sys.modules["torch_ema"] = ema


def _digest(t: torch.Tensor) -> dict:
    """Sum, sum of squares and the first 64 entries (float64) of a tensor."""
    t = t.detach().double().flatten()
    return {"sum": t.sum(), "sq": (t * t).sum(), "head": t[:64].clone(), "numel": t.numel()}


class _Graph:
    def __init__(self, d):
        self._d = d

    def to_dict(self):
        return dict(self._d)


def model_kwargs(avg: float) -> dict:
    return dict(elements=["H", "C", "N", "O"], r_max=5.0, n_hidden_feats=64, l_max_hidden_feats=2,
                l_max_edge_attrs=2, n_radial=8, n_interactions=2, correlation=3, layer_norm=True, nonlinearity=True,
                gate_activation="sigmoid", radial_mapping="cosine", path_reduced_product=False,
                fit_atomic_shifts=False, atomic_shifts=[0.0, 0.0, 0.0, 0.0], avg_neighbors=float(avg))


def main(ref_src: str) -> None:
    sys.path.insert(0, ROOT)
    sys.path.insert(1, ref_src)
    _shims()
    from flashcart.model.flashcart import FlashCartPotential as RefPotential
    from flashcart.training.optimizers import make_optimizer

    from flashcart_b200.training import batch_graph, synthetic_molecules

    mols = synthetic_molecules(4, rank=0, step=0)
    g = batch_graph(mols, 5.0, "cpu", dtype=torch.float64)
    avg = g["edge_index"].shape[1] / g["positions"].shape[0]
    graph = {k: v for k, v in g.items() if k != "use_shifts"}
    graph["pbc"] = torch.zeros(len(mols), 3, dtype=torch.bool)
    data = {f"graph/{k}": v for k, v in graph.items()}
    data["avg_neighbors"] = torch.tensor(avg)

    torch.manual_seed(1)
    teacher = RefPotential(**model_kwargs(avg)).double()
    lab = teacher.predict(_Graph(graph), compute_forces=True)
    e_lab, f_lab = lab["energy"].detach(), lab["forces"].detach()
    data["teacher/energy"], data["teacher/forces"] = e_lab, f_lab

    torch.manual_seed(0)
    student = RefPotential(**model_kwargs(avg)).double()
    data["student/state"] = {k: _digest(v) for k, v in student.state_dict().items() if v.is_floating_point()}
    out = student.predict(_Graph(graph), compute_forces=True, create_graph=True)
    n = graph["n_atoms"].double()
    loss = (((out["energy"] - e_lab) / n) ** 2).mean() + ((out["forces"] - f_lab) ** 2).mean()
    loss.backward()
    data["student/loss"] = loss.detach()
    data["student/grads"] = {k: _digest(p.grad) for k, p in student.named_parameters()}

    main_opt, aux = make_optimizer(student, optimizer="muon", lr=1e-2, weight_decay=1e-3)
    muon_ids = {id(p) for o in aux for gr in o.param_groups for p in gr["params"]}
    no_decay_ids = {id(p) for gr in main_opt.param_groups if gr["weight_decay"] == 0.0 for p in gr["params"]}
    data["routing/muon"] = [k for k, p in student.named_parameters() if id(p) in muon_ids]
    data["routing/no_decay"] = [k for k, p in student.named_parameters() if id(p) in no_decay_ids]
    for o in [main_opt, *aux]:
        o.step()
    data["student/after_step"] = {k: _digest(p) for k, p in student.named_parameters()}
    torch.save(data, os.path.join(HERE, "train_golden.pt"))
    print(f"{len(mols)} molecules, {g['positions'].shape[0]} atoms, {g['edge_index'].shape[1]} edges, "
          f"loss {float(loss):.6e}, {len(data['routing/muon'])} Muon parameters")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLASHCART_REFERENCE_SRC", ""))
