"""Golden energies / forces / stress of the REFERENCE FlashCart potential.

Run where the reference source is available (never needed at test time)::

    python tests/golden/make_model_golden.py <reference>/src

Cases (architecture flags of the reference's default.yaml, avg_neighbors = measured
mean degree; the architectures of the 192-atom CPU reference run and of the MD-scale
inference step):

* ``cfg0``: elements [H, O], r_max 5, 64 channels, hidden l<=2, edge l<=2, 8 radial
  functions, 2 interactions, correlation 3, layer norm, sigmoid gates, cosine
  Chebyshev mapping, path-resolved products;
* ``cfg3arch``: the same with 128 channels and hidden / edge l<=3.

Both run on the seeded 192-atom water box of ``flashcart_b200.data.synthetic``
with the canonical neighbour list of ``flashcart_b200.data.neighbors`` (the
reference's own list comes from matscipy, which is not installed; the TP result
does not depend on the order of a receiver's edges beyond rounding).
The model weights are the reference's seeded random initialisation
(``torch.manual_seed(0)`` before construction); per-parameter checksums are stored
so the tests can verify that the B200 model draws exactly the same weights.
Energies, forces and stress are recorded in float64 and float32 (CPU).

Output: ``tests/golden/model_golden.pt``.
"""

from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

sys.path.insert(0, ROOT)
from flashcart_b200.model.presets import WATER_ARCHS as CONFIGS, water_model_kwargs  # noqa: E402


def model_kwargs(name: str, avg_neighbors: float) -> dict:
    return water_model_kwargs(name, avg_neighbors)


def _fabric_shim():
    """The reference model module imports lightning.fabric for a type hint and a broadcast."""
    if "lightning" in sys.modules:
        return
    lightning = types.ModuleType("lightning")
    fabric = types.ModuleType("lightning.fabric")

    class Fabric:  # noqa: D401 - test-only placeholder
        pass

    fabric.Fabric = Fabric
    lightning.fabric = fabric
    sys.modules["lightning"] = lightning
    sys.modules["lightning.fabric"] = fabric


class _Graph:
    def __init__(self, d):
        self._d = d

    def to_dict(self):
        return dict(self._d)


def main(ref_src: str) -> None:
    sys.path.insert(0, ROOT)
    sys.path.insert(1, ref_src)
    _fabric_shim()
    from flashcart.model.flashcart import FlashCartPotential as RefPotential  # reference

    from flashcart_b200.data import neighbors, synthetic

    s = synthetic.config0_water()
    edge_index, shifts = neighbors.neighbor_list_bruteforce(s["positions"], s["cell"], s["pbc"], 5.0)
    n = len(s["positions"])
    avg = edge_index.shape[1] / n
    data = {"positions": torch.tensor(s["positions"]), "cell": torch.tensor(s["cell"]),
            "atom_types": torch.tensor(s["atom_types"]), "edge_index": torch.tensor(edge_index),
            "shifts": torch.tensor(shifts), "avg_neighbors": torch.tensor(avg)}
    for name in CONFIGS:
        torch.manual_seed(0)
        model = RefPotential(**model_kwargs(name, avg))
        sd = model.state_dict()
        for k, v in sd.items():
            if v.is_floating_point():
                data[f"{name}/param_sum/{k}"] = v.double().sum()
                data[f"{name}/param_sq/{k}"] = (v.double() ** 2).sum()
        data[f"{name}/param_keys"] = torch.tensor([len(sd)])
        for dtype, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
            m = RefPotential(**model_kwargs(name, avg))
            m.load_state_dict(sd)
            m = m.to(dtype)
            graph = {
                "positions": data["positions"].to(dtype), "cell": data["cell"].to(dtype).unsqueeze(0),
                "atom_types": data["atom_types"], "edge_index": data["edge_index"],
                "shifts": data["shifts"], "batch": torch.zeros(n, dtype=torch.int64),
                "n_atoms": torch.tensor([n]), "pbc": torch.tensor([True, True, True]),
            }
            out = m.predict(_Graph(graph), compute_forces=True, compute_stress=True)
            data[f"{name}/{tag}/energy"] = out["energy"].detach().double()
            data[f"{name}/{tag}/node_energies"] = out["node_energies"].detach().double()
            data[f"{name}/{tag}/forces"] = out["forces"].detach().double()
            data[f"{name}/{tag}/stress"] = out["stress"].detach().double()
            print(name, tag, float(out["energy"][0]) / n, float(out["forces"].abs().max()),
                  float(out["stress"].abs().max()))
    torch.save(data, os.path.join(HERE, "model_golden.pt"))
    print(f"wrote {len(data)} entries; E = {edge_index.shape[1]} edges ({avg:.2f}/atom)")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLASHCART_REFERENCE_SRC", ""))
