"""Module-level drop-in: the reference's own layer and model code on ``flashcart_b200.o3``.

The reference's ``nn/layers.py`` and ``model/flashcart.py`` import ``from flashcart import
o3``. Here that name resolves to ``flashcart_b200.o3`` (the one-import switch of the
integration guide), and the reference's ``FlashCartPotential`` (model/flashcart.py:25)
with its ``InteractionLayer`` / ``ProductLayer`` / gates (nn/layers.py:184-1138) is built
unchanged on top of the B200 modules:

* CPU: the seeded construction draws the same parameters, state-dict keys and shapes as
  the B200 mirror (``flashcart_b200.model``), and every tensor-product / linear / irreps
  module inside it is a B200 module;
* GPU: energy, forces and stress of the reference model on the B200 operators equal the
  mirror's on the 192-atom water box (float64).

The reference package is found in ``baseline/_ref`` (the offline ``pip install --target``
of the reference) or at ``$FLASHCART_REFERENCE_SRC``; without it the tests skip. Each case
runs in a spawned process, so the reference's ``flashcart`` operator registrations never
meet this library's in one interpreter.
"""

import os
import sys
import tempfile
import types

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_src():
    for cand in (os.environ.get("FLASHCART_REFERENCE_SRC"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isfile(os.path.join(cand, "flashcart", "model", "flashcart.py")):
            return cand
    return None


def _import_reference_on_b200(src):
    """Import the reference package with ``flashcart.o3`` bound to ``flashcart_b200.o3``."""
    if "lightning" not in sys.modules:  # model/flashcart.py imports lightning.fabric for a type hint
        lightning = types.ModuleType("lightning")
        fabric = types.ModuleType("lightning.fabric")
        fabric.Fabric = type("Fabric", (), {})
        lightning.fabric = fabric
        sys.modules["lightning"], sys.modules["lightning.fabric"] = lightning, fabric
    sys.path.insert(0, src)
    import flashcart

    import flashcart_b200.o3 as b200_o3

    sys.modules["flashcart.o3"] = b200_o3
    flashcart.o3 = b200_o3
    from flashcart.model.flashcart import FlashCartPotential

    return FlashCartPotential


class _Graph:
    def __init__(self, d):
        self._d = d

    def to_dict(self):
        return dict(self._d)


def _water(device, dtype):
    from flashcart_b200.data import neighbors, synthetic

    s = synthetic.config0_water()
    ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
    return synthetic.graph_from_structure(s, ei, sh, device=device, dtype=dtype), ei.shape[1] / len(s["positions"])


def _child(rank, src, arch, device, outpath):
    from flashcart_b200.model.flashcart import FlashCartPotential as Mirror
    from flashcart_b200.model.presets import water_model_kwargs

    RefOnB200 = _import_reference_on_b200(src)
    dtype = torch.float64
    graph, avg = _water(device, dtype)
    kw = water_model_kwargs(arch, avg)
    torch.manual_seed(0)
    ref = RefOnB200(**kw).to(device, dtype)
    torch.manual_seed(0)
    mirror = Mirror(**kw).to(device, dtype)
    res = {"ref_keys": list(ref.state_dict().keys()), "mirror_keys": list(mirror.state_dict().keys()),
           "max_param_diff": max(float((a.double() - b.double()).abs().max()) if a.numel() else 0.0
                                 for a, b in zip(ref.state_dict().values(), mirror.state_dict().values())),
           "ref_shapes": [tuple(v.shape) for v in ref.state_dict().values()],
           "mirror_shapes": [tuple(v.shape) for v in mirror.state_dict().values()],
           "o3_modules": sorted({type(m).__module__ for m in ref.modules()
                                 if type(m).__name__ in ("TensorProduct", "LinearLayer", "Irreps")
                                 and not type(m).__module__.startswith("flashcart.nn")}),
           "ref_o3": {k: type(getattr(ref.interactions[0], k)).__module__ for k in ("tp", "linear_first")},
           "ref_class_module": type(ref).__module__}
    if device.startswith("cuda"):
        out_r = ref.predict(_Graph(graph), compute_forces=True, compute_stress=True)
        out_m = mirror.predict(graph, compute_forces=True, compute_stress=True)
        for k in ("energy", "forces", "stress"):
            res[f"ref_{k}"] = out_r[k].detach().cpu()
            res[f"mirror_{k}"] = out_m[k].detach().cpu()
    torch.save(res, outpath)


def _run(arch, device):
    src = _reference_src()
    if src is None:
        pytest.skip("the reference package is not installed (baseline/_ref or $FLASHCART_REFERENCE_SRC)")
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "res.pt")
        mp.start_processes(_child, args=(src, arch, device, out), nprocs=1, start_method="spawn")
        return torch.load(out, weights_only=False)


@pytest.mark.parametrize("arch", ["cfg0", "cfg3arch"])
def test_reference_model_builds_on_b200_modules(arch):
    r = _run(arch, "cpu")
    assert r["ref_class_module"] == "flashcart.model.flashcart"
    # the reference's own nn.layers.LinearLayer is a dense MLP layer, not an o3 module
    assert r["o3_modules"] and all(m.startswith("flashcart_b200.o3") for m in r["o3_modules"]), r["o3_modules"]
    assert all(m.startswith("flashcart_b200.o3") for m in r["ref_o3"].values()), r["ref_o3"]
    assert r["ref_keys"] == r["mirror_keys"]
    assert r["ref_shapes"] == r["mirror_shapes"]
    assert r["max_param_diff"] == 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("arch", ["cfg0", "cfg3arch"])
def test_reference_model_on_b200_operators_matches_mirror(cuda_device, arch):
    r = _run(arch, "cuda:0")
    assert r["max_param_diff"] == 0.0
    e = float(r["mirror_energy"].abs().max())
    assert float((r["ref_energy"] - r["mirror_energy"]).abs().max()) <= 1e-10 * max(e, 1.0)
    assert float((r["ref_forces"] - r["mirror_forces"]).abs().max()) <= 1e-9
    assert float((r["ref_stress"] - r["mirror_stress"]).abs().max()) <= 1e-9
