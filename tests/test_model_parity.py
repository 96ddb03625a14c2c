"""FlashCart potential parity: seeded weights, oracle and B200 model vs the reference's golden E/F/S.

Tolerance policy for float32 (north star: energies 1e-5 eV/atom, forces 1e-4 eV/A,
stress 1e-4 eV/A^3): the B200 float32 result is judged against the reference float64
result and passes if |ours_f32 - ref_f64| <= max(tol, 2 |ref_f32 - ref_f64|).
float64 runs must agree with the reference float64 run to 1e-9 (relative to scale).
"""

import pytest
import torch

from flashcart_b200.model.flashcart import FlashCartPotential
from oracle import model_oracle

CASES = ["cfg0", "cfg3arch"]
TOL = {"energy_per_atom": 1e-5, "forces": 1e-4, "stress": 1e-4}


@pytest.fixture(scope="module")
def model_golden():
    import os

    root = os.path.dirname(os.path.abspath(__file__))
    return torch.load(os.path.join(root, "golden", "model_golden.pt"), map_location="cpu", weights_only=True)


def _kwargs(name, avg):
    from golden.make_model_golden import model_kwargs

    return model_kwargs(name, avg)


def _build(name, golden):
    torch.manual_seed(0)
    return FlashCartPotential(**_kwargs(name, float(golden["avg_neighbors"])))


def _graph(golden, dtype, device="cpu"):
    n = golden["positions"].shape[0]
    return {
        "positions": golden["positions"].to(device, dtype), "cell": golden["cell"].to(device, dtype).unsqueeze(0),
        "atom_types": golden["atom_types"].to(device), "edge_index": golden["edge_index"].to(device),
        "shifts": golden["shifts"].to(device), "batch": torch.zeros(n, dtype=torch.int64, device=device),
        "n_atoms": torch.tensor([n], device=device), "pbc": torch.tensor([True, True, True], device=device),
    }


@pytest.mark.parametrize("name", CASES)
def test_seeded_construction_draws_the_reference_weights(model_golden, name):
    model = _build(name, model_golden)
    sd = model.state_dict()
    assert len(sd) == int(model_golden[f"{name}/param_keys"])
    for k, v in sd.items():
        if not v.is_floating_point():
            continue
        assert f"{name}/param_sum/{k}" in model_golden, k
        assert float(v.double().sum()) == float(model_golden[f"{name}/param_sum/{k}"]), k
        assert float((v.double() ** 2).sum()) == float(model_golden[f"{name}/param_sq/{k}"]), k


@pytest.mark.parametrize("name", CASES)
def test_oracle_potential_matches_reference(model_golden, name):
    model = _build(name, model_golden)
    sd = {k: v.double() if v.is_floating_point() else v for k, v in model.state_dict().items()}
    out = model_oracle.predict(sd, _kwargs(name, float(model_golden["avg_neighbors"])),
                               _graph(model_golden, torch.float64))
    for key in ("energy", "forces", "stress"):
        ref = model_golden[f"{name}/f64/{key}"]
        assert (out[key] - ref).abs().max() <= 1e-9 * max(1.0, ref.abs().max().item()), key


def _check_f32(out, golden, name, n):
    f64, f32 = (lambda k: golden[f"{name}/f64/{k}"]), (lambda k: golden[f"{name}/f32/{k}"])
    e_err = (out["energy"].double().cpu() - f64("energy")).abs().max().item() / n
    e_ref = (f32("energy") - f64("energy")).abs().max().item() / n
    assert e_err <= max(TOL["energy_per_atom"], 2 * e_ref), (e_err, e_ref)
    for key in ("forces", "stress"):
        err = (out[key].double().cpu() - f64(key)).abs().max().item()
        ref_gap = (f32(key) - f64(key)).abs().max().item()
        assert err <= max(TOL[key], 2 * ref_gap), (key, err, ref_gap)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_b200_potential_matches_reference(model_golden, name, cuda_device):
    n = model_golden["positions"].shape[0]
    model = _build(name, model_golden)
    m64 = model.to(cuda_device, torch.float64)
    out = m64.predict(_graph(model_golden, torch.float64, cuda_device), compute_forces=True, compute_stress=True)
    for key in ("energy", "forces", "stress"):
        ref = model_golden[f"{name}/f64/{key}"]
        assert (out[key].cpu() - ref).abs().max() <= 1e-9 * max(1.0, ref.abs().max().item()), key
    model = _build(name, model_golden).to(cuda_device)
    out = model.predict(_graph(model_golden, torch.float32, cuda_device), compute_forces=True, compute_stress=True)
    _check_f32(out, model_golden, name, n)


def _isolated_atom_graph(dtype, device, with_molecule):
    """A water molecule (6 edges) and a hydrogen atom 20 A away with no neighbour, as two
    structures of one batch; or the lone atom alone (no edge in the whole batch)."""
    lone = [[30.0, 30.0, 30.0]]
    if with_molecule:
        pos = [[10.0, 10.0, 10.0], [10.96, 10.0, 10.0], [9.76, 10.93, 10.0]] + lone
        types, batch, counts = [1, 0, 0, 0], [0, 0, 0, 1], [3, 1]
        edges = [[0, 0, 1, 1, 2, 2], [1, 2, 0, 2, 0, 1]]
    else:
        pos, types, batch, counts, edges = lone, [0], [0], [1], [[], []]
    g = len(counts)
    return {
        "positions": torch.tensor(pos, dtype=dtype, device=device),
        "cell": (40.0 * torch.eye(3, dtype=dtype, device=device)).expand(g, 3, 3).contiguous(),
        "atom_types": torch.tensor(types, device=device), "edge_index": torch.tensor(edges, dtype=torch.int64,
                                                                                     device=device),
        "shifts": torch.zeros(len(edges[0]), 3, dtype=torch.int32, device=device),
        "batch": torch.tensor(batch, device=device), "n_atoms": torch.tensor(counts, device=device),
        "pbc": torch.tensor([False, False, False], device=device),
    }


@pytest.mark.gpu
@pytest.mark.parametrize("with_molecule", [True, False])
def test_b200_potential_with_isolated_atoms(model_golden, with_molecule, cuda_device):
    """Atoms without neighbours (and a batch without a single edge) give the oracle's
    energies, zero forces on the lone atom and finite stress, in float64."""
    name = "cfg0"
    model = _build(name, model_golden)
    sd = {k: v.double() if v.is_floating_point() else v for k, v in model.state_dict().items()}
    ref = model_oracle.predict(sd, _kwargs(name, float(model_golden["avg_neighbors"])),
                               _isolated_atom_graph(torch.float64, "cpu", with_molecule))
    m64 = model.to(cuda_device, torch.float64)
    out = m64.predict(_isolated_atom_graph(torch.float64, cuda_device, with_molecule), compute_forces=True,
                      compute_stress=True)
    for key in ("energy", "forces", "stress"):
        r = ref[key]
        assert (out[key].cpu() - r).abs().max() <= 1e-9 * max(1.0, r.abs().max().item()), key
    assert (out["forces"][-1] == 0).all()
