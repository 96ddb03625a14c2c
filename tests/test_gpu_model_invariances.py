"""Symmetries of the B200 potential, as the reference's model tests check them
(``tests/model/test_flashcart.py:43-168``): energy invariant and forces / stress
equivariant under a rotation of the whole periodic box, invariant under a translation,
forces permuted with the atoms, and the virial stress equal to a central finite
difference of the energy under strain. float64 on the 192-atom water box with the
config-0 architecture; the reference's tolerances (1e-9 / 1e-10 relative, stress
atol 1e-7 / rtol 1e-6).
"""

import pytest
import torch

from test_model_parity import _build, _graph

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def setup(model_golden, cuda_device):
    model = _build("cfg0", model_golden).to(cuda_device, torch.float64)
    graph = _graph(model_golden, torch.float64, cuda_device)
    out = model.predict(graph, compute_forces=True, compute_stress=True)
    return model, graph, out


@pytest.fixture(scope="module")
def model_golden():
    import os

    root = os.path.dirname(os.path.abspath(__file__))
    return torch.load(os.path.join(root, "golden", "model_golden.pt"), map_location="cpu", weights_only=True)


def _voigt_to_full(s):
    xx, yy, zz, yz, xz, xy = s.unbind(-1)
    return torch.stack([torch.stack([xx, xy, xz], -1), torch.stack([xy, yy, yz], -1),
                        torch.stack([xz, yz, zz], -1)], -2)


def _close(a, b, rel):
    return (a - b).abs().max().item() <= rel * max(1.0, b.abs().max().item())


def test_gpu_rotation_of_the_box(setup):
    model, graph, out = setup
    g = torch.Generator().manual_seed(1234)
    q, r = torch.linalg.qr(torch.randn(3, 3, generator=g, dtype=torch.float64))
    R = (q * torch.sign(torch.diagonal(r))).to(graph["positions"].device)
    if torch.det(R) < 0:
        R = -R
    rot = dict(graph, positions=graph["positions"] @ R.T, cell=graph["cell"] @ R.T)
    o = model.predict(rot, compute_forces=True, compute_stress=True)
    assert _close(o["energy"], out["energy"], 1e-9)
    assert _close(o["forces"], out["forces"] @ R.T, 1e-9)
    assert _close(_voigt_to_full(o["stress"]), R @ _voigt_to_full(out["stress"]) @ R.T, 1e-9)


def test_gpu_translation(setup):
    model, graph, out = setup
    t = torch.tensor([1.7, -0.3, 2.9], dtype=torch.float64, device=graph["positions"].device)
    o = model.predict(dict(graph, positions=graph["positions"] + t), compute_forces=True, compute_stress=True)
    assert _close(o["energy"], out["energy"], 1e-10)
    assert _close(o["forces"], out["forces"], 1e-10)
    assert _close(o["stress"], out["stress"], 1e-10)


def test_gpu_permutation_of_the_atoms(setup):
    model, graph, out = setup
    dev = graph["positions"].device
    n = graph["positions"].shape[0]
    perm = torch.randperm(n, generator=torch.Generator().manual_seed(7)).to(dev)
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(n, device=dev)
    ei = inv[graph["edge_index"]]
    order = torch.sort(ei[0] * n + ei[1]).indices  # receiver-sorted again
    p = dict(graph, positions=graph["positions"][perm], atom_types=graph["atom_types"][perm],
             edge_index=ei[:, order].contiguous(), shifts=graph["shifts"][order].contiguous())
    o = model.predict(p, compute_forces=True, compute_stress=True)
    assert _close(o["energy"], out["energy"], 1e-10)
    assert _close(o["forces"], out["forces"][perm], 1e-10)
    assert _close(o["stress"], out["stress"], 1e-10)


def test_gpu_stress_matches_finite_difference(setup):
    model, graph, out = setup
    dev = graph["positions"].device
    h = 1.0e-5
    volume = torch.det(graph["cell"][0])

    def energy_at(strain):
        tr = torch.eye(3, dtype=torch.float64, device=dev) + strain
        g = dict(graph, positions=graph["positions"] @ tr.T, cell=graph["cell"] @ tr.T)
        return model.predict(g, compute_forces=False, compute_stress=False)["energy"][0]

    fd = torch.zeros(3, 3, dtype=torch.float64, device=dev)
    for i in range(3):
        for j in range(3):
            s = torch.zeros(3, 3, dtype=torch.float64, device=dev)
            s[i, j] = h
            e_plus = energy_at(s)
            s[i, j] = -h
            fd[i, j] = (e_plus - energy_at(s)) / (2.0 * h)
    fd = (fd + fd.T) / (2.0 * volume)
    torch.testing.assert_close(_voigt_to_full(out["stress"][0]), fd, atol=1.0e-7, rtol=1.0e-6)
    assert fd.abs().max().item() > 1e-5  # the box is not at a stress-free point


def test_gpu_batch_equals_structures_one_by_one(setup, cuda_device):
    """A batch of the periodic box, a water molecule and a lone atom gives each structure's
    energy, forces and stress as evaluated alone (reference
    ``tests/model/test_flashcart.py:107-124``)."""
    from test_model_parity import _isolated_atom_graph

    model, box, out_box = setup
    mol = _isolated_atom_graph(torch.float64, cuda_device, with_molecule=True)
    out_mol = model.predict(mol, compute_forces=True, compute_stress=True)
    nb = box["positions"].shape[0]
    batch = {
        "positions": torch.cat([box["positions"], mol["positions"]]),
        "cell": torch.cat([box["cell"], mol["cell"]]),
        "atom_types": torch.cat([box["atom_types"], mol["atom_types"]]),
        "edge_index": torch.cat([box["edge_index"], mol["edge_index"] + nb], dim=1),
        "shifts": torch.cat([box["shifts"], mol["shifts"].to(box["shifts"].dtype)]),
        "batch": torch.cat([box["batch"], mol["batch"] + 1]),
        "n_atoms": torch.cat([box["n_atoms"], mol["n_atoms"]]),
        "pbc": box["pbc"],
    }
    o = model.predict(batch, compute_forces=True, compute_stress=True)
    for key in ("energy", "forces", "stress"):
        assert _close(o[key], torch.cat([out_box[key], out_mol[key]]), 1e-10), key
