"""LAMMPS ML-IAP interface on the GPU: edge forces, ghost exchanges on the halo kernels.

* the vectors-given fused geometry kernel equals the composed chain (float64);
* ``compute_forces`` on a periodic chain split into owned atoms + ghost images (the
  reference's check, tests/calculators/test_lammps.py:159-208): energies and the folded
  forces equal the undecomposed evaluation for 1-3 interaction layers, with the exchange
  hooks as host copies and as this library's device halo kernels (GhostImageExchange);
* pair forces dE/d(rij), accumulated per atom, equal the model's position forces on the
  192-atom water box (update_pair_forces and data.f paths; shuffled pair order);
* the domain-decomposed ML-IAP evaluation (DomainMLIAPData: halo kernels, gloo ranks
  sharing this GPU) equals the single-cell energy and forces.
"""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_lammps_cpu import HostMLIAPData

pytestmark = pytest.mark.gpu


def _model(n_interactions, r_max, dtype=torch.float64, seed=7):
    from flashcart_b200.model.flashcart import FlashCartPotential

    torch.manual_seed(seed)
    return FlashCartPotential(elements=["H", "O"], r_max=r_max, n_hidden_feats=8, l_max_hidden_feats=1,
                              l_max_edge_attrs=2, n_radial=4, n_interactions=n_interactions, correlation=2,
                              hidden_radial=[8], hidden_readout=[8], fit_atomic_shifts=False,
                              atomic_shifts=[0.0, 0.0]).to(dtype)


class CudaMLIAPData(HostMLIAPData):
    """The host stand-in with its arrays and buffers on the GPU (KOKKOS ML-IAP layout)."""

    def to_cuda(self, dev):
        for k in ("pair_i", "pair_j", "elems"):
            setattr(self, k, torch.as_tensor(getattr(self, k), device=dev))
        self.rij = torch.as_tensor(self.rij, dtype=torch.float64, device=dev)
        self.f = torch.zeros(self.ntotal, 3, dtype=torch.float64, device=dev)
        self.eatoms = torch.zeros(self.nlocal, dtype=torch.float64, device=dev)
        return self


BOX, X1, CUT = 2.0, 0.9, 1.2  # chain of period BOX with atoms at 0 and X1; pairs at 0.9 and 1.1


def _chain_serial(dev):
    d = CudaMLIAPData([[0.0, 0.0, 0.0], [X1, 0.0, 0.0]], elems=[0, 1])
    d.set_pairs([0, 0, 1, 1], [1, 1, 0, 0], [[X1, 0, 0], [X1 - BOX, 0, 0], [-X1, 0, 0], [BOX - X1, 0, 0]])
    return d.to_cuda(dev)


def _chain_decomposed(dev):
    # atoms 0, 1 owned; ghost 2 = image of 0 at +BOX, ghost 3 = image of 1 at X1 - BOX
    d = CudaMLIAPData([[0.0, 0.0, 0.0], [X1, 0.0, 0.0], [BOX, 0.0, 0.0], [X1 - BOX, 0.0, 0.0]], nlocal=2,
                      elems=[0, 1, 0, 1])
    d.ghost_owner = {2: 0, 3: 1}
    d.pairs_within(CUT)
    return d.to_cuda(dev)


def _fold(d):
    f = d.f.clone()
    out = f[:d.nlocal].clone()
    for g, o in d.ghost_owner.items():
        out[o] += f[g]
    return out


def test_vec_geometry_matches_composed_chain(cuda_device):
    from flashcart_b200 import ops

    model = _model(2, 3.0).to(cuda_device)
    g = torch.Generator(device="cpu").manual_seed(1)
    v = (torch.randn(4000, 3, generator=g, dtype=torch.float64) * 1.6).to(cuda_device)
    v[0] = 0.0
    v[1] = torch.tensor([3e-5, 0.0, 0.0])   # below the direction clamp
    v[2] = torch.tensor([0.0, 3.5, 0.0])    # beyond the cutoff
    v.requires_grad_(True)
    with ops.first_order_only():
        attrs, radial = ops.edge_geometry_vec(v, model.irreps.l_max, *model._geometry_args)
    # composed chain on the edges of valid length only: Irreps.forward_normalized rejects
    # the non-unit directions of edges shorter than the 1e-4 clamp (rows 0 and 1)
    vv = v[2:]
    r = vv.norm(dim=-1)
    d = vv / r.clamp_min(1e-4).unsqueeze(-1)
    attrs_c = model.irreps.forward_normalized(d)
    radial_c = model.radial_basis(r) * model.cutoff_fn(r).unsqueeze(-1)
    assert float((attrs[2:] - attrs_c).abs().max()) < 1e-12
    assert float((radial[2:] - radial_c).abs().max()) < 1e-12
    ga = torch.randn(attrs.shape, generator=g, dtype=torch.float64).to(cuda_device)
    gr = torch.randn(radial.shape, generator=g, dtype=torch.float64).to(cuda_device)
    (gv,) = torch.autograd.grad((attrs * ga).sum() + (radial * gr).sum(), v)
    (gv_c,) = torch.autograd.grad((attrs_c * ga[2:]).sum() + (radial_c * gr[2:]).sum(), v)
    assert float((gv[2:] - gv_c[2:]).abs().max()) < 1e-10
    assert torch.isfinite(gv).all() and torch.isfinite(attrs).all() and torch.isfinite(radial).all()
    ops.check_device_status(cuda_device)


@pytest.mark.parametrize("n_interactions", [1, 2, 3])
def test_mliap_decomposed_chain_matches_serial(cuda_device, n_interactions):
    from flashcart_b200.lammps import FlashCartLAMMPSUnified, GhostImageExchange

    unified = FlashCartLAMMPSUnified(_model(n_interactions, CUT))
    serial = _chain_serial(cuda_device)
    unified.compute_forces(serial)
    assert serial.forward_exchange_calls == n_interactions - 1  # ranks without ghosts still exchange
    assert unified.device.type == "cuda"
    assert float(serial.f.abs().max()) > 0.0

    host = _chain_decomposed(cuda_device)
    unified.compute_forces(host)
    assert host.forward_exchange_calls == n_interactions - 1
    assert host.reverse_exchange_calls == n_interactions - 1
    assert torch.allclose(host.eatoms, serial.eatoms, atol=1e-10, rtol=1e-10)
    assert torch.allclose(_fold(host), serial.f, atol=1e-10, rtol=1e-10)
    assert host.energy == pytest.approx(serial.energy, abs=1e-10)

    # the same exchanges on the device halo kernels
    dev = _chain_decomposed(cuda_device)
    hooks = GhostImageExchange(torch.tensor([0, 1]), nlocal=2)
    dev.forward_exchange, dev.reverse_exchange = hooks.forward_exchange, hooks.reverse_exchange
    unified.compute_forces(dev)
    assert hooks.forward_exchange_calls == n_interactions - 1
    assert hooks.reverse_exchange_calls == n_interactions - 1
    assert torch.allclose(dev.eatoms, host.eatoms, atol=1e-12, rtol=1e-12)
    assert torch.allclose(dev.f, host.f, atol=1e-12, rtol=1e-12)


def _water(dev, dtype):
    from flashcart_b200.data import neighbors, synthetic
    from flashcart_b200.model.flashcart import FlashCartPotential
    from flashcart_b200.model.presets import water_model_kwargs

    s = synthetic.config0_water()
    ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
    graph = synthetic.graph_from_structure(s, ei, sh, device=dev, dtype=dtype)
    torch.manual_seed(0)
    model = FlashCartPotential(**water_model_kwargs("cfg3arch", ei.shape[1] / len(s["positions"]))).to(dev)
    return s, ei, sh, graph, model.to(dtype)


def _water_mliap(s, ei, sh, dev, perm=None):
    pos = np.asarray(s["positions"], np.float64)
    rij = pos[ei[1]] - pos[ei[0]] + np.asarray(sh, np.float64) @ np.asarray(s["cell"], np.float64)
    d = CudaMLIAPData(pos, elems=np.asarray(s["atom_types"]))
    pi, pj = ei[0], ei[1]
    if perm is not None:
        pi, pj, rij = pi[perm], pj[perm], rij[perm]
    d.set_pairs(pi, pj, rij)
    return d.to_cuda(dev)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-9), (torch.float32, 2e-4)])
def test_pair_forces_equal_position_forces_on_water(cuda_device, dtype, tol):
    from flashcart_b200.lammps import FlashCartLAMMPSUnified

    s, ei, sh, graph, model = _water(cuda_device, dtype)
    ref = model.predict(graph, compute_forces=True)
    unified = FlashCartLAMMPSUnified(model)
    d = _water_mliap(s, ei, sh, cuda_device)
    unified.compute_forces(d)
    assert d.energy == pytest.approx(float(ref["energy"][0]), abs=tol * 192)
    assert float((d.eatoms - ref["node_energies"].double()).abs().max()) < tol
    assert float((d.f - ref["forces"].double()).abs().max()) < tol

    # LAMMPS's own accumulation of pair forces (update_pair_forces), and a shuffled pair list
    got = {}
    perm = np.random.default_rng(3).permutation(ei.shape[1])
    shuffled = _water_mliap(s, ei, sh, cuda_device, perm)
    shuffled.update_pair_forces = lambda pf: got.__setitem__("pf", pf.clone())
    unified.compute_forces(shuffled)
    pf = got["pf"]
    assert pf.dtype == torch.float64 and pf.shape == (ei.shape[1], 3)
    f = torch.zeros(192, 3, dtype=torch.float64, device=cuda_device)
    pi = torch.as_tensor(ei[0][perm], device=cuda_device)
    pj = torch.as_tensor(ei[1][perm], device=cuda_device)
    f.index_add_(0, pi, pf).index_add_(0, pj, -pf)
    assert float((f - d.f).abs().max()) < tol / 10


def _domain_worker(rank, world, port, outdir):
    from flashcart_b200.domain import build_plans
    from flashcart_b200.lammps import DomainMLIAPData, FlashCartLAMMPSUnified

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        s, ei, sh, graph, model = _water(dev, torch.float64)
        plan = build_plans(s["positions"], s["cell"], ei, sh, world)[rank]
        data = DomainMLIAPData(plan, graph["positions"], s["cell"], graph["atom_types"])
        unified = FlashCartLAMMPSUnified(model)
        unified.compute_forces(data)
        torch.save({"owned": plan.owned, "forces": data.owned_forces().cpu(), "eatoms": data.eatoms.cpu(),
                    "energy": data.energy, "n_ghost": plan.n_ghost, "calls": data.forward_exchange_calls},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_domain_mliap_over_halo_kernels_matches_single_cell(cuda_device):
    s, ei, sh, graph, model = _water(cuda_device, torch.float64)
    ref = model.predict(graph, compute_forces=True)
    world = 2
    with tempfile.TemporaryDirectory() as d:
        port = 29800 + (os.getpid() % 150)
        mp.start_processes(_domain_worker, args=(world, port, d), nprocs=world, start_method="spawn")
        parts = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    assert all(p["n_ghost"] > 0 and p["calls"] == model.n_interactions - 1 for p in parts)
    forces = torch.full((192, 3), float("nan"), dtype=torch.float64)
    eatoms = torch.full((192,), float("nan"), dtype=torch.float64)
    for p in parts:
        forces[p["owned"]] = p["forces"]
        eatoms[p["owned"]] = p["eatoms"]
    assert not torch.isnan(forces).any()
    assert float((forces - ref["forces"].cpu()).abs().max()) < 1e-9
    assert float((eatoms - ref["node_energies"].cpu()).abs().max()) < 1e-9
    assert sum(p["energy"] for p in parts) == pytest.approx(float(ref["energy"][0]), abs=1e-8)
