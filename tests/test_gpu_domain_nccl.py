"""Atom-domain decomposition over NCCL, one process per GPU (skipped with fewer GPUs).

The same path the multi-GPU benchmark runs: each rank owns one domain of a periodic water
box (128 channels, ranks <= 3), packs and unpacks its halo rows with this library's
kernels, moves them with NCCL all-to-all, and the whole step is also captured as a CUDA
graph (NCCL collectives included) and replayed. Energy, the owned atoms' forces and the
stress of the eager step and of the replay must match the single-cell evaluation on one
GPU to float32 summation-order differences (reference semantics: the domain-decomposed
LAMMPS evaluation equals the serial one, ``tests/calculators/test_lammps.py:190-208``).
"""

import datetime
import os
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _setup(dev):
    from flashcart_b200.data import neighbors, synthetic
    from flashcart_b200.model.flashcart import FlashCartPotential
    from flashcart_b200.model.presets import water_model_kwargs

    s = synthetic.water_box(8, 8, 4, seed=0)  # 768 atoms, 24.8 x 24.8 x 12.4 A
    ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
    graph = synthetic.graph_from_structure(s, ei, sh, device=dev, dtype=torch.float32)
    torch.manual_seed(0)
    model = FlashCartPotential(**water_model_kwargs("cfg3arch", ei.shape[1] / len(s["positions"]))).to(dev)
    return graph, model


def _worker(rank, world, port, outdir):
    from flashcart_b200.domain import build_plans
    from flashcart_b200.graphs import GraphedStep
    from flashcart_b200.ops import check_device_status

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    graphed = None
    try:
        graph, model = _setup(dev)
        plan = build_plans(graph["positions"].cpu(), graph["cell"][0].cpu(), graph["edge_index"].cpu(),
                           graph["shifts"].cpu(), world)[rank].to(dev)
        step = lambda g: model.predict_domain(g, plan)
        eager = {k: v.detach().cpu() for k, v in step(graph).items()}
        graphed = GraphedStep(step, dict(graph), warmup=2)
        rep = {k: v.detach().cpu() for k, v in graphed().items()}
        torch.cuda.synchronize()
        check_device_status(dev)
        torch.save({"owned": plan.owned.cpu(), "eager": eager, "replay": rep, "n_ghost": plan.n_ghost},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        if graphed is not None:
            graphed.release()
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gpu_domain_decomposition_over_nccl(cuda_device, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    graph, model = _setup(cuda_device)
    ref = model.predict(graph, compute_forces=True, compute_stress=True)
    ref = {k: v.detach().cpu() for k, v in ref.items()}
    n = ref["forces"].shape[0]
    with tempfile.TemporaryDirectory() as d:
        port = 29900 + world + (os.getpid() % 97)
        mp.start_processes(_worker, args=(world, port, d), nprocs=world, start_method="spawn")
        parts = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    assert all(p["n_ghost"] > 0 for p in parts)
    for kind in ("eager", "replay"):
        forces = torch.full_like(ref["forces"], float("nan"))
        for p in parts:
            out = p[kind]
            forces[p["owned"]] = out["forces"]
            assert abs(float(out["energy"][0]) - float(ref["energy"][0])) <= 1e-5 * n, kind
            assert float((out["stress"] - ref["stress"]).abs().max()) <= 1e-5, kind
        assert not torch.isnan(forces).any(), kind
        assert float((forces - ref["forces"]).abs().max()) <= 1e-4, kind


def _mliap_worker(rank, world, port, outdir):
    from flashcart_b200.domain import build_plans
    from flashcart_b200.lammps import DomainMLIAPData, FlashCartLAMMPSUnified
    from flashcart_b200.ops import check_device_status

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        graph, model = _setup(dev)
        plan = build_plans(graph["positions"].cpu(), graph["cell"][0].cpu(), graph["edge_index"].cpu(),
                           graph["shifts"].cpu(), world)[rank]
        data = DomainMLIAPData(plan, graph["positions"], graph["cell"][0], graph["atom_types"],
                               dtype=torch.float32)
        unified = FlashCartLAMMPSUnified(model)
        unified.compute_forces(data)
        forces = data.owned_forces()
        torch.cuda.synchronize()
        check_device_status(dev)
        torch.save({"owned": plan.owned.cpu(), "forces": forces.cpu(), "eatoms": data.eatoms.cpu(),
                    "energy": data.energy, "n_ghost": plan.n_ghost}, os.path.join(outdir, f"m{rank}.pt"))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 8])
def test_gpu_lammps_mliap_domains_over_nccl(cuda_device, world):
    """The LAMMPS ML-IAP interface on domain ranks (DomainMLIAPData: halo kernels + NCCL
    all-to-all as its forward / reverse exchange hooks) equals the single-cell evaluation."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    graph, model = _setup(cuda_device)
    ref = model.predict(graph, compute_forces=True)
    ref = {k: v.detach().cpu() for k, v in ref.items()}
    n = ref["forces"].shape[0]
    with tempfile.TemporaryDirectory() as d:
        port = 29950 + world + (os.getpid() % 37)
        mp.start_processes(_mliap_worker, args=(world, port, d), nprocs=world, start_method="spawn")
        parts = [torch.load(os.path.join(d, f"m{r}.pt")) for r in range(world)]
    assert all(p["n_ghost"] > 0 for p in parts)
    forces = torch.full((n, 3), float("nan"), dtype=torch.float64)
    eatoms = torch.full((n,), float("nan"), dtype=torch.float64)
    for p in parts:
        forces[p["owned"]] = p["forces"]
        eatoms[p["owned"]] = p["eatoms"]
    assert not torch.isnan(forces).any()
    assert float((forces - ref["forces"].double()).abs().max()) <= 1e-4
    assert float((eatoms - ref["node_energies"].double()).abs().max()) <= 1e-5
    assert abs(sum(p["energy"] for p in parts) - float(ref["energy"][0])) <= 1e-5 * n
