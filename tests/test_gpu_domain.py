"""Atom-domain decomposition of the real potential on the GPU.

The config-3 architecture (C = 128, ranks <= 3) evaluates the 192-atom water box once in
this process and then as 2 and 4 domains, each domain a spawned process on the same GPU
(halo exchange over gloo, staged through host memory; no kernel waits on another
process). Energy, the owned atoms' forces and the stress must match the single-cell
evaluation to float32 summation-order differences.
"""

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

    s = synthetic.config0_water()
    ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
    graph = synthetic.graph_from_structure(s, ei, sh, device=dev, dtype=torch.float32)
    torch.manual_seed(0)
    model = FlashCartPotential(**water_model_kwargs("cfg3arch", ei.shape[1] / len(s["positions"]))).to(dev)
    return graph, model


def _worker(rank, world, port, outdir):
    from flashcart_b200.domain import build_plans

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        graph, model = _setup(dev)
        plan = build_plans(graph["positions"].cpu(), graph["cell"][0].cpu(), graph["edge_index"].cpu(),
                           graph["shifts"].cpu(), world)[rank].to(dev)
        out = model.predict_domain(graph, plan)
        torch.save({"owned": plan.owned.cpu(), "forces": out["forces"].cpu(), "energy": out["energy"].cpu(),
                    "stress": out["stress"].cpu(), "n_ghost": plan.n_ghost}, os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gpu_domain_decomposition_matches_single_cell(cuda_device, world):
    graph, model = _setup(cuda_device)
    ref = model.predict(graph, compute_forces=True, compute_stress=True)
    ref = {k: v.detach().cpu() for k, v in ref.items()}
    with tempfile.TemporaryDirectory() as d:
        port = 29700 + world + (os.getpid() % 200)
        mp.start_processes(_worker, args=(world, port, d), nprocs=world, start_method="spawn")
        parts = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    assert all(p["n_ghost"] > 0 for p in parts)
    forces = torch.full_like(ref["forces"], float("nan"))
    for p in parts:
        forces[p["owned"]] = p["forces"]
        # energy ~ 1e2 eV over 192 atoms: fp32 summation order only
        assert abs(float(p["energy"][0]) - float(ref["energy"][0])) <= 1e-5 * 192
        assert float((p["stress"] - ref["stress"]).abs().max()) <= 1e-5
    assert not torch.isnan(forces).any()
    assert float((forces - ref["forces"]).abs().max()) <= 1e-4
