"""Atom-domain decomposition on CPU ranks (gloo): plans, halo exchange and its backward.

A torch-only two-layer message-passing potential (layer 2 reads the senders' layer-1
outputs, so ghosts need the exchanged features) is evaluated serially and with 2 and 4
gloo ranks in spawned processes; energy, every atom's force and the stress must agree
to float64 round-off. The same evaluation driver (``evaluate_domain``) runs the real
potential on GPU ranks.
"""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashcart_b200.data import neighbors, synthetic
from flashcart_b200.domain import build_plans, domain_grid, evaluate_domain

C = 6


def _structure():
    s = synthetic.config0_water()
    ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
    g = torch.Generator().manual_seed(3)
    params = {"emb": torch.randn(2, C, generator=g, dtype=torch.float64),
              "W1": torch.randn(C, C, generator=g, dtype=torch.float64) / C ** 0.5,
              "W2": torch.randn(C, C, generator=g, dtype=torch.float64) / C ** 0.5}
    graph = {"positions": torch.as_tensor(s["positions"], dtype=torch.float64),
             "cell": torch.as_tensor(s["cell"], dtype=torch.float64).reshape(1, 3, 3),
             "atom_types": torch.as_tensor(s["atom_types"]), "edge_index": torch.as_tensor(ei),
             "shifts": torch.as_tensor(sh)}
    return graph, params


def _toy_energy(params):
    def fn(g, n_out, halo_fn):
        pos, cell, ei = g["positions"], g["cell"], g["edge_index"]
        vec = pos[ei[1]] - pos[ei[0]] + g["shifts"].to(pos.dtype) @ cell[0]
        r2 = (vec * vec).sum(-1)
        f1 = torch.exp(-r2 / 4.0) * (1.0 - r2 / 25.0) ** 2
        h0 = params["emb"][g["atom_types"]]
        m1 = h0.new_zeros(n_out, C).index_add(0, ei[0], f1.unsqueeze(-1) * h0[ei[1]])
        h1 = torch.tanh(m1 @ params["W1"] + h0[:n_out])
        if halo_fn is not None:
            h1 = torch.cat([h1, halo_fn(h1)], dim=0)
        f2 = torch.exp(-r2 / 9.0) * (1.0 - r2 / 25.0) ** 2 * vec[:, 0]
        m2 = h1.new_zeros(n_out, C).index_add(0, ei[0], f2.unsqueeze(-1) * h1[ei[1]])
        return torch.tanh(m2 @ params["W2"] + h1[:n_out]).sum(-1)
    return fn


def _worker(rank, world, port, outdir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        graph, params = _structure()
        plan = build_plans(graph["positions"], graph["cell"], graph["edge_index"], graph["shifts"], world)[rank]
        out = evaluate_domain(_toy_energy(params), graph, plan)
        torch.save({"owned": plan.owned, "forces": out["forces"].detach(), "energy": out["energy"],
                    "stress": out["stress"], "n_ghost": plan.n_ghost},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_domain_grid_factors():
    assert domain_grid(2, [74.5, 74.5, 49.7]) == (2, 1, 1)
    assert domain_grid(4, [74.5, 74.5, 49.7]) == (2, 2, 1)
    assert domain_grid(8, [74.5, 74.5, 49.7]) == (2, 2, 2)
    assert domain_grid(3, [10, 20, 5]) == (1, 3, 1)


def test_plans_partition_every_edge_and_atom_once():
    graph, _ = _structure()
    n = graph["positions"].shape[0]
    e = graph["edge_index"].shape[1]
    for world in (1, 2, 4, 8):
        plans = build_plans(graph["positions"], graph["cell"], graph["edge_index"], graph["shifts"], world)
        owned = torch.cat([p.owned for p in plans]).sort().values
        assert torch.equal(owned, torch.arange(n))
        edges = torch.cat([p.global_edges for p in plans]).sort().values
        assert torch.equal(edges, torch.arange(e))
        for p in plans:
            li = p.edge_index[0]
            assert bool((li[1:] >= li[:-1]).all()) and int(li.max()) < p.n_own
            gl = p.local_atoms[p.edge_index]
            assert torch.equal(gl, graph["edge_index"][:, p.global_edges])
            assert torch.equal(p.shifts, graph["shifts"][p.global_edges])
            # every ghost arrives from exactly its owner
            n_recv = sum(int(x.numel()) for x in p.recv_pos)
            assert n_recv == p.n_ghost
        for s in plans:
            for d in plans:
                assert torch.equal(s.owned[s.send_idx[d.rank]], d.ghosts[d.recv_pos[s.rank]])


@pytest.mark.parametrize("world", [2, 4])
def test_domain_decomposition_matches_serial(world):
    graph, params = _structure()
    serial_plan = build_plans(graph["positions"], graph["cell"], graph["edge_index"], graph["shifts"], 1)[0]
    ref = evaluate_domain(_toy_energy(params), graph, serial_plan)
    with tempfile.TemporaryDirectory() as d:
        port = 29600 + world + (os.getpid() % 200)
        mp.start_processes(_worker, args=(world, port, d), nprocs=world, start_method="spawn")
        parts = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    assert all(p["n_ghost"] > 0 for p in parts)
    forces = torch.zeros_like(ref["forces"])
    for p in parts:
        forces[p["owned"]] = p["forces"]
        assert torch.allclose(p["energy"], ref["energy"], rtol=0, atol=1e-10)
        assert torch.allclose(p["stress"], ref["stress"], rtol=0, atol=1e-12)
    assert torch.allclose(forces, ref["forces"], rtol=0, atol=1e-11)
    assert float(ref["forces"].abs().max()) > 1e-3 and float(ref["stress"].abs().max()) > 1e-6


def _abi_halo_worker(rank, world, port, outdir):
    """One rank's ghost exchange through the C ABI (host-emulation build: host pointers):
    fc_halo_pack into the send buffer, all-to-all, fc_halo_unpack into the ghost rows;
    the reverse exchange packs the ghost gradients and adds them into the owners."""
    import abi_calls as A
    from flashcart_b200 import _native, build_ext
    from flashcart_b200.domain import HaloExchange

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lib = _native.bind(build_ext.EMU_LIB)
        graph, _ = _structure()
        plan = build_plans(graph["positions"], graph["cell"], graph["edge_index"], graph["shifts"], world)[rank]
        g = torch.Generator().manual_seed(100 + rank)
        x_own = torch.randn(plan.n_own, 2048, generator=g, dtype=torch.float64)
        send = A.halo_pack(lib, x_own, torch.cat(plan.send_idx))
        recv = torch.empty(plan.n_ghost, 2048, dtype=torch.float64)
        dist.all_to_all_single(recv, send, [int(p.numel()) for p in plan.recv_pos],
                               [int(i.numel()) for i in plan.send_idx])
        ghosts = A.halo_unpack(lib, recv, torch.cat(plan.recv_pos), torch.full_like(recv, float("nan")),
                               accumulate=False)
        leaf = x_own.clone().requires_grad_(True)
        ref = HaloExchange.apply(leaf, plan, None)
        g_ghost = torch.randn(plan.n_ghost, 2048, generator=g, dtype=torch.float64)
        (ref_grad,) = torch.autograd.grad(ref, [leaf], g_ghost)
        back = A.halo_pack(lib, g_ghost, torch.cat(plan.recv_pos))
        recv_b = torch.empty(sum(int(i.numel()) for i in plan.send_idx), 2048, dtype=torch.float64)
        dist.all_to_all_single(recv_b, back, [int(i.numel()) for i in plan.send_idx],
                               [int(p.numel()) for p in plan.recv_pos])
        grad = A.halo_unpack(lib, recv_b, torch.cat(plan.send_idx), torch.zeros_like(x_own), accumulate=True)
        torch.save({"fwd_equal": bool(torch.equal(ghosts, ref.detach())),
                    "bwd_err": float((grad - ref_grad).abs().max()), "n_ghost": plan.n_ghost},
                   os.path.join(outdir, f"h{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_c_abi_halo_exchange_matches_domain_exchange(emu_lib):
    """The C-ABI pack / unpack entry points, composed with a 2-rank gloo all-to-all, give
    the same ghost rows and owner gradients as the operator-level HaloExchange."""
    with tempfile.TemporaryDirectory() as d:
        port = 29900 + (os.getpid() % 200)
        mp.start_processes(_abi_halo_worker, args=(2, port, d), nprocs=2, start_method="spawn")
        parts = [torch.load(os.path.join(d, f"h{r}.pt")) for r in range(2)]
    for p in parts:
        assert p["n_ghost"] > 0 and p["fwd_equal"] and p["bwd_err"] < 1e-12
