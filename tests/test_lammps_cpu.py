"""LAMMPS ML-IAP interface: host logic (no GPU).

Covers the ML-IAP graph layout (owned atoms first, ghosts after, LAMMPS's rij as edge
vectors), the exchange operators and their autograd (each the other's adjoint), the
device-exchange hook classes on CPU tensors (their torch-indexing host form), the domain
exchange hooks over gloo ranks, and the interface's error paths, checkpoint loading and
serialisation. Model evaluation needs the CUDA kernels: tests/test_gpu_lammps.py.
The ML-IAP stand-in follows the reference's own test double
(tests/calculators/test_lammps.py:19-80): ghosts with an owner map, exchanges as host copies.
"""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashcart_b200 import lammps as L


class HostMLIAPData:
    """ML-IAP data with ghost atoms whose owners are listed in ``ghost_owner``; the
    exchanges are row copies on the host (what LAMMPS's forward / reverse communication
    does across ranks)."""

    def __init__(self, positions, nlocal=None, elems=None):
        positions = np.asarray(positions, dtype=np.float64).reshape(-1, 3)
        self.ntotal = len(positions)
        self.nlocal = self.ntotal if nlocal is None else nlocal
        self.nghosts = self.ntotal - self.nlocal
        self.positions = positions
        self.elems = np.zeros(self.ntotal, np.int32) if elems is None else np.asarray(elems, np.int32)
        self.ghost_owner = {}
        self.set_pairs([], [], np.zeros((0, 3)))
        self.forward_exchange_calls = 0
        self.reverse_exchange_calls = 0

    def set_pairs(self, pair_i, pair_j, rij):
        self.pair_i = np.asarray(pair_i, np.int32)
        self.pair_j = np.asarray(pair_j, np.int32)
        self.rij = np.asarray(rij, np.float64).reshape(-1, 3)
        self.npairs = len(self.pair_i)

    def pairs_within(self, cutoff):
        pi, pj, v = [], [], []
        for i in range(self.ntotal):
            for j in range(self.ntotal):
                d = self.positions[j] - self.positions[i]
                if i != j and np.linalg.norm(d) < cutoff:
                    pi.append(i)
                    pj.append(j)
                    v.append(d)
        self.set_pairs(pi, pj, np.array(v).reshape(-1, 3))

    def forward_exchange(self, feats, out, vec_len):
        self.forward_exchange_calls += 1
        out.copy_(feats)
        for g, o in self.ghost_owner.items():
            out[g].copy_(feats[o])

    def reverse_exchange(self, grads, out, vec_len):
        self.reverse_exchange_calls += 1
        out.copy_(grads)
        for g, o in self.ghost_owner.items():
            out[o].add_(grads[g])
            out[g].zero_()


def _tiny_model(n_interactions=2, r_max=2.0):
    from flashcart_b200.model.flashcart import FlashCartPotential

    return FlashCartPotential(elements=["H", "O"], r_max=r_max, n_hidden_feats=4, l_max_hidden_feats=1,
                              l_max_edge_attrs=2, n_radial=4, n_interactions=n_interactions, correlation=2,
                              hidden_radial=[8], hidden_readout=[8], fit_atomic_shifts=False,
                              atomic_shifts=[0.0, 0.0])


def test_graph_from_mliap_owned_then_ghost_layout():
    fake = HostMLIAPData([[0.0, 0.0, 0.0], [0.8, 0.0, 0.0], [1.7, 0.1, 0.0]], nlocal=2, elems=[0, 1, 1])
    fake.pairs_within(1.5)
    g = L.graph_from_mliap(fake, ["H", "O"], r_max=1.5, device="cpu", dtype=torch.float64)
    assert g["num_nodes"] == 3 and g["nlocal"] == 2 and g["ntotal"] == 3 and g["nghost"] == 1
    assert g["n_atoms"].tolist() == [2] and g["batch"].shape == (2,) and g["atom_types"].shape == (3,)
    assert g["atomic_numbers"].tolist() == [1, 8, 8]
    assert g["edge_index"].shape == (2, fake.npairs) and g["vectors"].shape == (fake.npairs, 3)
    assert torch.equal(g["vectors"], torch.as_tensor(fake.rij)) and g["use_shifts"] is False
    d = L.graph_dict_from_mliap(fake, ["H", "O"], device="cpu", dtype=torch.float32)
    assert d["vectors"].dtype == torch.float32 and d["lammps_exchange"] and "positions" not in d


def test_graph_validation_rejects_out_of_range_indices():
    fake = HostMLIAPData([[0.0, 0.0, 0.0], [0.8, 0.0, 0.0]])
    fake.set_pairs([0, 2], [1, 0], [[0.8, 0, 0], [-0.8, 0, 0]])
    with pytest.raises(ValueError, match="pair_i"):
        L.graph_dict_from_mliap(fake, ["H"], device="cpu", validate=True)
    fake.set_pairs([0, 1], [1, 0], [[0.8, 0, 0], [-0.8, 0, 0]])
    fake.elems = np.array([0, 3], np.int32)
    with pytest.raises(ValueError, match="atom_types"):
        L.graph_dict_from_mliap(fake, ["H", "O"], device="cpu", validate=True)
    empty = HostMLIAPData(np.zeros((0, 3)))
    with pytest.raises(ValueError, match="Empty ML-IAP layout"):
        L.graph_dict_from_mliap(empty, ["H"], device="cpu")


def _owner_map(nlocal, nghost, seed):
    rng = np.random.default_rng(seed)
    return {nlocal + k: int(rng.integers(nlocal)) for k in range(nghost)}


def test_exchange_operators_and_their_adjoints():
    fake = HostMLIAPData(np.zeros((7, 3)), nlocal=4)
    fake.ghost_owner = _owner_map(4, 3, 0)
    x = torch.randn(7, 5, dtype=torch.float64, requires_grad=True)
    y = torch.randn(7, 5, dtype=torch.float64)
    with L.lammps_data_slot(fake):
        fx = torch.ops.flashcart.lammps_forward_exchange(x)
        for g, o in fake.ghost_owner.items():
            assert torch.equal(fx[g], x[o].detach())
        assert torch.equal(fx[:4], x[:4].detach())
        (gx,) = torch.autograd.grad((fx * y).sum(), x)
        ry = torch.ops.flashcart.lammps_reverse_exchange(y)
    # the backward of the forward exchange is the reverse exchange: <F x, y> = <x, R y>
    assert torch.allclose(gx, ry, atol=1e-14)
    assert float((fx.detach() * y).sum()) == pytest.approx(float((x.detach() * ry).sum()), rel=1e-12)
    assert torch.equal(ry[4:], torch.zeros(3, 5, dtype=torch.float64))
    assert fake.forward_exchange_calls == 1 and fake.reverse_exchange_calls == 2


def test_exchange_accepts_noncontiguous_input_and_pads_owned_rows():
    fake = HostMLIAPData(np.zeros((5, 3)), nlocal=3)
    fake.ghost_owner = {3: 0, 4: 2}
    feats = torch.randn(4, 3, dtype=torch.float64).t()
    assert not feats.is_contiguous()
    with L.lammps_data_slot(fake):
        full = L.lammps_exchange_features(feats, nlocal=3, ntotal=5)
        assert torch.equal(full[:3], feats) and torch.equal(full[3], feats[0]) and torch.equal(full[4], feats[2])
        with pytest.raises(RuntimeError, match="expected 3 or 5 rows"):
            L.lammps_exchange_features(torch.zeros(4, 2), nlocal=3, ntotal=5)
    with pytest.raises(RuntimeError, match="lammps_data_slot"):
        torch.ops.flashcart.lammps_forward_exchange(torch.zeros(5, 2))


def test_data_slot_restores_the_previous_object():
    a, b = HostMLIAPData(np.zeros((1, 3))), HostMLIAPData(np.zeros((1, 3)))
    with L.lammps_data_slot(a):
        with L.lammps_data_slot(b):
            assert L._LAMMPS_DATA is b
        assert L._LAMMPS_DATA is a
    assert L._LAMMPS_DATA is None


def test_ghost_image_exchange_equals_host_copies():
    nlocal, nghost = 6, 9
    owner = _owner_map(nlocal, nghost, 4)
    fake = HostMLIAPData(np.zeros((nlocal + nghost, 3)), nlocal=nlocal)
    fake.ghost_owner = owner
    hooks = L.GhostImageExchange(torch.tensor([owner[nlocal + k] for k in range(nghost)]), nlocal)
    x = torch.randn(nlocal + nghost, 7, dtype=torch.float64)
    a, b = torch.empty_like(x), torch.empty_like(x)
    fake.forward_exchange(x, a, 7)
    hooks.forward_exchange(x, b, 7)
    assert torch.equal(a, b)
    fake.reverse_exchange(x, a, 7)
    hooks.reverse_exchange(x, b, 7)
    assert torch.allclose(a, b, atol=1e-14)
    with pytest.raises(ValueError, match="owners"):
        L.GhostImageExchange(torch.tensor([0, 6]), 6)


def _domain_worker(rank, world, port, outdir):
    from flashcart_b200.data import neighbors, synthetic
    from flashcart_b200.domain import build_plans

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = synthetic.config0_water()
        ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
        plans = build_plans(s["positions"], s["cell"], ei, sh, world)
        plan = plans[rank]
        hooks = L.DomainGhostExchange(plan)
        g = torch.Generator().manual_seed(11)
        x_glob = torch.randn(len(s["positions"]), 5, generator=g, dtype=torch.float64)
        y_glob = torch.randn(len(s["positions"]), 5, generator=g, dtype=torch.float64)
        x = x_glob.index_select(0, plan.local_atoms)
        y = torch.randn(plan.n_own + plan.n_ghost, 5, generator=torch.Generator().manual_seed(100 + rank),
                        dtype=torch.float64)
        fx, ry = torch.empty_like(x), torch.empty_like(y)
        hooks.forward_exchange(x.clone(), fx, 5)
        hooks.reverse_exchange(y.clone(), ry, 5)
        data = L.DomainMLIAPData(plan, torch.as_tensor(s["positions"]), s["cell"],
                                 torch.as_tensor(s["atom_types"]))
        rij = data.rij
        v_ref = (torch.as_tensor(s["positions"])[ei[1]] - torch.as_tensor(s["positions"])[ei[0]]
                 + torch.as_tensor(sh, dtype=torch.float64) @ torch.as_tensor(s["cell"], dtype=torch.float64))
        data.f[:] = y_glob.index_select(0, plan.local_atoms)[:, :3]
        folded = data.owned_forces()
        torch.save({"fx": fx, "x": x, "y": y, "ry": ry, "local": plan.local_atoms, "n_own": plan.n_own,
                    "rij_err": float((rij - v_ref[plan.global_edges]).abs().max()), "folded": folded,
                    "owned": plan.owned},
                   os.path.join(outdir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


def test_domain_ghost_exchange_over_gloo_ranks():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        port = 29500 + (os.getpid() % 300)
        mp.start_processes(_domain_worker, args=(world, port, d), nprocs=world, start_method="spawn")
        parts = [torch.load(os.path.join(d, f"r{r}.pt")) for r in range(world)]
    assert all(p["local"].numel() > p["n_own"] for p in parts)  # both ranks hold ghosts
    for p in parts:
        # forward: every row (owned and ghost) holds the global row of its atom
        assert torch.equal(p["fx"], p["x"])
        assert p["rij_err"] < 1e-12
    # reverse exchange is the adjoint of the forward exchange summed over ranks
    lhs = sum(float((p["fx"] * p["y"]).sum()) for p in parts)
    rhs = sum(float((p["x"] * p["ry"]).sum()) for p in parts)
    assert lhs == pytest.approx(rhs, rel=1e-12)
    for p in parts:
        assert torch.equal(p["ry"][p["n_own"]:], torch.zeros_like(p["ry"][p["n_own"]:]))
    # folding f: each atom's rows on every rank add up on its owner
    n = 1 + int(max(int(p["local"].max()) for p in parts))
    total = torch.zeros(n, 3, dtype=torch.float64)
    folded = torch.zeros(n, 3, dtype=torch.float64)
    g = torch.Generator().manual_seed(11)
    torch.randn(n, 5, generator=g, dtype=torch.float64)
    y_glob = torch.randn(n, 5, generator=g, dtype=torch.float64)[:, :3]
    for p in parts:
        total.index_add_(0, p["local"], y_glob.index_select(0, p["local"]))
        folded[p["owned"]] = p["folded"]
    assert torch.allclose(folded, total, atol=1e-12)


def test_unified_interface_settings_and_errors(monkeypatch, capsys):
    model = _tiny_model().double()
    with pytest.raises(ValueError, match="compile_mode"):
        L.FlashCartLAMMPSUnified(model, compile_mode="reduce-overhead")
    unified = L.FlashCartLAMMPSUnified(model, compile_mode="default")
    assert unified.compile_mode == "default" and unified.device == torch.device("cpu")
    assert unified.element_types == ["H", "O"] and unified.rcutfac == 0.5 * unified.r_max
    assert not any(p.requires_grad for p in unified.model.parameters())
    assert unified.dtype == torch.float64
    with pytest.raises(RuntimeError, match="neighbor pairs"):
        unified.compute_forces(HostMLIAPData(np.zeros((0, 3)), nlocal=0))
    lonely = HostMLIAPData([[0.0, 0.0, 0.0], [5.0, 0.0, 0.0]])
    lonely.pairs_within(1.0)
    with pytest.raises(RuntimeError, match="neighbor pairs"):
        unified.compute_forces(lonely)
    # a rank inside LAMMPS exits instead of raising (the other ranks would wait forever)
    unified.interface = object()

    def _exit(status):
        raise SystemExit(status)

    monkeypatch.setattr(L.os, "_exit", _exit)
    with pytest.raises(SystemExit) as exc:
        unified.compute_forces(HostMLIAPData(np.zeros((0, 3)), nlocal=0))
    assert exc.value.code == 1
    assert "owns 0 atoms with 0 neighbor pairs" in capsys.readouterr().err


def test_ghosts_without_exchange_hooks_need_kokkos():
    class NoHooks(HostMLIAPData):
        def __getattribute__(self, name):
            if name in ("forward_exchange", "reverse_exchange"):
                raise AttributeError(name)
            return super().__getattribute__(name)

    unified = L.FlashCartLAMMPSUnified(_tiny_model(n_interactions=2).double())
    data = NoHooks([[0.0, 0.0, 0.0], [0.8, 0.0, 0.0], [1.6, 0.0, 0.0]], nlocal=2)
    data.pairs_within(1.0)
    with pytest.raises(RuntimeError, match="KOKKOS"):
        unified.compute_forces(data)
    assert isinstance(L._exchange_object(data, 3, 3), L._IdentityExchange)


def test_checkpoint_build_and_serialise_roundtrip(tmp_path):
    torch.manual_seed(5)
    model = _tiny_model()
    model.save_inference_checkpoint(tmp_path / "best", meta={"note": "tiny"})
    unified = L.build_lammps_unified(tmp_path / "best")
    assert isinstance(unified, L.FlashCartLAMMPSUnified) and unified.element_types == ["H", "O"]
    for k, v in model.state_dict().items():
        assert torch.equal(unified.model.state_dict()[k], v), k
    out = L.save_lammps_unified(unified, tmp_path / "sub" / "flashcart-mliap.pt")
    loaded = torch.load(out, weights_only=False)
    assert isinstance(loaded, L.FlashCartLAMMPSUnified) and loaded.r_max == model.r_max
