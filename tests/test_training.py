"""Data-parallel training step (config 4 at test size): data, routing, gradients, update.

Golden vectors (``tests/golden/make_train_golden.py``) come from the reference model on
4 seeded molecules: teacher labels, the student's loss and every parameter gradient
(through the forces' double backward), the optimizer routing and one optimizer step.
"""

import os
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashcart_b200.training import GradientBuckets, allreduce_gradients, batch_graph, synthetic_molecules

HERE = os.path.dirname(__file__)


@pytest.fixture(scope="module")
def train_golden():
    return torch.load(os.path.join(HERE, "golden", "train_golden.pt"), weights_only=False)


def _student(avg, device="cpu", dtype=torch.float64):
    from flashcart_b200.model.flashcart import FlashCartPotential

    kw = dict(elements=["H", "C", "N", "O"], r_max=5.0, n_hidden_feats=64, l_max_hidden_feats=2, l_max_edge_attrs=2,
              n_radial=8, n_interactions=2, correlation=3, layer_norm=True, nonlinearity=True,
              gate_activation="sigmoid", radial_mapping="cosine", path_reduced_product=False,
              fit_atomic_shifts=False, atomic_shifts=[0.0, 0.0, 0.0, 0.0], avg_neighbors=float(avg))
    torch.manual_seed(0)
    return FlashCartPotential(**kw).to(device=device, dtype=dtype)


def _graph(train_golden, device, dtype=torch.float64):
    g = {k[len("graph/"):]: v for k, v in train_golden.items() if k.startswith("graph/")}
    g = {k: (v.to(device=device, dtype=dtype) if v.is_floating_point() else v.to(device)) for k, v in g.items()}
    g["use_shifts"] = False
    g.pop("pbc", None)
    return g


def _digest_close(ours: torch.Tensor, ref: dict, rtol: float, what: str):
    t = ours.detach().double().flatten().cpu()
    scale = max(float(ref["head"].abs().max()), 1e-30)
    assert t.numel() == ref["numel"], what
    assert float((t[:64] - ref["head"]).abs().max()) <= rtol * scale, what
    assert abs(float(t.sum()) - float(ref["sum"])) <= rtol * max(float(ref["sq"]) ** 0.5 * t.numel() ** 0.5, 1e-30), what
    assert abs(float((t * t).sum()) - float(ref["sq"])) <= rtol * max(float(ref["sq"]), 1e-30), what


def test_synthetic_molecules_follow_the_recipe():
    a = synthetic_molecules(32, rank=1, step=7)
    b = synthetic_molecules(32, rank=1, step=7)
    assert all(np.array_equal(x["positions"], y["positions"]) for x, y in zip(a, b))
    sizes = [len(m["positions"]) for m in a]
    assert min(sizes) >= 20 and max(sizes) <= 60
    types = np.concatenate([m["atom_types"] for m in a])
    assert abs(float((types == 0).mean()) - 0.5) < 0.1
    d = np.linalg.norm(np.diff(a[0]["positions"], axis=0), axis=1)
    assert 0.6 < d.min() and d.max() < 2.0  # 1.1-1.5 A bonds plus N(0, 0.1 A) noise on both ends
    assert not synthetic_molecules(4, rank=0, step=0)[0]["pbc"].any()


def test_graph_matches_reference_batch(train_golden):
    g = batch_graph(synthetic_molecules(4, rank=0, step=0), 5.0, "cpu", dtype=torch.float64)
    for k in ("positions", "atom_types", "edge_index", "batch", "n_atoms"):
        assert torch.equal(g[k], train_golden[f"graph/{k}"]), k


def test_student_init_and_optimizer_routing_match_reference(train_golden):
    from flashcart_b200.training import make_optimizer

    m = _student(float(train_golden["avg_neighbors"]))
    for k, v in m.state_dict().items():
        if v.is_floating_point() and k in train_golden["student/state"]:
            _digest_close(v, train_golden["student/state"][k], 1e-12, k)
    main, aux = make_optimizer(m, lr=1e-2, weight_decay=1e-3)
    names = {id(p): n for n, p in m.named_parameters()}
    muon = [names[id(p)] for o in aux for g in o.param_groups for p in g["params"]]
    no_decay = [names[id(p)] for g in main.param_groups if g["weight_decay"] == 0.0 for p in g["params"]]
    assert sorted(muon) == sorted(train_golden["routing/muon"])
    assert sorted(no_decay) == sorted(train_golden["routing/no_decay"])


def _net():
    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(3, 5), torch.nn.Tanh(), torch.nn.Linear(5, 4), torch.nn.Tanh(),
                              torch.nn.Linear(4, 2))
    net.register_parameter("unused", torch.nn.Parameter(torch.ones(3)))  # receives no gradient
    return net


def _loss(net, rank, step):
    x = torch.arange(6.0).reshape(2, 3) + rank + 0.5 * step
    return net(x).square().sum()


def _dp_worker(rank, world, port, outdir, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        net = _net()
        # tiny buckets: one parameter or two per bucket, started during the backward
        buckets = GradientBuckets(net, bucket_bytes=64) if mode == "buckets" else None
        out = []
        for step in range(2):
            net.zero_grad(set_to_none=True)
            _loss(net, rank, step).backward()
            if buckets is not None:
                buckets.finish()
            else:
                allreduce_gradients(net)
            out.append({k: (p.grad.clone() if p.grad is not None else None) for k, p in net.named_parameters()})
        torch.save(out, os.path.join(outdir, f"g{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["flat", "buckets"])
def test_gradient_allreduce_averages_over_ranks(mode):
    """Gradient averaging over two gloo ranks, flat after the backward and bucketed during
    it (two steps in a row, a parameter without gradient)."""
    with tempfile.TemporaryDirectory() as d:
        port = 29800 + os.getpid() % 100 + (7 if mode == "buckets" else 0)
        mp.start_processes(_dp_worker, args=(2, port, d, mode), nprocs=2, start_method="spawn")
        got = [torch.load(os.path.join(d, f"g{r}.pt")) for r in range(2)]
    for step in range(2):
        ref = {}
        for r in range(2):
            net = _net()
            _loss(net, r, step).backward()
            for k, p in net.named_parameters():
                if p.grad is not None:
                    ref[k] = ref.get(k, 0) + p.grad / 2
        for g in got:
            for k in ref:
                assert torch.allclose(g[step][k], ref[k], atol=1e-6), (mode, step, k)
            if mode == "buckets":
                assert torch.equal(g[step]["unused"], torch.zeros(3))


@pytest.mark.gpu
def test_gpu_training_loss_and_gradients_match_reference(train_golden, cuda_device):
    """float64: loss and every parameter gradient of energy + force MSE (forces with
    create_graph, so the backward runs the double backward of every operator)."""
    from flashcart_b200.training import energy_force_loss

    m = _student(float(train_golden["avg_neighbors"]), cuda_device)
    g = _graph(train_golden, cuda_device)
    loss, _ = energy_force_loss(m, g, train_golden["teacher/energy"].to(cuda_device),
                                train_golden["teacher/forces"].to(cuda_device))
    loss.backward()
    assert abs(float(loss) - float(train_golden["student/loss"])) <= 1e-10 * abs(float(train_golden["student/loss"]))
    for k, p in m.named_parameters():
        _digest_close(p.grad, train_golden["student/grads"][k], 1e-8, k)
    from flashcart_b200.ops import check_device_status
    check_device_status(cuda_device)


@pytest.mark.gpu
def test_gpu_optimizer_step_matches_reference(train_golden, cuda_device):
    """One AdamW + Muon step. AdamW-routed parameters: float64 round-off. Muon-routed ones:
    the Newton-Schulz update runs in bf16, whose rounding the iteration amplifies, so the
    step may differ from the reference's (CPU bf16) by at most twice what torch's own CUDA
    bf16 iteration of the same update differs by (and 0.1% of the update at least)."""
    from oracle import muon_oracle
    from flashcart_b200.training import NS_COEFF, energy_force_loss, make_optimizer

    m = _student(float(train_golden["avg_neighbors"]), cuda_device)
    before = {k: p.detach().clone() for k, p in m.named_parameters()}
    g = _graph(train_golden, cuda_device)
    main, aux = make_optimizer(m, lr=1e-2, weight_decay=1e-3)
    loss, _ = energy_force_loss(m, g, train_golden["teacher/energy"].to(cuda_device),
                                train_golden["teacher/forces"].to(cuda_device))
    loss.backward()
    grads = {k: p.grad.detach().clone() for k, p in m.named_parameters()}
    for o in [main, *aux]:
        o.step()
    muon = set(train_golden["routing/muon"])
    lr, wd, mom = 1e-2, 1e-3, 0.95
    for k, p in m.named_parameters():
        ref = train_golden["student/after_step"][k]
        ref_delta = ref["head"] - before[k].double().flatten()[:64].cpu()
        ours_delta = (p.detach().double() - before[k].double()).flatten()[:64].cpu()
        scale = max(float(ref_delta.abs().max()), 1e-30)
        err = float((ours_delta - ref_delta).abs().max())
        if k not in muon:
            assert err <= 1e-7 * scale, (k, err, scale)
            continue
        upd = grads[k] + mom * ((1 - mom) * grads[k] - grads[k])  # first Nesterov step from a zero buffer
        ns = muon_oracle.newton_schulz(upd[None].float(), NS_COEFF, 5, 1e-7).double()[0]  # torch CUDA bf16
        alr = lr * 0.2 * max(p.shape) ** 0.5
        torch_delta = (-lr * wd * before[k].double() - alr * ns).flatten()[:64].cpu()
        base = float((torch_delta - ref_delta).abs().max())
        assert err <= max(2 * base, 1e-3 * scale), (k, err, base, scale)
