"""Data-parallel training step of the potential (energy + force loss, Muon).

* ``synthetic_molecules``: the seeded random-walk molecules of the DP training
  benchmark (20-60 atoms, elements H/C/N/O drawn 50/30/10/10, bonds U(1.1, 1.5) A along
  isotropic random directions plus N(0, 0.1 A) noise, non-periodic; seed
  ``1000 * rank + step``).
* ``batch_graph``: one graph dict for a list of molecules (brute-force neighbour lists
  per molecule, canonical order, receivers ascending).
* ``energy_force_loss``: energy MSE per atom + force MSE, forces from ``predict`` with
  ``create_graph=True`` so that the loss backward runs the operators' double backward.
* ``HybridMuon`` / ``make_optimizer``: the reference's optimizer routing
  (``training/optimizers.py:7-118``): trainable 2-D parameters not reported by the
  ``non_muon_parameters`` hooks go to Muon (momentum, Nesterov, batched Newton-Schulz
  per shape bucket on the tensor cores via ``flashcart::newton_schulz``, match-RMS
  learning-rate scaling, decoupled weight decay), the rest to AdamW.
* ``allreduce_gradients``: one flat NCCL all-reduce of all gradients, averaged over
  ranks (data parallel over molecules: each rank owns whole structures).
"""

from __future__ import annotations

import math
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.distributed as dist
import torch.nn as nn

ELEMENTS = ["H", "C", "N", "O"]
ELEMENT_P = [0.5, 0.3, 0.1, 0.1]
NS_COEFF = (3.4445, -4.7750, 2.0315)
NS_POLISH = (2.0, -1.5, 0.5)


def synthetic_molecules(n_mol: int, rank: int = 0, step: int = 0, box: float = 100.0) -> List[Dict[str, np.ndarray]]:
    rng = np.random.default_rng(1000 * rank + step)
    mols = []
    for _ in range(n_mol):
        n = int(rng.integers(20, 61))
        types = rng.choice(len(ELEMENTS), size=n, p=ELEMENT_P).astype(np.int64)
        d = rng.normal(size=(n - 1, 3))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        steps = d * rng.uniform(1.1, 1.5, size=(n - 1, 1))
        pos = np.concatenate([np.zeros((1, 3)), np.cumsum(steps, axis=0)], axis=0)
        pos += rng.normal(scale=0.1, size=pos.shape)
        pos += box / 2 - pos.mean(axis=0)
        mols.append({"positions": pos, "atom_types": types, "cell": np.eye(3) * box,
                     "pbc": np.array([False, False, False])})
    return mols


def batch_graph(mols: Sequence[Dict[str, np.ndarray]], r_max: float, device, dtype=torch.float32) -> Dict:
    from flashcart_b200.data.neighbors import neighbor_list_bruteforce

    pos, types, ei, sh, batch, cells = [], [], [], [], [], []
    off = 0
    for g, m in enumerate(mols):
        e, s = neighbor_list_bruteforce(m["positions"], m["cell"], m["pbc"], r_max)
        pos.append(m["positions"])
        types.append(m["atom_types"])
        ei.append(e + off)
        sh.append(s)
        batch.append(np.full(len(m["positions"]), g))
        cells.append(m["cell"])
        off += len(m["positions"])
    t = lambda a, dt: torch.as_tensor(np.concatenate(a) if isinstance(a, list) else a, dtype=dt, device=device)
    return {"positions": t(pos, dtype), "atom_types": t(types, torch.long),
            "edge_index": torch.as_tensor(np.concatenate(ei, axis=1), dtype=torch.long, device=device),
            "shifts": t(sh, dtype), "batch": t(batch, torch.long),
            "cell": torch.as_tensor(np.stack(cells), dtype=dtype, device=device),
            "n_atoms": torch.as_tensor([len(m["positions"]) for m in mols], dtype=torch.long, device=device),
            "use_shifts": False}


def energy_force_loss(model, graph: Dict, energy_label: torch.Tensor, forces_label: torch.Tensor,
                      energy_weight: float = 1.0, force_weight: float = 1.0) -> Tuple[torch.Tensor, Dict]:
    out = model.predict(graph, compute_forces=True, create_graph=True)
    n = graph["n_atoms"].to(out["energy"].dtype)
    e_loss = (((out["energy"] - energy_label) / n) ** 2).mean()
    f_loss = ((out["forces"] - forces_label) ** 2).mean()
    return energy_weight * e_loss + force_weight * f_loss, out


class HybridMuon(torch.optim.Optimizer):
    """Muon with batched Newton-Schulz per shape bucket (reference ``training/muon.py:100-330``
    without alignment damping): ``buf = lerp(buf, grad, 1 - momentum)``, update =
    ``lerp(grad, buf, momentum)`` (Nesterov) or ``buf``, orthogonalised in bf16, cast to
    the parameter dtype and applied with ``lr * ns_rms_scale * sqrt(max(rows, cols))``
    (``adjust_lr_fn="match_rms_adamw"``); weight decay multiplies the parameters by
    ``1 - lr * weight_decay`` first."""

    def __init__(self, params: Iterable, lr: float = 1e-3, weight_decay: float = 0.1, momentum: float = 0.95,
                 nesterov: bool = True, ns_coefficients: Tuple[float, float, float] = NS_COEFF, eps: float = 1e-7,
                 ns_steps: int = 5, adjust_lr_fn: Optional[str] = None, ns_polish_steps: int = 0,
                 ns_polish_coefficients: Tuple[float, float, float] = NS_POLISH, ns_rms_scale: float = 0.2):
        params = [p[1] if isinstance(p, tuple) else p for p in params]
        for p in params:
            if p.ndim != 2:
                raise ValueError(f"Muon only supports 2D parameters, got shape {tuple(p.shape)}")
        defaults = dict(lr=lr, weight_decay=weight_decay, momentum=momentum, nesterov=nesterov,
                        ns_coefficients=ns_coefficients, eps=eps, ns_steps=ns_steps, adjust_lr_fn=adjust_lr_fn,
                        ns_polish_steps=ns_polish_steps, ns_polish_coefficients=ns_polish_coefficients,
                        ns_rms_scale=ns_rms_scale)
        super().__init__(params, defaults)

    @staticmethod
    def _adjust_lr(lr: float, fn: Optional[str], shape, rms_scale: float) -> float:
        a, b = shape[:2]
        if fn is None or fn == "original":
            return lr * math.sqrt(max(1, a / b))
        if fn == "match_rms_adamw":
            return lr * rms_scale * math.sqrt(max(a, b))
        return lr

    @torch.no_grad()
    def step(self, closure=None):
        from flashcart_b200 import ops  # noqa: F401  (registers flashcart::newton_schulz)

        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        for group in self.param_groups:
            lr, wd, mom = group["lr"], group["weight_decay"], group["momentum"]
            live = [p for p in group["params"] if p.grad is not None]
            if wd != 0.0 and live:
                torch._foreach_mul_(live, 1 - lr * wd)
            buckets: Dict[tuple, List[torch.Tensor]] = {}
            for p in live:
                buckets.setdefault((tuple(p.shape), p.device, p.dtype), []).append(p)
            for (shape, _, dtype), ps in buckets.items():
                grads = torch.stack([p.grad for p in ps])
                bufs = []
                for p in ps:
                    st = self.state[p]
                    if "momentum_buffer" not in st:
                        st["momentum_buffer"] = torch.zeros_like(p.grad)
                    bufs.append(st["momentum_buffer"])
                buf = torch.stack(bufs)
                buf.lerp_(grads, 1 - mom)
                torch._foreach_copy_(bufs, list(buf.unbind(0)))
                upd = torch.lerp(grads, buf, mom) if group["nesterov"] else buf
                upd = torch.ops.flashcart.newton_schulz(
                    upd.float().contiguous(), list(group["ns_coefficients"]), int(group["ns_steps"]),
                    list(group["ns_polish_coefficients"]), int(group["ns_polish_steps"]), float(group["eps"]))
                alr = self._adjust_lr(lr, group["adjust_lr_fn"], shape, group["ns_rms_scale"])
                torch._foreach_add_(ps, list(upd.to(dtype).unbind(0)), alpha=-alr)
        return loss


def make_optimizer(model: nn.Module, lr: float = 1e-2, weight_decay: float = 1e-3, ns_steps: int = 5,
                   ns_polish_steps: int = 0, ns_rms_scale: float = 0.2):
    """(AdamW main optimizer, [HybridMuon]) as the reference's ``make_optimizer(optimizer="muon")``."""
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    non_muon = {id(p) for p in model.non_muon_parameters()} if hasattr(model, "non_muon_parameters") else set()
    non_decay = ({id(p) for p in model.non_decayable_parameters()}
                 if hasattr(model, "non_decayable_parameters") else set())
    muon = [(n, p) for n, p in named if id(p) not in non_muon and p.ndim == 2]
    adam = [p for _, p in named if id(p) in non_muon or p.ndim != 2]
    aux = [HybridMuon(muon, lr=lr, weight_decay=weight_decay, ns_steps=ns_steps, ns_polish_steps=ns_polish_steps,
                      ns_rms_scale=ns_rms_scale, adjust_lr_fn="match_rms_adamw")] if muon else []
    main = torch.optim.AdamW([{"params": [p for p in adam if id(p) not in non_decay], "weight_decay": weight_decay},
                              {"params": [p for p in adam if id(p) in non_decay], "weight_decay": 0.0}], lr=lr)
    return main, aux


class GradientBuckets:
    """Bucketed gradient averaging overlapped with the backward pass (the DDP scheme that
    Lightning Fabric applies in ``fabric.backward``, reference ``training/tasks.py:444``).

    Parameters are grouped, in reverse registration order (the order in which their
    gradients tend to become ready), into buckets of about ``bucket_bytes``. A hook after
    each parameter's gradient accumulation copies the gradient into its bucket's flat
    buffer; a full bucket starts its all-reduce asynchronously while the backward goes on.
    Buckets start strictly in index order, so every rank issues the same collectives in the
    same order whatever the order in which its gradients complete. :meth:`finish` (after
    ``backward``) starts the buckets that are still pending (a parameter without gradient
    counts as zeros), waits for all of them, averages and writes the gradients back.
    CUDA tensors on a gloo group are staged through host memory (synchronously).
    """

    def __init__(self, model: nn.Module, group=None, bucket_bytes: int = 4 << 20):
        self.group = group
        self.world = dist.get_world_size(group)
        params = [p for p in model.parameters() if p.requires_grad]
        self.buckets: List[List[nn.Parameter]] = []
        cur, size = [], 0
        for p in reversed(params):
            cur.append(p)
            size += p.numel() * p.element_size()
            if size >= bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self.where = {id(p): b for b, ps in enumerate(self.buckets) for p in ps}
        self._hooks = [p.register_post_accumulate_grad_hook(self._ready) for p in params]
        self._reset()

    def _reset(self) -> None:
        self.pending = [len(ps) for ps in self.buckets]
        self.flat: List[Optional[torch.Tensor]] = [None] * len(self.buckets)
        self.handles: List[Optional[object]] = [None] * len(self.buckets)
        self.next = 0

    def _fill(self, b: int) -> torch.Tensor:
        ps = self.buckets[b]
        ref = ps[0]
        flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1) for p in ps])
        return flat.to(ref.dtype)

    def _launch_ready(self, force: bool = False) -> None:
        while self.next < len(self.buckets) and (force or self.pending[self.next] == 0):
            b = self.next
            flat = self._fill(b)
            if flat.is_cuda and dist.get_backend(self.group) == "gloo":
                host = flat.cpu()
                dist.all_reduce(host, group=self.group)
                flat.copy_(host)
                self.handles[b] = None
            else:
                self.handles[b] = dist.all_reduce(flat, group=self.group, async_op=True)
            self.flat[b] = flat
            self.next += 1

    def _ready(self, p: torch.Tensor) -> None:
        b = self.where[id(p)]
        self.pending[b] -= 1
        if self.world > 1:
            self._launch_ready()

    def finish(self) -> None:
        if self.world > 1:
            self._launch_ready(force=True)
            for b, ps in enumerate(self.buckets):
                if self.handles[b] is not None:
                    self.handles[b].wait()
                flat = self.flat[b] / self.world
                off = 0
                for p in ps:
                    n = p.numel()
                    if p.grad is not None:
                        p.grad.copy_(flat[off:off + n].view_as(p))
                    else:
                        p.grad = flat[off:off + n].view_as(p).clone()
                    off += n
        self._reset()

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()


def allreduce_gradients(model: nn.Module, group=None) -> None:
    """Average the gradients over the ranks with one flat all-reduce (after the backward;
    :class:`GradientBuckets` overlaps the same averaging with the backward)."""
    world = dist.get_world_size(group)
    if world == 1:
        return
    grads = [p.grad for p in model.parameters() if p.grad is not None]
    if not grads:
        return
    flat = torch.cat([g.reshape(-1) for g in grads])
    if flat.is_cuda and dist.get_backend(group) == "gloo":
        host = flat.cpu()
        dist.all_reduce(host, group=group)
        flat.copy_(host)
    else:
        dist.all_reduce(flat, group=group)
    flat /= world
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


def train_step(model, graph, energy_label, forces_label, optimizers, group=None,
               buckets: Optional[GradientBuckets] = None) -> torch.Tensor:
    """Loss, backward (double backward through the forces), gradient all-reduce (bucketed
    and overlapped with the backward when ``buckets`` is given), updates."""
    main, aux = optimizers
    for opt in [main, *aux]:
        opt.zero_grad(set_to_none=True)
    loss, _ = energy_force_loss(model, graph, energy_label, forces_label)
    loss.backward()
    if buckets is not None:
        buckets.finish()
    elif dist.is_available() and dist.is_initialized():
        allreduce_gradients(model, group)
    for opt in [main, *aux]:
        opt.step()
    return loss.detach()
