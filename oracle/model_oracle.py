"""CPU oracle of the FlashCart potential -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py`` may use
it (as the checker and as the timed CPU reference). A functional restatement of the
reference forward pass (``model/flashcart.py:223-317``, ``nn/layers.py``,
``nn/radial.py``) on the oracle's full-Cartesian operators, reading parameters by the
reference's state_dict keys; forces and stress come from autograd with the symmetric
virtual strain of ``model/atomistic.py:158-340``.
"""

from __future__ import annotations

import math
from typing import Dict, List

import torch
import torch.nn.functional as F

from oracle import stf_oracle as O



def _c(v: float) -> float:
    """A constant as the reference holds it: a buffer created under the float32 default
    dtype (scales of linear layers and activations), then widened with the module."""
    return float(torch.tensor(v, dtype=torch.float32))


SILU_SCALE = _c(1.6765324703310907)
SIGMOID_SCALE = _c(1.8462285453386054)


def _dense(x, w, bias=None):
    return F.linear(x, w * _c(w.shape[1] ** -0.5), bias)


def _mlp(x, sd, prefix, n_layers):
    for k in range(n_layers):
        x = _dense(x, sd[f"{prefix}.{2 * k}.weight"])
        if k < n_layers - 1:
            x = SILU_SCALE * F.silu(x)
    return x


def _o3_linear(x, sd, prefix, in_l, out_l, fin, fout, in_paths=None):
    common = min(in_l, out_l)
    ws = [sd[f"{prefix}.weight.{l}"] for l in range(common + 1)]
    scales = [_c(s) for s in O.linear_scales(in_l, out_l, fin, in_paths)]
    return O.linear(x, ws, in_l, out_l, fin, fout, in_paths, scales=scales)


def _paths(l1, l2, lo, sym=False):
    per = [0] * (lo + 1)
    for a, b, o, _ in O.enumerate_paths(l1, l2, lo, sym):
        per[o] += 1
    return per, sum(per)


def _rms_norm(x, sd, prefix, l_max, C, eps=1.0e-6):
    n = x.shape[0]
    _, npaths = _paths(l_max, l_max, 0, True)
    ones = torch.ones(npaths * C, dtype=x.dtype)
    inv = O.tensor_product(x, x, ones, None, None, l_max, l_max, 0, C, C, True, True, False).view(n, l_max + 1, C)
    lw = torch.tensor([1.0 / ((2 * l + 1) * (l_max + 1)) for l in range(l_max + 1)], dtype=torch.float64)
    mean_sq = (inv * lw.to(inv.dtype).view(1, -1, 1)).sum(1).mean(-1, keepdim=True)
    scaled = x * torch.pow(mean_sq + eps, -0.5)
    gains = torch.cat([sd[f"{prefix}.weights.{l}"].repeat(2 * l + 1) for l in range(l_max + 1)])
    return scaled * gains


def _chebyshev(d, n_radial, r_max, mapping):
    t = d / r_max
    x = torch.cos(t * math.pi) if mapping == "cosine" else 2.0 * t - 1.0
    terms = [torch.ones_like(x), x]
    for _ in range(2, n_radial):
        terms.append(2.0 * x * terms[-1] - terms[-2])
    return torch.stack(terms[:n_radial], -1)


def _cutoff(d, r_max, p):
    d = torch.clamp(d, min=0.0)
    t = d / r_max
    tp = t ** p
    env = 1.0 - (p + 1.0) * (p + 2.0) / 2.0 * tp + p * (p + 2.0) * tp * t - p * (p + 1.0) / 2.0 * tp * t * t
    return torch.clamp(env * (d < r_max).to(env.dtype), 0.0, 1.0)


def node_energies(sd: Dict[str, torch.Tensor], cfg: Dict, graph: Dict[str, torch.Tensor]) -> torch.Tensor:
    """Site energies of one graph for the path-resolved, element-agnostic architecture."""
    C = cfg["n_hidden_feats"]
    Lh = cfg["l_max_hidden_feats"]
    Le = cfg["l_max_edge_attrs"]
    n_int = cfg["n_interactions"]
    corr = cfg["correlation"]
    assert cfg.get("path_reduced_product", True) is False and cfg.get("element_agnostic_interaction", True)
    ei = graph["edge_index"]
    idx_i, idx_j = ei[0], ei[1]
    pos, cell = graph["positions"], graph["cell"]
    batch = graph["batch"]
    vec = pos[idx_j] - pos[idx_i] + (graph["shifts"].to(cell.dtype).unsqueeze(-2) @ cell[batch[idx_i]]).squeeze(-2)
    dist = vec.norm(dim=-1)
    direc = vec / dist.clamp_min(1.0e-4).unsqueeze(-1)
    edge_attrs = O.irreps(direc, Le)
    edge_feats = _chebyshev(dist, cfg["n_radial"], cfg["r_max"], cfg["radial_mapping"])
    env = _cutoff(dist, cfg["r_max"], cfg.get("cutoff_poly_order", 6))
    feats = sd["embedding.weight"][graph["atom_types"]]
    outs: List[torch.Tensor] = []
    n_mlp = len(cfg.get("hidden_radial", [64, 64])) + 1
    for k in range(n_int):
        p = f"interactions.{k}"
        lin = 0 if k == 0 else Lh
        lout = Le
        out_paths, _ = _paths(lin, Le, lout)
        residual = feats
        h = _o3_linear(feats, sd, f"{p}.linear_first", lin, lin, C, C)
        w = _mlp(edge_feats * env.unsqueeze(-1), sd, f"{p}.radial_mlp", n_mlp)
        agg = O.tensor_product(h, edge_attrs, w, idx_i, idx_j, lin, Le, lout, C, 1)
        agg = agg / sd[f"{p}.sqrt_avg_neighbors"]
        x = _o3_linear(agg, sd, f"{p}.linear_second", lout, lout, C, C, out_paths)
        if lin == 0:
            skip = _dense(residual, sd[f"{p}.skip_projection.weight"])
            x = torch.cat([x[:, :C] + skip, x[:, C:]], -1)
        else:
            x = x + _o3_linear(residual, sd, f"{p}.skip_projection", lin, lout, C, C)
        if cfg.get("layer_norm", False):
            x = _rms_norm(x, sd, f"{p}.layer_norm", lout, C)
        if cfg.get("nonlinearity", False):
            q = f"nonlinearities.{k}"
            vals = _o3_linear(x, sd, f"{q}.value_linear", lout, lout, C, C)
            act = cfg.get("gate_activation", "silu")
            gl = _dense(x[:, :C], sd[f"{q}.gate_linear.weight"], sd.get(f"{q}.gate_linear.bias"))
            gates = SIGMOID_SCALE * torch.sigmoid(gl) if act == "sigmoid" else SILU_SCALE * F.silu(gl)
            gates = gates.view(-1, lout + 1, C)
            parts = []
            off = 0
            for l in range(lout + 1):
                blk = vals[:, off:off + (2 * l + 1) * C].view(-1, 2 * l + 1, C)
                off += (2 * l + 1) * C
                parts.append((blk * gates[:, l].unsqueeze(1)).flatten(1))
            x = x + _o3_linear(torch.cat(parts, -1), sd, f"{q}.output_linear", lout, lout, C, C)
        # product layer
        q = f"products.{k}"
        p_out = Lh if k < n_int - 1 else 0
        out = x.new_zeros(x.shape[0], (p_out + 1) ** 2 * C)
        prod = x
        for step in range(corr):
            s_out = p_out if step == corr - 1 else Le
            if step > 0:
                ppl, ptot = _paths(Le, Le, s_out)
                ones = torch.ones(ptot * C, dtype=x.dtype)
                prod = O.tensor_product(prod, x, ones, None, None, Le, Le, s_out, C, C, False, True, False)
                paths_in = ppl
            else:
                paths_in, _ = _paths(Le, 0, s_out)
            lin_out = s_out if step < corr - 1 else p_out
            prod = _o3_linear(prod, sd, f"{q}.product_linears.{step}", s_out, lin_out, C, C, paths_in)
            out = out + prod[:, :(p_out + 1) ** 2 * C]
        out = out + _o3_linear(x, sd, f"{q}.skip_projection", Le, p_out, C, C)
        if cfg.get("layer_norm", False):
            out = _rms_norm(out, sd, f"{q}.layer_norm", p_out, C)
        feats = out
        outs.append(feats[:, :C])
    e = _mlp(torch.cat(outs, 1), sd, "readout.readout_mlp", len(cfg.get("hidden_readout", [64, 64])) + 1)
    return sd["scale_shift.scales"][graph["atom_types"]] * e.squeeze(-1)


def predict(sd, cfg, graph, compute_forces=True, compute_stress=True):
    """Energies, forces and Voigt stress of one periodic graph (CPU autograd)."""
    pos = graph["positions"].detach()
    cell = graph["cell"].detach()
    disp = torch.zeros_like(cell).requires_grad_(True)
    sym = 0.5 * (disp + disp.transpose(-1, -2))
    scaling = torch.eye(3, dtype=cell.dtype).unsqueeze(0) + sym
    pos = (pos.unsqueeze(-2) @ scaling[graph["batch"]]).squeeze(-2)
    cell = cell @ scaling
    pos.requires_grad_(True)
    g = dict(graph, positions=pos, cell=cell)
    e_node = node_energies(sd, cfg, g)
    energy = torch.zeros(int(graph["batch"].max()) + 1, dtype=e_node.dtype).index_add(0, graph["batch"], e_node)
    dR, dD = torch.autograd.grad(energy.sum(), [pos, disp])
    vol = torch.det(cell)
    st = dD / vol.view(-1, 1, 1)
    stress = torch.stack([st[..., 0, 0], st[..., 1, 1], st[..., 2, 2], (st[..., 1, 2] + st[..., 2, 1]) / 2,
                          (st[..., 0, 2] + st[..., 2, 0]) / 2, (st[..., 0, 1] + st[..., 1, 0]) / 2], -1)
    return {"energy": energy.detach(), "node_energies": e_node.detach(), "forces": -dR, "stress": stress}
