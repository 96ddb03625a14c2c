"""Generate golden vectors of the o3 hot path from the REFERENCE implementation.

Run in a container where the reference source tree is available (it is never
needed at test time)::

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py [<reference>/src]

Every case uses the reference's PyTorch path (``use_triton=False``) in float64 on
seeded inputs and records forward outputs, first derivatives for a random output
cotangent and the second derivative (VJP of the VJP) for random tangents:

* tensor products: the 14 rank <= 3 configurations of the reference's own parity
  tests (``tests/o3/test_tensor_product.py:54-73``; its four l = 4 cases are above the
  compiled rank limit) plus the interaction-layer shape (2,2)->2 with in2_features=1
  and a symmetric shared reduced product, each as a dense product and as an edge
  convolution on the neighbour-list pattern of ``:95-123`` (4 nodes, 8 edges);
* direction tensors ``Irreps(l)`` for l = 0..3 (``tests/o3/test_irreps.py``);
* equivariant linear maps including path-resolved inputs and asymmetric ranks
  (``tests/o3/test_linear.py:34-146``).

Output: ``tests/golden/o3_golden.pt`` (a dict of float64 CPU tensors).
"""

from __future__ import annotations

import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _tp_cases():
    def c(name, l1, l2, lo, f1, f2, sym=False, shared=False, reduce=False):
        return dict(name=name, l1=l1, l2=l2, lo=lo, f1=f1, f2=f2, sym=sym, shared=shared, reduce=reduce)

    return [
        c("l0x0to3_f22", 0, 0, 3, 2, 2),
        c("l3x3to3_f22", 3, 3, 3, 2, 2),
        c("l3x3to3_f12", 3, 3, 3, 1, 2),
        c("l3x3to3_f21", 3, 3, 3, 2, 1),
        c("l3x3to3_f22_shared", 3, 3, 3, 2, 2, shared=True),
        c("l3x3to3_f22_reduce", 3, 3, 3, 2, 2, reduce=True),
        c("l3x3to3_f22_shared_reduce", 3, 3, 3, 2, 2, shared=True, reduce=True),
        c("l3x3to3_f22_sym", 3, 3, 3, 2, 2, sym=True),
        c("l3x3to0_f22_sym_shared", 3, 3, 0, 2, 2, sym=True, shared=True),
        c("l3x3to0_f22_shared", 3, 3, 0, 2, 2, shared=True),
        c("l3x3to2_f22_shared", 3, 3, 2, 2, 2, shared=True),
        c("l0x3to3_f21", 0, 3, 3, 2, 1),
        c("l1x3to3_f21", 1, 3, 3, 2, 1),
        c("l2x3to3_f21", 2, 3, 3, 2, 1),
        c("l2x2to2_f41", 2, 2, 2, 4, 1),
        c("l3x3to3_f33_shared_reduce_sym", 3, 3, 3, 3, 3, sym=True, shared=True, reduce=True),
    ]


def _neighbourlist(n_edges=8, n_neighbors=2):
    n_atoms = max(1, (n_edges + n_neighbors - 1) // n_neighbors)
    dst = torch.arange(n_atoms).repeat_interleave(n_neighbors)[:n_edges]
    src = torch.randint(0, n_atoms - 1, (n_edges,))
    src = src + (src >= dst).to(src.dtype)
    return n_atoms, src, dst


def _second_order(fn, inputs, outputs_cot):
    """(outputs, first grads, second grads) of fn at inputs for random cotangents/tangents."""
    leaves = [t.detach().clone().requires_grad_(True) for t in inputs]
    out = fn(*leaves)
    g = outputs_cot(out)
    grads = torch.autograd.grad(out, leaves, g, create_graph=True, allow_unused=True)
    grads = [torch.zeros_like(l) if gr is None else gr for l, gr in zip(leaves, grads)]
    tangents = [torch.randn_like(gr) for gr in grads]
    g_leaf = g.detach().clone().requires_grad_(True)
    out2 = fn(*leaves)
    grads2 = torch.autograd.grad(out2, leaves, g_leaf, create_graph=True, allow_unused=True)
    s = sum((gr * v).sum() for gr, v in zip(grads2, tangents) if gr is not None)
    second = torch.autograd.grad(s, leaves + [g_leaf], allow_unused=True)
    second = [torch.zeros_like(t) if d is None else d for t, d in zip(leaves + [g_leaf], second)]
    return out.detach(), g, [gr.detach() for gr in grads], tangents, [d.detach() for d in second]


def main(ref_src: str) -> None:
    sys.path.insert(0, ref_src)
    from flashcart import o3  # reference

    torch.set_default_dtype(torch.float64)
    data = {}
    for case in _tp_cases():
        for scatter in (False, True):
            if scatter and case["sym"]:
                continue
            torch.manual_seed(1234)
            tp = o3.TensorProduct(case["l1"], case["l2"], case["lo"], case["f1"], case["f2"],
                                  symmetric_product=case["sym"], shared_weights=case["shared"],
                                  reduce_paths=case["reduce"], use_triton=False)
            F = max(case["f1"], case["f2"])
            if scatter:
                n_atoms, idx_j, idx_i = _neighbourlist()
                in1 = torch.randn(n_atoms, tp.in1_dim)
                in2 = torch.randn(idx_i.numel(), tp.in2_dim)
                rows = idx_i.numel()
            else:
                idx_i = idx_j = None
                in1 = torch.randn(4, tp.in1_dim)
                in2 = in1.clone() if case["sym"] else torch.randn(4, tp.in2_dim)
                rows = 4
            w = torch.randn(tp.n_total_paths * F) if case["shared"] else torch.randn(rows, tp.n_total_paths * F)
            key = f"tp/{case['name']}/{'conv' if scatter else 'dense'}"
            if case["sym"]:
                fn = lambda a, ww: tp(a, a, ww, idx_i, idx_j)  # noqa: E731
                out, g, grads, tan, second = _second_order(fn, [in1, w], torch.randn_like)
            else:
                fn = lambda a, b, ww: tp(a, b, ww, idx_i, idx_j)  # noqa: E731
                out, g, grads, tan, second = _second_order(fn, [in1, in2, w], torch.randn_like)
            data[key + "/in1"] = in1
            data[key + "/in2"] = in2
            data[key + "/w"] = w
            if scatter:
                data[key + "/idx_i"] = idx_i
                data[key + "/idx_j"] = idx_j
            data[key + "/out"] = out
            data[key + "/g"] = g
            for nm, t in zip(("in1", "in2", "w") if not case["sym"] else ("in1", "w"), grads):
                data[key + f"/grad_{nm}"] = t
            for nm, t in zip(("in1", "in2", "w") if not case["sym"] else ("in1", "w"), tan):
                data[key + f"/tan_{nm}"] = t
            names = (("in1", "in2", "w") if not case["sym"] else ("in1", "w")) + ("g",)
            for nm, t in zip(names, second):
                data[key + f"/dd_{nm}"] = t
            data[key + "/meta"] = torch.tensor([case["l1"], case["l2"], case["lo"], case["f1"], case["f2"],
                                                int(case["sym"]), int(case["shared"]), int(case["reduce"]),
                                                int(scatter)])
    for l in range(4):
        torch.manual_seed(100 + l)
        x = torch.nn.functional.normalize(torch.randn(16, 3), dim=-1)
        ir = o3.Irreps(l, use_triton=False)
        out, g, grads, tan, second = _second_order(lambda a: ir.forward_normalized(a) + 0.0 * a.sum(), [x],
                                                   torch.randn_like)
        key = f"irreps/l{l}"
        data[key + "/x"] = x
        data[key + "/out"] = out
        data[key + "/g"] = g
        data[key + "/grad_x"] = grads[0]
        data[key + "/tan_x"] = tan[0]
        data[key + "/dd_x"] = second[0]
        data[key + "/dd_g"] = second[1]
    lin_cases = [
        ("l3to3_f4to5", 3, 3, 4, 5, None, None),
        ("l3to2_paths", 3, 2, 4, 5, [1, 2, 3, 2], None),
        ("l1to3_f3to2", 1, 3, 3, 2, None, None),
        ("l2to2_f8_scale1", 2, 2, 8, 8, None, 1.0),
    ]
    for name, li, lo, fi, fo, paths, ws in lin_cases:
        torch.manual_seed(7)
        lin = o3.LinearLayer(li, lo, fi, fo, in_paths=paths, weight_scale=ws, use_triton=False)
        x = torch.randn(6, lin.in_dim)
        ws_t = [w.detach().clone() for w in lin.weight]

        def fn(xx, *wts, _lin=lin):
            from flashcart.o3._linear import py_linear
            return py_linear(xx, list(wts), _lin.in_l_max, _lin.out_l_max, _lin.in_features, _lin.out_features,
                             in_paths=_lin.in_paths, scale=_lin.scale)

        out, g, grads, tan, second = _second_order(fn, [x, *ws_t], torch.randn_like)
        key = f"linear/{name}"
        data[key + "/x"] = x
        for l, w in enumerate(ws_t):
            data[key + f"/w{l}"] = w
            data[key + f"/grad_w{l}"] = grads[1 + l]
            data[key + f"/tan_w{l}"] = tan[1 + l]
            data[key + f"/dd_w{l}"] = second[1 + l]
        data[key + "/out"] = out
        data[key + "/g"] = g
        data[key + "/grad_x"] = grads[0]
        data[key + "/tan_x"] = tan[0]
        data[key + "/dd_x"] = second[0]
        data[key + "/dd_g"] = second[-1]
        data[key + "/meta"] = torch.tensor([li, lo, fi, fo, -1 if ws is None else 1] + (paths or [1] * (li + 1)))
    torch.save(data, os.path.join(HERE, "o3_golden.pt"))
    print(f"wrote {len(data)} tensors to {os.path.join(HERE, 'o3_golden.pt')}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FLASHCART_REFERENCE_SRC", ""))
