"""Pin the CPU oracle against golden vectors produced by the reference itself.

The golden file holds forward outputs, first derivatives and second derivatives of
the reference's PyTorch path (``tests/golden/make_golden.py``); the oracle must
reproduce all of them in float64 before anything is checked against it.
"""

import pytest
import torch

from oracle import stf_oracle as O

TOL = 1e-10


def _tp_keys(golden):
    return sorted({k.rsplit("/", 1)[0] for k in golden if k.startswith("tp/")})


def _second_order(fn, leaves, g, tangents):
    leaves = [t.detach().clone().requires_grad_(True) for t in leaves]
    g_leaf = g.detach().clone().requires_grad_(True)
    out = fn(*leaves)
    grads = torch.autograd.grad(out, leaves, g_leaf, create_graph=True, allow_unused=True)
    s = sum((gr * v).sum() for gr, v in zip(grads, tangents) if gr is not None)
    second = torch.autograd.grad(s, leaves + [g_leaf], allow_unused=True)
    second = [torch.zeros_like(t) if d is None else d for t, d in zip(leaves + [g_leaf], second)]
    grads = [torch.zeros_like(l) if gr is None else gr for l, gr in zip(leaves, grads)]
    return out.detach(), [x.detach() for x in grads], second


def test_golden_file_covers_all_parts(golden):
    keys = _tp_keys(golden)
    assert len(keys) >= 28
    assert any(k.endswith("/conv") for k in keys)
    assert all(f"irreps/l{l}/out" in golden for l in range(4))
    assert any(k.startswith("linear/") for k in golden)


@pytest.mark.parametrize("l", range(4))
def test_oracle_irreps_matches_reference(golden, l):
    k = f"irreps/l{l}"
    fn = lambda a: O.irreps(a, l) + 0.0 * a.sum()  # noqa: E731
    out, grads, second = _second_order(fn, [golden[k + "/x"]], golden[k + "/g"], [golden[k + "/tan_x"]])
    assert (out - golden[k + "/out"]).abs().max() < TOL
    assert (grads[0] - golden[k + "/grad_x"]).abs().max() < TOL
    assert (second[0] - golden[k + "/dd_x"]).abs().max() < TOL
    assert (second[1] - golden[k + "/dd_g"]).abs().max() < TOL


def test_oracle_tensor_products_match_reference(golden):
    for key in _tp_keys(golden):
        m = [int(v) for v in golden[key + "/meta"]]
        l1, l2, lo, f1, f2, sym, shared, red, conv = m
        idx_i = golden.get(key + "/idx_i")
        idx_j = golden.get(key + "/idx_j")
        names = ("in1", "w") if sym else ("in1", "in2", "w")
        leaves = [golden[f"{key}/{n}"] for n in names]
        tangents = [golden[f"{key}/tan_{n}"] for n in names]
        if sym:
            fn = lambda a, w: O.tensor_product(a, a, w, idx_i, idx_j, l1, l2, lo, f1, f2, True, shared, red)  # noqa
        else:
            fn = lambda a, b, w: O.tensor_product(a, b, w, idx_i, idx_j, l1, l2, lo, f1, f2, False, shared, red)  # noqa
        out, grads, second = _second_order(fn, leaves, golden[key + "/g"], tangents)
        assert (out - golden[key + "/out"]).abs().max() < TOL, key
        for n, gr in zip(names, grads):
            assert (gr - golden[f"{key}/grad_{n}"]).abs().max() < TOL, (key, n)
        for n, d in zip(names + ("g",), second):
            assert (d - golden[f"{key}/dd_{n}"]).abs().max() < TOL, (key, "dd", n)


def test_oracle_linear_matches_reference(golden):
    names = sorted({k.split("/")[1] for k in golden if k.startswith("linear/")})
    for name in names:
        k = f"linear/{name}"
        meta = [int(v) for v in golden[k + "/meta"]]
        li, lo, fi, fo, has_ws = meta[:5]
        paths = meta[5:]
        common = min(li, lo)
        ws = [golden[f"{k}/w{l}"] for l in range(common + 1)]
        scale = 1.0 if has_ws == 1 else None
        fn = lambda x, *w: O.linear(x, list(w), li, lo, fi, fo, paths, scale)  # noqa: E731
        tangents = [golden[k + "/tan_x"]] + [golden[f"{k}/tan_w{l}"] for l in range(common + 1)]
        out, grads, second = _second_order(fn, [golden[k + "/x"], *ws], golden[k + "/g"], tangents)
        assert (out - golden[k + "/out"]).abs().max() < TOL, name
        assert (grads[0] - golden[k + "/grad_x"]).abs().max() < TOL, name
        for l in range(common + 1):
            assert (grads[1 + l] - golden[f"{k}/grad_w{l}"]).abs().max() < TOL, (name, l)
            assert (second[1 + l] - golden[f"{k}/dd_w{l}"]).abs().max() < TOL, (name, l)
        assert (second[0] - golden[k + "/dd_x"]).abs().max() < TOL, name
        assert (second[-1] - golden[k + "/dd_g"]).abs().max() < TOL, name
