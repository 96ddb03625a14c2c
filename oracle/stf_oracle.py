"""CPU oracle of the FlashCart o3 hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` may import this module, and only as the checker / the timed CPU
reference. The product (``flashcart_b200``) never imports it.

A plain restatement in PyTorch (CPU, any float dtype; float64 for parity) of the
reference's arithmetic, written on FULL Cartesian tensors so it shares no code path
with the product's generated kernels (which use exact stored-component tables):

* stored <-> full STF components: reference ``o3/_codegen_common.py:37-73`` (order)
  and ``o3/_codegen_tensor_product.py:233-271`` (tracelessness recursion);
* one tensor-product path ``N * STF_lo(Sym(contract_k(T1 (x) T2)))`` with the
  explicit trace-removal series ``c_k(L)`` and normalisation ``N``: reference
  ``o3/_codegen_tensor_product.py:7-58, 103-142, 296-414``;
* the weighted product, path order, feature broadcast, gather / scatter_sum of the
  convolution: reference ``o3/_codegen_tensor_product.py:833-1012`` and
  ``o3/utils.py:127-203``;
* direction tensors ``T^l(x)`` (Eq. (1)) with constant Kronecker deltas:
  reference ``o3/_codegen_irreps.py:1-32, 148-164``;
* equivariant linear map: reference ``o3/_linear.py:64-110, 113-166``.

Backward and double backward of every op come from torch.autograd on these
expressions (the reference derives them symbolically from the same forward).
Pinned against golden vectors produced by the reference itself
(``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import itertools
import math
from functools import lru_cache
from typing import List, Optional, Sequence, Tuple

import torch


def double_factorial(n: int) -> int:
    out = 1
    while n > 1:
        out *= n
        n -= 2
    return out


def stored_basis(l: int) -> List[Tuple[int, int, int]]:
    """Reference ``o3/_codegen_common.py:37-73``."""
    if l == 0:
        return [(0, 0, 0)]
    if l == 1:
        return [(1, 0, 0), (0, 1, 0), (0, 0, 1)]
    if l == 2:
        return [(2, 0, 0), (0, 2, 0), (1, 1, 0), (1, 0, 1), (0, 1, 1)]
    if l == 3:
        return [(3, 0, 0), (2, 1, 0), (2, 0, 1), (1, 2, 0), (1, 1, 1), (0, 2, 1), (0, 3, 0)]
    comps = [(a, l - a, 0) for a in range(l, -1, -1)]
    comps += [(a, l - 1 - a, 1) for a in range(l - 1, -1, -1)]
    return comps


@lru_cache(maxsize=None)
def _rebuild_matrix(l: int) -> torch.Tensor:
    """(3**l, 2l+1) float64 matrix: full components from stored ones."""
    basis = stored_basis(l)
    index = {t: i for i, t in enumerate(basis)}
    memo = {}

    def comp(a, b, c):
        if (a, b, c) in memo:
            return memo[(a, b, c)]
        v = torch.zeros(2 * l + 1, dtype=torch.float64)
        if (a, b, c) in index:
            v[index[(a, b, c)]] = 1.0
        else:
            v = -comp(a + 2, b, c - 2) - comp(a, b + 2, c - 2)
        memo[(a, b, c)] = v
        return v

    rows = [comp(m.count(0), m.count(1), m.count(2)) for m in itertools.product(range(3), repeat=l)]
    return torch.stack(rows) if l > 0 else torch.ones(1, 1, dtype=torch.float64)


@lru_cache(maxsize=None)
def _stored_positions(l: int) -> List[int]:
    out = []
    for a, b, c in stored_basis(l):
        flat = 0
        for d in (0,) * a + (1,) * b + (2,) * c:
            flat = flat * 3 + d
        out.append(flat)
    return out


def to_full(s: torch.Tensor, l: int) -> torch.Tensor:
    """(..., 2l+1) stored -> (..., 3, ..., 3) full symmetric traceless tensor."""
    m = _rebuild_matrix(l).to(s.dtype)
    full = s @ m.T
    return full.reshape(*s.shape[:-1], *([3] * l))


def to_stored(t: torch.Tensor, l: int) -> torch.Tensor:
    """(..., 3, ..., 3) -> (..., 2l+1) by picking the stored components."""
    flat = t.reshape(*t.shape[: t.dim() - l], 3 ** l) if l > 0 else t.unsqueeze(-1)
    return flat[..., _stored_positions(l)]


def symmetrize(t: torch.Tensor, L: int) -> torch.Tensor:
    """Average over all permutations of the last L axes."""
    if L <= 1:
        return t
    lead = t.dim() - L
    acc = torch.zeros_like(t)
    for perm in itertools.permutations(range(L)):
        acc = acc + t.permute(*range(lead), *(lead + p for p in perm))
    return acc / math.factorial(L)


def _delta_power(k: int, dtype) -> torch.Tensor:
    """delta (x) ... (x) delta (k factors), shape (3,)*2k."""
    eye = torch.eye(3, dtype=dtype)
    out = torch.ones((), dtype=dtype)
    for _ in range(k):
        out = torch.tensordot(out, eye, dims=0)
    return out


def stf(t: torch.Tensor, L: int) -> torch.Tensor:
    """Symmetric trace-free part of a symmetric tensor over its last L axes.

    STF_L(R) = sum_k c_k(L) Sym{delta^k (x) Tr^k R},
    c_k(L) = (-1)^k L! (2L-2k-1)!! / (k! (L-2k)! (2L-1)!! 2^k)
    (reference ``o3/_codegen_tensor_product.py:15-23, 351-378``).
    """
    if L < 2:
        return t
    lead = t.dim() - L
    out = t.clone()
    tr = t
    for k in range(1, L // 2 + 1):
        tr = torch.diagonal(tr, dim1=lead, dim2=lead + 1).sum(-1)  # trace over the first two axes
        c = ((-1) ** k * math.factorial(L) * double_factorial(2 * L - 2 * k - 1)
             / (math.factorial(k) * math.factorial(L - 2 * k) * double_factorial(2 * L - 1) * 2 ** k))
        prod = torch.tensordot(tr, _delta_power(k, t.dtype), dims=0)
        out = out + c * symmetrize(prod, L)
    return out


def path_norm(l1: int, l2: int, lo: int) -> float:
    """Reference ``o3/_codegen_tensor_product.py:103-142``."""
    k = (l1 + l2 - lo) // 2
    j = l1 + l2 + lo
    j1, j2, j3 = j - 2 * l1 - 1, j - 2 * l2 - 1, j - 2 * lo - 1
    num = (math.factorial(l1) * math.factorial(l2) * double_factorial(2 * lo - 1)
           * math.factorial((j1 + 1) // 2) * math.factorial((j2 + 1) // 2))
    den = (math.factorial(lo) * double_factorial(j1) * double_factorial(j2) * double_factorial(j3)
           * math.factorial(j // 2))
    shuffle = math.factorial(lo) / (math.factorial(l1 - k) * math.factorial(l2 - k))
    return shuffle * num / den


def path_allowed(l1: int, l2: int, lo: int) -> bool:
    return abs(l1 - l2) <= lo <= l1 + l2 and (l1 + l2 + lo) % 2 == 0


def contract_path(s1: torch.Tensor, s2: torch.Tensor, l1: int, l2: int, lo: int) -> torch.Tensor:
    """One unweighted path on stored inputs (..., 2l1+1), (..., 2l2+1) -> (..., 2lo+1).

    The last k axes of T1 are contracted with the first k axes of T2.
    """
    k = (l1 + l2 - lo) // 2
    t1 = to_full(s1, l1)
    t2 = to_full(s2, l2)
    lead = s1.dim() - 1
    letters = "abcdefghijkl"
    a1 = letters[: l1 - k]
    c = letters[l1 - k: l1]
    a2 = letters[l1: l1 + l2 - k]
    batch = "xyz"[:lead]
    eq = f"{batch}{a1}{c},{batch}{c}{a2}->{batch}{a1}{a2}"
    r = torch.einsum(eq, t1, t2)
    r = stf(symmetrize(r, lo), lo)
    return path_norm(l1, l2, lo) * to_stored(r, lo)


def enumerate_paths(in1_l_max: int, in2_l_max: int, out_l_max: int, symmetric: bool):
    """(l1, l2, lo, swapped) in weight order (reference ``o3/utils.py:157-203``)."""
    lmax = max(in1_l_max, in2_l_max)
    out = []
    for lo in range(out_l_max + 1):
        for l1 in range(lmax + 1):
            for l2 in range(l1 + 1):
                if path_allowed(l1, l2, lo) and l1 <= in1_l_max and l2 <= in2_l_max:
                    out.append((l1, l2, lo, False))
        if not symmetric:
            for l1 in range(lmax + 1):
                for l2 in range(l1):
                    if path_allowed(l1, l2, lo) and l1 <= in2_l_max and l2 <= in1_l_max:
                        out.append((l1, l2, lo, True))
    return out


@lru_cache(maxsize=None)
def path_coefficients(l1: int, l2: int, lo: int) -> torch.Tensor:
    """Dense float64 K[k, a, b] of one path on stored components, evaluated once by
    running ``contract_path`` (full Cartesian tensors, explicit detracer) on every pair of
    stored basis vectors; the product is then sum_ab K[k,a,b] S1_a S2_b."""
    n1, n2 = 2 * l1 + 1, 2 * l2 + 1
    e1 = torch.eye(n1, dtype=torch.float64)
    e2 = torch.eye(n2, dtype=torch.float64)
    s1 = e1[:, None, :].expand(n1, n2, n1).reshape(-1, n1)
    s2 = e2[None, :, :].expand(n1, n2, n2).reshape(-1, n2)
    y = contract_path(s1, s2, l1, l2, lo)  # (n1*n2, 2lo+1)
    return y.reshape(n1, n2, 2 * lo + 1).permute(2, 0, 1).contiguous()


def _apply_path(K: torch.Tensor, a: torch.Tensor, b: torch.Tensor, n: int, F: int) -> torch.Tensor:
    """y[n, k, f] = sum_ij K[k, i, j] a[n, i, f] b[n, j, f]."""
    return torch.einsum("kab,naf,nbf->nkf", K.to(a.dtype), a.expand(n, K.shape[1], F), b.expand(n, K.shape[2], F))


def _rank_block(x: torch.Tensor, l: int, features: int) -> torch.Tensor:
    start = l * l * features
    return x[:, start: start + (2 * l + 1) * features].reshape(x.shape[0], 2 * l + 1, features)


def _rank_blocks(x: torch.Tensor, l_max: int, features: int) -> List[torch.Tensor]:
    """All rank blocks of x as (rows, 2l+1, features) views from one split (columns past
    the last full block, if any, are left out)."""
    sizes = [(2 * l + 1) * features for l in range(l_max + 1)]
    rest = x.shape[1] - sum(sizes)
    parts = torch.split(x, sizes + ([rest] if rest > 0 else []), dim=1)
    return [parts[l].reshape(x.shape[0], 2 * l + 1, features) for l in range(l_max + 1)]


def tensor_product(in1, in2, weights, idx_i, idx_j, in1_l_max, in2_l_max, out_l_max, in1_features,
                   in2_features, symmetric_product=False, shared_weights=False, reduce_paths=False):
    """Weighted Cartesian tensor product, optionally as an edge convolution.

    Semantics of the reference py path (``o3/_codegen_tensor_product.py:833-1012``):
    in1 rows are gathered by sender (idx_j), each path output is multiplied by its
    per-feature weight, stacked as (2l+1, paths, F) per rank (or summed when reduced)
    and summed at the receivers (idx_i).
    """
    conv = idx_i is not None and idx_j is not None
    n_nodes = in1.shape[0]
    if conv:
        in1 = in1.index_select(0, idx_j)
    n = in1.shape[0]
    n_out = n_nodes if conv else n
    F = max(in1_features, in2_features)
    paths = enumerate_paths(in1_l_max, in2_l_max, out_l_max, symmetric_product)
    per_l: List[List[torch.Tensor]] = [[] for _ in range(out_l_max + 1)]
    # rank blocks split once (one backward concatenation instead of a zero-filled full-width
    # gradient per sliced path)
    split1 = _rank_blocks(in1, in1_l_max, in1_features)
    split2 = _rank_blocks(in2, in2_l_max, in2_features)
    wparts = torch.split(weights, F, dim=0 if shared_weights else 1)
    for p, (l1, l2, lo, swapped) in enumerate(paths):
        if swapped:
            a = split2[l1]
            b = split1[l2]
        else:
            a = split1[l1]
            b = split2[l2]
        y = _apply_path(path_coefficients(l1, l2, lo), a, b, n, F)
        w = wparts[p] if shared_weights else wparts[p].unsqueeze(1)
        y = y * w
        if conv:
            # the sum over a receiver's edges, path by path (the same sum as scattering the
            # stacked edge rows, without the edges x output-width intermediate)
            y = y.new_zeros((n_nodes,) + tuple(y.shape[1:])).index_add(0, idx_i, y)
        per_l[lo].append(y)
    blocks = []
    for lo, bucket in enumerate(per_l):
        if not bucket:
            continue
        # explicit widths: with no edges (n = 0) a reshape to (n, -1) is ambiguous and the
        # reference py path raises there, while its CUDA operator writes every receiver row
        # as an empty sum (CSR grid over receivers, o3/_tensor_product.py:396-412); the
        # oracle gives that empty sum
        t = sum(bucket) if reduce_paths else torch.stack(bucket, dim=2)
        blocks.append(t.reshape(n_out, math.prod(t.shape[1:])))
    return torch.cat(blocks, dim=-1) if blocks else in1.new_zeros(n_out, 0)


def irreps(x: torch.Tensor, l_max: int) -> torch.Tensor:
    """Stored components of T^l(x), l = 0..l_max, rows concatenated by rank.

    T^l = sum_m a_m * (number of placements) * Sym(x^(l-2m) (x) delta^m) with
    a_m = (2l-1)!!/l! * (-1)^m (2l-2m-1)!!/(2l-1)!!; the deltas are constants
    (reference ``o3/_codegen_irreps.py:148-164``).
    """
    parts = [torch.ones(x.shape[0], 1, dtype=x.dtype)]
    for l in range(1, l_max + 1):
        t = torch.zeros(x.shape[0], *([3] * l), dtype=x.dtype)
        for m in range(l // 2 + 1):
            p = l - 2 * m
            am = (double_factorial(2 * l - 1) / math.factorial(l)
                  * (-1) ** m * double_factorial(2 * l - 2 * m - 1) / double_factorial(2 * l - 1))
            count = math.factorial(l) / (math.factorial(p) * math.factorial(m) * 2 ** m)
            xp = torch.ones(x.shape[0], dtype=x.dtype)
            for _ in range(p):
                xp = xp.unsqueeze(-1) * x.reshape(x.shape[0], *([1] * (xp.dim() - 1)), 3)
            d = _delta_power(m, x.dtype)
            term = xp.reshape(*xp.shape, *([1] * (2 * m))) * d
            t = t + am * count * symmetrize(term, l)
        parts.append(to_stored(t, l))
    return torch.cat(parts, dim=-1)


def linear(x: torch.Tensor, weights: Sequence[torch.Tensor], in_l_max: int, out_l_max: int, in_features: int,
           out_features: int, in_paths: Optional[Sequence[int]] = None,
           weight_scale: Optional[float] = None, scales: Optional[Sequence[float]] = None) -> torch.Tensor:
    """Per-rank channel mixing (reference ``o3/_linear.py:64-110``); missing ranks are zero.

    ``scales`` (one per shared rank) overrides the default 1/sqrt(in_features * paths_l).
    """
    in_paths = [1] * (in_l_max + 1) if in_paths is None else list(in_paths)
    common = min(in_l_max, out_l_max)
    n = x.shape[0]
    outs = []
    off = 0
    for l in range(in_l_max + 1):
        width = in_features * in_paths[l]
        blk = x[:, off: off + (2 * l + 1) * width].reshape(n, 2 * l + 1, width)
        off += (2 * l + 1) * width
        if l <= common:
            if scales is not None:
                scale = scales[l]
            else:
                scale = weight_scale if weight_scale is not None else (in_features * in_paths[l]) ** -0.5
            outs.append((blk @ (weights[l] * scale).T).reshape(n, -1))
    for l in range(common + 1, out_l_max + 1):
        outs.append(x.new_zeros(n, (2 * l + 1) * out_features))
    return torch.cat(outs, dim=-1)


def linear_scales(in_l_max: int, out_l_max: int, in_features: int, in_paths=None, weight_scale=None):
    in_paths = [1] * (in_l_max + 1) if in_paths is None else list(in_paths)
    common = min(in_l_max, out_l_max)
    if weight_scale is not None:
        return [float(weight_scale)] * (common + 1)
    return [(in_features * in_paths[l]) ** -0.5 for l in range(common + 1)]
