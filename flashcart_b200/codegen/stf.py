"""Exact symmetric-traceless (STF) Cartesian tensor algebra used to generate kernels.

Everything here is computed in exact rational arithmetic (``fractions.Fraction``)
and only at build time. The results are

* the stored-component convention of the reference (``stored_basis``,
  reference ``src/flashcart/o3/_codegen_common.py:37-73``): ``2l+1`` independent
  components of a rank-l STF tensor, every other Cartesian component following
  from symmetry and tracelessness;
* the bilinear coupling tensor ``K[a, i, j]`` of every natural-parity path
  ``(l1, l2) -> lo``: ``out_a = sum_ij K[a,i,j] * S1_i * S2_j`` in stored
  components. The path is ``N(l1,l2,lo) * STF_lo(contract_k(T1 (x) T2))`` with
  ``k = (l1+l2-lo)/2`` (Eq. (2) of Zaverkin et al., NeurIPS 2024; reference
  ``src/flashcart/o3/_codegen_tensor_product.py:7-58, 400-414``);
* the monomial expansion of the direction-tensor polynomials ``T^l(r)``
  (Eq. (1), reference ``src/flashcart/o3/_codegen_irreps.py:1-32, 148-164``).

Derivation used here (not the reference's): the STF part of any rank-L tensor R
is its orthogonal projection, under the Frobenius inner product on full
Cartesian tensors, onto the span of STF tensors. With ``B`` the (3^L x (2L+1))
matrix that rebuilds full components from stored ones, the stored components of
that projection are ``(B^T B)^-1 B^T vec(R)``. The projection of R equals the
projection of its index-symmetrisation (STF tensors are symmetric), so no
explicit permutation average is needed. Both agree with the explicit
trace-removal series of the reference; the generated tables are pinned against
golden vectors produced by the reference in ``tests/golden``.
"""

from __future__ import annotations

import itertools
import math
from fractions import Fraction
from functools import lru_cache
from typing import Dict, List, Tuple

Frac = Fraction


def double_factorial(n: int) -> int:
    """n!! with the convention (-1)!! = 1 (and 1 for every negative n)."""
    out = 1
    while n > 1:
        out *= n
        n -= 2
    return out


@lru_cache(maxsize=None)
def stored_basis(l: int) -> Tuple[Tuple[int, int, int], ...]:
    """(nx, ny, nz) index counts of the stored components of a rank-l STF tensor.

    Order matches reference ``_codegen_common.py:37-73``: l=1 x,y,z; l=2
    xx,yy,xy,xz,yz; l=3 xxx,xxy,xxz,xyy,xyz,yyz,yyy; l>=4 the nz=0 components by
    descending nx, then the nz=1 components by descending nx.
    """
    if l == 0:
        return ((0, 0, 0),)
    if l == 1:
        return ((1, 0, 0), (0, 1, 0), (0, 0, 1))
    if l == 2:
        return ((2, 0, 0), (0, 2, 0), (1, 1, 0), (1, 0, 1), (0, 1, 1))
    if l == 3:
        return ((3, 0, 0), (2, 1, 0), (2, 0, 1), (1, 2, 0), (1, 1, 1), (0, 2, 1), (0, 3, 0))
    comps = [(a, l - a, 0) for a in range(l, -1, -1)]
    comps += [(a, l - 1 - a, 1) for a in range(l - 1, -1, -1)]
    return tuple(comps)


@lru_cache(maxsize=None)
def _counts_to_stored(l: int) -> Dict[Tuple[int, int, int], Tuple[Frac, ...]]:
    """Map every (nx,ny,nz) with nx+ny+nz=l to its stored-component coefficients.

    A component with nz >= 2 is rewritten by tracelessness over one z-pair:
    T(a,b,c) = -T(a+2,b,c-2) - T(a,b+2,c-2).
    """
    n = 2 * l + 1
    basis = stored_basis(l)
    table: Dict[Tuple[int, int, int], Tuple[Frac, ...]] = {}
    for idx, cnt in enumerate(basis):
        vec = [Frac(0)] * n
        vec[idx] = Frac(1)
        table[cnt] = tuple(vec)

    def solve(a: int, b: int, c: int) -> Tuple[Frac, ...]:
        key = (a, b, c)
        if key in table:
            return table[key]
        if c < 2:
            raise ValueError(f"component {key} of rank {l} is neither stored nor reducible")
        u = solve(a + 2, b, c - 2)
        v = solve(a, b + 2, c - 2)
        res = tuple(-x - y for x, y in zip(u, v))
        table[key] = res
        return res

    for c in range(l + 1):
        for b in range(l - c + 1):
            solve(l - b - c, b, c)
    return table


@lru_cache(maxsize=None)
def full_from_stored(l: int) -> Tuple[Tuple[Frac, ...], ...]:
    """Matrix B (3^l rows, 2l+1 columns): full Cartesian components from stored ones.

    Rows follow the flattened Cartesian index with the last index fastest.
    """
    table = _counts_to_stored(l)
    rows = []
    for multi in itertools.product(range(3), repeat=l):
        rows.append(table[(multi.count(0), multi.count(1), multi.count(2))])
    return tuple(rows)


def _solve_exact(a: List[List[Frac]], b: List[List[Frac]]) -> List[List[Frac]]:
    """Solve A X = B for square nonsingular A by Gauss-Jordan elimination."""
    n = len(a)
    m = len(b[0])
    aug = [list(a[r]) + list(b[r]) for r in range(n)]
    for col in range(n):
        piv = next(r for r in range(col, n) if aug[r][col] != 0)
        aug[col], aug[piv] = aug[piv], aug[col]
        inv = 1 / aug[col][col]
        aug[col] = [v * inv for v in aug[col]]
        for r in range(n):
            if r != col and aug[r][col] != 0:
                f = aug[r][col]
                aug[r] = [x - f * y for x, y in zip(aug[r], aug[col])]
    return [row[n:] for row in aug]


@lru_cache(maxsize=None)
def stf_readout(l: int) -> Tuple[Tuple[Frac, ...], ...]:
    """Matrix R ((2l+1) x 3^l): stored components of the STF projection of a full tensor.

    R = (B^T B)^-1 B^T with B = full_from_stored(l).
    """
    bmat = full_from_stored(l)
    n = 2 * l + 1
    rows = len(bmat)
    btb = [[sum(bmat[r][i] * bmat[r][j] for r in range(rows)) for j in range(n)] for i in range(n)]
    bt = [[bmat[r][i] for r in range(rows)] for i in range(n)]
    return tuple(tuple(row) for row in _solve_exact(btb, bt))


def path_allowed(l1: int, l2: int, lo: int) -> bool:
    """Triangle rule plus even l1+l2+lo (reference ``_codegen_tensor_product.py:145-163``)."""
    if min(l1, l2, lo) < 0:
        return False
    return abs(l1 - l2) <= lo <= l1 + l2 and (l1 + l2 + lo) % 2 == 0


def path_norm(l1: int, l2: int, lo: int) -> Frac:
    """Normalisation of one path: the closed-form Eq. (2) factor times the shuffle count.

    C = l1! l2! (2lo-1)!! ((J1+1)/2)! ((J2+1)/2)! / (lo! J1!! J2!! J3!! (J/2)!) with
    J = l1+l2+lo and Ji = J - 2 li - 1, multiplied by lo! / ((l1-k)! (l2-k)!), the
    number of distinct placements of the two uncontracted index groups. It is
    symmetric in (l1, l2). Reference: ``_codegen_tensor_product.py:103-142``.
    """
    if not path_allowed(l1, l2, lo):
        raise ValueError(f"path ({l1},{l2})->{lo} not allowed")
    k = (l1 + l2 - lo) // 2
    j = l1 + l2 + lo
    j1, j2, j3 = j - 2 * l1 - 1, j - 2 * l2 - 1, j - 2 * lo - 1
    num = (math.factorial(l1) * math.factorial(l2) * double_factorial(2 * lo - 1)
           * math.factorial((j1 + 1) // 2) * math.factorial((j2 + 1) // 2))
    den = (math.factorial(lo) * double_factorial(j1) * double_factorial(j2)
           * double_factorial(j3) * math.factorial(j // 2))
    shuffle = Frac(math.factorial(lo), math.factorial(l1 - k) * math.factorial(l2 - k))
    return Frac(num, den) * shuffle


@lru_cache(maxsize=None)
def path_tensor(l1: int, l2: int, lo: int) -> Tuple[Tuple[Tuple[Frac, ...], ...], ...]:
    """Exact K[a][i][j] for the path with first operand rank l1, second operand rank l2.

    The last k indices of T1 are contracted with the first k indices of T2
    (any choice gives the same STF part since both operands are symmetric).
    """
    if not path_allowed(l1, l2, lo):
        raise ValueError(f"path ({l1},{l2})->{lo} not allowed")
    k = (l1 + l2 - lo) // 2
    b1 = full_from_stored(l1)
    b2 = full_from_stored(l2)
    ro = stf_readout(lo)
    norm = path_norm(l1, l2, lo)
    n1, n2, no = 2 * l1 + 1, 2 * l2 + 1, 2 * lo + 1
    idx1 = list(itertools.product(range(3), repeat=l1))
    idx2 = list(itertools.product(range(3), repeat=l2))
    pos1 = {t: r for r, t in enumerate(idx1)}
    pos2 = {t: r for r, t in enumerate(idx2)}
    out_idx = list(itertools.product(range(3), repeat=lo))
    # contraction pattern: out index = (first l1-k of T1) + (last l2-k of T2),
    # summed over the shared k-tuple c.
    pattern = []
    for o in out_idx:
        pre, suf = o[: l1 - k], o[l1 - k:]
        pairs = []
        for c in itertools.product(range(3), repeat=k):
            pairs.append((pos1[pre + c], pos2[c + suf]))
        pattern.append(pairs)
    K = [[[Frac(0)] * n2 for _ in range(n1)] for _ in range(no)]
    for i in range(n1):
        for j in range(n2):
            # full contracted tensor for the basis pair (e_i, e_j)
            full = []
            for pairs in pattern:
                s = Frac(0)
                for r1, r2 in pairs:
                    v1 = b1[r1][i]
                    if v1:
                        v2 = b2[r2][j]
                        if v2:
                            s += v1 * v2
                full.append(s)
            for a in range(no):
                val = sum((ro[a][r] * full[r] for r in range(len(full)) if full[r]), Frac(0))
                K[a][i][j] = val * norm
    return tuple(tuple(tuple(row) for row in plane) for plane in K)


# ----------------------------------------------------------------------------------
# path enumeration (weights / output layout order)
# ----------------------------------------------------------------------------------


def enumerate_paths(in1_l_max: int, in2_l_max: int, out_l_max: int,
                    symmetric_product: bool = False) -> List[Tuple[int, int, int]]:
    """Paths in weight order as (r1, r2, lo): r1 = in1 rank, r2 = in2 rank.

    Per output rank: canonical pairs (l1 >= l2) by ascending l1 then l2 with
    l1 from in1 and l2 from in2, then (unless symmetric) the swapped unequal pairs
    with l1 taken from in2 and l2 from in1, in the same order. Reference
    ``o3/utils.py:157-203`` and ``_codegen_tensor_product.py:967-989``.
    """
    lmax = max(in1_l_max, in2_l_max)
    paths = []
    for lo in range(out_l_max + 1):
        for l1 in range(lmax + 1):
            for l2 in range(l1 + 1):
                if path_allowed(l1, l2, lo) and l1 <= in1_l_max and l2 <= in2_l_max:
                    paths.append((l1, l2, lo))
        if not symmetric_product:
            for l1 in range(lmax + 1):
                for l2 in range(l1):
                    if path_allowed(l1, l2, lo) and l1 <= in2_l_max and l2 <= in1_l_max:
                        paths.append((l2, l1, lo))
    return paths


def oriented_path_tensor(r1: int, r2: int, lo: int):
    """K for in1 rank r1 and in2 rank r2 (transposes the canonical table for swaps)."""
    if r1 >= r2:
        return path_tensor(r1, r2, lo)
    kt = path_tensor(r2, r1, lo)
    no, n1, n2 = 2 * lo + 1, 2 * r1 + 1, 2 * r2 + 1
    return tuple(tuple(tuple(kt[a][j][i] for j in range(n2)) for i in range(n1)) for a in range(no))


# ----------------------------------------------------------------------------------
# direction-tensor polynomials T^l(r) (edge attributes)
# ----------------------------------------------------------------------------------

Monomial = Tuple[int, int, int]


def _pairings(n: int, k: int) -> int:
    """Number of ways to pick k disjoint unordered pairs out of n labelled slots."""
    if 2 * k > n:
        return 0
    return math.comb(n, 2 * k) * double_factorial(2 * k - 1)


@lru_cache(maxsize=None)
def irreps_polynomials(l: int) -> Tuple[Dict[Monomial, Frac], ...]:
    """Stored components of T^l as polynomials {(px,py,pz): coeff} in (x, y, z).

    T^l = (2l-1)!!/l! * sum_m (-1)^m (2l-2m-1)!!/(2l-1)!! {x^(l-2m) (x) I^m}, the
    braces summing every distinct placement of the Kronecker pairs. For a
    component with index counts (a, b, c) a pair can only sit on two equal
    indices, so the placements factorise over the three axes. The Kronecker
    deltas are constants: the polynomial is not rewritten with |x|^2 = 1, which
    fixes its derivatives (reference ``_codegen_irreps.py:148-230``).
    """
    pref = Frac(double_factorial(2 * l - 1), math.factorial(l))
    out = []
    for a, b, c in stored_basis(l):
        poly: Dict[Monomial, Frac] = {}
        for m in range(l // 2 + 1):
            cm = Frac((-1) ** m * double_factorial(2 * l - 2 * m - 1), double_factorial(2 * l - 1))
            for mx in range(m + 1):
                for my in range(m - mx + 1):
                    mz = m - mx - my
                    cnt = _pairings(a, mx) * _pairings(b, my) * _pairings(c, mz)
                    if cnt == 0:
                        continue
                    mono = (a - 2 * mx, b - 2 * my, c - 2 * mz)
                    poly[mono] = poly.get(mono, Frac(0)) + pref * cm * cnt
        out.append({k: v for k, v in poly.items() if v != 0})
    return tuple(out)


def poly_diff(poly: Dict[Monomial, Frac], axis: int) -> Dict[Monomial, Frac]:
    """Partial derivative of a monomial dictionary along axis 0/1/2."""
    out: Dict[Monomial, Frac] = {}
    for mono, c in poly.items():
        p = mono[axis]
        if p == 0:
            continue
        m = list(mono)
        m[axis] -= 1
        key = tuple(m)
        out[key] = out.get(key, Frac(0)) + c * p
    return {k: v for k, v in out.items() if v != 0}
