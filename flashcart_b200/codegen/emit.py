"""Emit the generated CUDA sources of the tensor-product and direction-tensor kernels.

Run ``python -m flashcart_b200.codegen.emit`` (``build()`` does it) to rewrite
``flashcart_b200/csrc/gen``. Every formula comes from the exact tables of
:mod:`flashcart_b200.codegen.stf`; nothing is read from the reference.

One CUDA file is written per tensor-product *signature* ``(L1, L2, LO, SYM)``
(maximum ranks of in1, in2 and the output, and whether only the canonical
``l1 >= l2`` paths are kept). Each file holds, for float and double:

* ``fwd``   per-(receiver, channel) body: receiver-CSR edge loop (convolution)
            or one row (dense), accumulating every path in registers;
* ``bwd``   per-(receiver, channel) body: grad_out held in registers, edge loop
            producing grad_weights per edge, grad_in2 per edge and grad_in1
            scattered to senders with ``red.global.add``;
* ``dbwd``  per-(receiver, channel) body of the second derivative.

Bodies are ``__host__ __device__`` so the CPU test build (``FC_HOST_EMU``)
executes the exact generated arithmetic; ``__global__`` wrappers map
(block, thread) onto (receiver, channel).
"""

from __future__ import annotations

import os
import sys
from fractions import Fraction
from typing import Dict, List, Sequence, Tuple

from flashcart_b200.codegen import emit_conv, emit_dense, emit_pair, stf

L_MAX = 3
GEN_DIR = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc", "gen")


# ----------------------------------------------------------------------------------
# expression helpers
# ----------------------------------------------------------------------------------


def const(fr: Fraction) -> str:
    return f"T({float(fr)!r})"


def lin(terms: Sequence[Tuple[Fraction, str]]) -> str:
    """sum_k c_k * v_k as C source (terms with c == 0 dropped)."""
    parts = []
    for c, v in terms:
        if c == 0:
            continue
        if c == 1:
            s = f"+{v}"
        elif c == -1:
            s = f"-{v}"
        elif c > 0:
            s = f"+{const(c)}*{v}"
        else:
            s = f"-{const(-c)}*{v}"
        parts.append(s)
    if not parts:
        return "T(0)"
    out = "".join(parts)
    return out[1:] if out[0] == "+" else out


def prod_sum(pairs: Sequence[Tuple[str, str]]) -> str:
    """sum_k a_k * (b_k) as C source."""
    if not pairs:
        return "T(0)"
    return " + ".join(f"{a}*({b})" for a, b in pairs)


# ----------------------------------------------------------------------------------
# signature bookkeeping
# ----------------------------------------------------------------------------------


class Sig:
    def __init__(self, l1: int, l2: int, lo: int, sym: bool):
        self.l1, self.l2, self.lo, self.sym = l1, l2, lo, sym
        self.paths = stf.enumerate_paths(l1, l2, lo, sym)
        self.npl = [sum(1 for p in self.paths if p[2] == l) for l in range(lo + 1)]
        self.d1 = (l1 + 1) ** 2
        self.d2 = (l2 + 1) ** 2
        # accumulator base per path
        self.base = []
        k = 0
        pl_count = [0] * (lo + 1)
        self.pl = []
        for r1, r2, o in self.paths:
            self.base.append(k)
            k += 2 * o + 1
            self.pl.append(pl_count[o])
            pl_count[o] += 1
        self.nacc = k

    @property
    def name(self) -> str:
        return f"{self.l1}{self.l2}{self.lo}{'s' if self.sym else 'n'}"

    @property
    def npaths(self) -> int:
        return len(self.paths)

    def out_store_exprs(self) -> List[Tuple[str, str]]:
        """(offset-in-components expression for non-reduced, for reduced) per accumulator.

        Returned offsets are in units of F (channels): the store address is
        row_base + off * F + c.
        """
        res = []
        # non-reduced component offset: sum_{l<lo} npl[l]*(2l+1) + a*npl[lo] + pl
        nr_block = []
        r_block = []
        s_nr = 0
        s_r = 0
        for l in range(self.lo + 1):
            nr_block.append(s_nr)
            r_block.append(s_r)
            s_nr += self.npl[l] * (2 * l + 1)
            s_r += (2 * l + 1) if self.npl[l] > 0 else 0
        self.out_comps_nr = s_nr
        self.out_comps_r = s_r
        for p, (r1, r2, o) in enumerate(self.paths):
            for a in range(2 * o + 1):
                res.append((nr_block[o] + a * self.npl[o] + self.pl[p], r_block[o] + a))
        return res


def q1(r: int, i: int) -> int:
    return r * r + i


# ----------------------------------------------------------------------------------
# per-path code fragments
# ----------------------------------------------------------------------------------


def fwd_path_code(sig: Sig, p: int, ind: str) -> List[str]:
    r1, r2, o = sig.paths[p]
    K = stf.oriented_path_tensor(r1, r2, o)
    lines = [f"{ind}{{ // path {p}: in1 l={r1} x in2 l={r2} -> l={o}", f"{ind}  const T wp = WLOAD({p});"]
    for a in range(2 * o + 1):
        pairs = []
        for i in range(2 * r1 + 1):
            m = lin([(K[a][i][j], f"x2[{q1(r2, j)}]") for j in range(2 * r2 + 1)])
            if m != "T(0)":
                pairs.append((f"x1[{q1(r1, i)}]", m))
        k = sig.base[p] + a
        lines.append(f"{ind}  acc[{k}] += wp * ({prod_sum(pairs)});")
    lines.append(f"{ind}}}")
    return lines


def bwd_path_code(sig: Sig, p: int, ind: str) -> List[str]:
    """grad wrt w (gw[p]), in1 (gx1) and in2 (gx2) for one path, g = grad_out."""
    r1, r2, o = sig.paths[p]
    K = stf.oriented_path_tensor(r1, r2, o)
    b = sig.base[p]
    lines = [f"{ind}{{ // path {p}: in1 l={r1} x in2 l={r2} -> l={o}", f"{ind}  const T wp = WLOAD({p});"]
    # h_i = sum_a g_a * m_{a,i};  m_{a,i} = sum_j K x2_j
    hnames = []
    for i in range(2 * r1 + 1):
        pairs = []
        for a in range(2 * o + 1):
            m = lin([(K[a][i][j], f"x2[{q1(r2, j)}]") for j in range(2 * r2 + 1)])
            if m != "T(0)":
                pairs.append((f"g[{b + a}]", m))
        if pairs:
            lines.append(f"{ind}  const T h{i} = {prod_sum(pairs)};")
            hnames.append((i, f"h{i}"))
    gw = " + ".join(f"x1[{q1(r1, i)}]*{h}" for i, h in hnames) or "T(0)"
    lines.append(f"{ind}  if (NEED_W) gw[{p}] = {gw};")
    if hnames:
        lines.append(f"{ind}  if (NEED_1) {{")
        for i, h in hnames:
            lines.append(f"{ind}    gx1[{q1(r1, i)}] += wp * {h};")
        lines.append(f"{ind}  }}")
    # gx2_j += wp * sum_a g_a * n_{a,j};  n_{a,j} = sum_i K x1_i
    body2 = []
    for j in range(2 * r2 + 1):
        pairs = []
        for a in range(2 * o + 1):
            n = lin([(K[a][i][j], f"x1[{q1(r1, i)}]") for i in range(2 * r1 + 1)])
            if n != "T(0)":
                pairs.append((f"g[{b + a}]", n))
        if pairs:
            body2.append(f"{ind}    gx2[{q1(r2, j)}] += wp * ({prod_sum(pairs)});")
    if body2:
        lines.append(f"{ind}  if (NEED_2) {{")
        lines.extend(body2)
        lines.append(f"{ind}  }}")
    lines.append(f"{ind}}}")
    return lines


def dbwd_path_code(sig: Sig, p: int, ind: str) -> List[str]:
    """Second derivative of one path.

    Forward y_a = w * f_a(x1, x2), f bilinear. The backward maps
    (g; x1, x2, w) -> (gx1, gx2, gw) with gx1_i = w sum_a g_a df_a/dx1_i,
    gx2_j = w sum_a g_a df_a/dx2_j, gw = sum_a g_a f_a. Given tangents
    (v1, v2, vw) on (gx1, gx2, gw) the VJP of the backward is
      d_g_a  = w (J1 v1 + J2 v2)_a + vw f_a
      d_x1_i = sum_a g_a [ w sum_j K v2_j + vw sum_j K x2_j ]_{a,i}
      d_x2_j = sum_a g_a [ w sum_i K v1_i + vw sum_i K x1_i ]_{a,j}
      d_w    = sum_a g_a [ (J1 v1)_a + (J2 v2)_a ]
    with (J1 v1)_a = sum_ij K v1_i x2_j and (J2 v2)_a = sum_ij K x1_i v2_j.
    Reference: ``_codegen_tensor_product.py:468-519`` and the weighted rule at
    ``:30-44``.
    """
    r1, r2, o = sig.paths[p]
    K = stf.oriented_path_tensor(r1, r2, o)
    b = sig.base[p]
    lines = [f"{ind}{{ // path {p}: in1 l={r1} x in2 l={r2} -> l={o}",
             f"{ind}  const T wp = WLOAD({p});",
             f"{ind}  const T vw = HAS_VW ? VWLOAD({p}) : T(0);"]
    for a in range(2 * o + 1):
        # J1 v1 and J2 v2 and f for component a
        j1 = []
        j2 = []
        f = []
        for i in range(2 * r1 + 1):
            m = lin([(K[a][i][j], f"x2[{q1(r2, j)}]") for j in range(2 * r2 + 1)])
            if m != "T(0)":
                j1.append((f"v1[{q1(r1, i)}]", m))
                f.append((f"x1[{q1(r1, i)}]", m))
            mv = lin([(K[a][i][j], f"v2[{q1(r2, j)}]") for j in range(2 * r2 + 1)])
            if mv != "T(0)":
                j2.append((f"x1[{q1(r1, i)}]", mv))
        lines.append(f"{ind}  {{")
        lines.append(f"{ind}    const T jv = (HAS_V1 ? ({prod_sum(j1)}) : T(0)) + (HAS_V2 ? ({prod_sum(j2)}) : T(0));")
        lines.append(f"{ind}    if (NEED_DG) dg[{b + a}] += wp * jv + (HAS_VW ? vw * ({prod_sum(f)}) : T(0));")
        lines.append(f"{ind}    if (NEED_DW) dw[{p}] += g[{b + a}] * jv;")
        lines.append(f"{ind}  }}")
    # d_x1_i = sum_a g_a sum_j K (w v2_j + vw x2_j)
    body1 = []
    for i in range(2 * r1 + 1):
        pairs = []
        for a in range(2 * o + 1):
            m = lin([(K[a][i][j], f"e2[{q1(r2, j)}]") for j in range(2 * r2 + 1)])
            if m != "T(0)":
                pairs.append((f"g[{b + a}]", m))
        if pairs:
            body1.append(f"{ind}    dx1[{q1(r1, i)}] += {prod_sum(pairs)};")
    body2 = []
    for j in range(2 * r2 + 1):
        pairs = []
        for a in range(2 * o + 1):
            n = lin([(K[a][i][j], f"e1[{q1(r1, i)}]") for i in range(2 * r1 + 1)])
            if n != "T(0)":
                pairs.append((f"g[{b + a}]", n))
        if pairs:
            body2.append(f"{ind}    dx2[{q1(r2, j)}] += {prod_sum(pairs)};")
    if body1:
        lines.append(f"{ind}  if (NEED_DX1) {{")
        lines.append(f"{ind}    T e2[{sig.d2}];")
        lines.append(f"{ind}    for (int q = {r2 * r2}; q < {(r2 + 1) ** 2}; ++q) "
                     f"e2[q] = (HAS_V2 ? wp * v2[q] : T(0)) + (HAS_VW ? vw * x2[q] : T(0));")
        lines.extend(body1)
        lines.append(f"{ind}  }}")
    if body2:
        lines.append(f"{ind}  if (NEED_DX2) {{")
        lines.append(f"{ind}    T e1[{sig.d1}];")
        lines.append(f"{ind}    for (int q = {r1 * r1}; q < {(r1 + 1) ** 2}; ++q) "
                     f"e1[q] = (HAS_V1 ? wp * v1[q] : T(0)) + (HAS_VW ? vw * x1[q] : T(0));")
        lines.extend(body2)
        lines.append(f"{ind}  }}")
    lines.append(f"{ind}}}")
    return lines


# ----------------------------------------------------------------------------------
# signature file
# ----------------------------------------------------------------------------------


def emit_signature(sig: Sig) -> str:
    stores = sig.out_store_exprs()
    n = sig.name
    L = []
    w = L.append
    w(f"// Generated by flashcart_b200/codegen/emit.py -- signature in1 l<={sig.l1}, in2 l<={sig.l2}, "
      f"out l<={sig.lo}, {'symmetric (canonical paths only)' if sig.sym else 'all paths'}.")
    w(f"// paths (in1 rank, in2 rank, out rank) in weight order: {sig.paths}")
    w('#include "../tp_common.cuh"')
    w("namespace fc {")
    w(f"namespace sig_{n} {{")
    w(f"constexpr int D1 = {sig.d1}, D2 = {sig.d2}, NP = {sig.npaths}, NACC = {sig.nacc};")
    w(f"constexpr int OUT_COMPS = {sig.out_comps_nr}, OUT_COMPS_RED = {sig.out_comps_r};")
    w("")
    # ---------------- forward body
    w("template <typename T>")
    w("FC_HD FC_INLINE void fwd_body(const TpParams<T>& P, int64_t row, int c) {")
    w("  const int F = P.F; const int c1 = P.F1 == 1 ? 0 : c; const int c2 = P.F2 == 1 ? 0 : c;")
    w("  T acc[NACC];")
    w("  for (int k = 0; k < NACC; ++k) acc[k] = T(0);")
    w("  int64_t e0, e1;")
    w("  if (P.rowptr) { e0 = P.rowptr[row]; e1 = P.rowptr[row + 1]; } else { e0 = row; e1 = row + 1; }")
    w("  for (int64_t e = e0; e < e1; ++e) {")
    w("    const int64_t j = P.rowptr ? P.idx_j[e] : row;")
    w("    if ((uint64_t)j >= (uint64_t)P.n_in1) { fc_flag(P.status, FC_DEV_BAD_INDEX); continue; }")
    w("    const T* __restrict__ a1 = P.in1 + j * (int64_t)(D1 * P.F1) + c1;")
    w("    const T* __restrict__ a2 = P.in2 + e * (int64_t)(D2 * P.F2) + c2;")
    w("    const T* __restrict__ wr = P.w + (P.shared_w ? 0 : e * (int64_t)(NP * F)) + c;")
    w("    T x1[D1], x2[D2];")
    w("    for (int q = 0; q < D1; ++q) x1[q] = fc_ldg(a1 + q * P.F1);")
    w("    for (int q = 0; q < D2; ++q) x2[q] = fc_ldg(a2 + q * P.F2);")
    w("#define WLOAD(p) fc_ldg(wr + (p) * F)")
    for p in range(sig.npaths):
        L.extend(fwd_path_code(sig, p, "    "))
    w("#undef WLOAD")
    w("  }")
    w("  T* __restrict__ o = P.out + row * (int64_t)((P.reduce ? OUT_COMPS_RED : OUT_COMPS) * F) + c;")
    w("  if (!P.reduce) {")
    for k, (nr, r) in enumerate(stores):
        w(f"    o[{nr} * F] = acc[{k}];")
    w("  } else {")
    red: Dict[int, List[int]] = {}
    for k, (nr, r) in enumerate(stores):
        red.setdefault(r, []).append(k)
    for r, ks in sorted(red.items()):
        w(f"    o[{r} * F] = {' + '.join(f'acc[{k}]' for k in ks)};")
    w("  }")
    w("}")
    w("")
    # ---------------- backward body
    w("template <typename T>")
    w("FC_HD FC_INLINE void bwd_body(const TpBwdParams<T>& P, int64_t row, int c, bool active, "
      "T* gw_keep) {")
    w("  const int F = P.F; const int c1 = P.F1 == 1 ? 0 : c; const int c2 = P.F2 == 1 ? 0 : c;")
    w("  const bool NEED_1 = P.g_in1 != nullptr, NEED_2 = P.g_in2 != nullptr, NEED_W = P.g_w != nullptr;")
    w("  T g[NACC];")
    w("  {")
    w("    const T* __restrict__ go = P.g_out + row * (int64_t)((P.reduce ? OUT_COMPS_RED : OUT_COMPS) * F) + c;")
    w("    if (!active) { for (int k = 0; k < NACC; ++k) g[k] = T(0); }")
    w("    else if (!P.reduce) {")
    for k, (nr, r) in enumerate(stores):
        w(f"      g[{k}] = fc_ldg(go + {nr} * F);")
    w("    } else {")
    for k, (nr, r) in enumerate(stores):
        w(f"      g[{k}] = fc_ldg(go + {r} * F);")
    w("    }")
    w("  }")
    w("  int64_t e0, e1;")
    w("  if (P.rowptr) { e0 = P.rowptr[row]; e1 = P.rowptr[row + 1]; } else { e0 = row; e1 = row + 1; }")
    w("  for (int64_t e = e0; e < e1; ++e) {")
    w("    const int64_t j = P.rowptr ? P.idx_j[e] : row;")
    w("    if ((uint64_t)j >= (uint64_t)P.n_in1) { fc_flag(P.status, FC_DEV_BAD_INDEX); continue; }")
    w("    const int cc = active ? c : 0;")
    w("    const int cc1 = active ? c1 : 0, cc2 = active ? c2 : 0;")
    w("    const T* __restrict__ a1 = P.in1 + j * (int64_t)(D1 * P.F1) + cc1;")
    w("    const T* __restrict__ a2 = P.in2 + e * (int64_t)(D2 * P.F2) + cc2;")
    w("    const T* __restrict__ wr = P.w + (P.shared_w ? 0 : e * (int64_t)(NP * F)) + cc;")
    w("    T x1[D1], x2[D2], gx1[D1], gx2[D2], gw[NP];")
    w("    for (int q = 0; q < D1; ++q) { x1[q] = fc_ldg(a1 + q * P.F1); gx1[q] = T(0); }")
    w("    for (int q = 0; q < D2; ++q) { x2[q] = fc_ldg(a2 + q * P.F2); gx2[q] = T(0); }")
    w("    for (int q = 0; q < NP; ++q) gw[q] = T(0);")
    w("#define WLOAD(p) fc_ldg(wr + (p) * F)")
    for p in range(sig.npaths):
        L.extend(bwd_path_code(sig, p, "    "))
    w("#undef WLOAD")
    w("    if (NEED_W) {")
    w("      if (P.shared_w) { for (int q = 0; q < NP; ++q) gw_keep[q] += gw[q]; }")
    w("      else if (active) { T* gwr = P.g_w + e * (int64_t)(NP * F) + c; "
      "for (int q = 0; q < NP; ++q) gwr[q * F] = gw[q]; }")
    w("    }")
    w("    if (NEED_1) fc_scatter_rows<T, D1>(P.g_in1 + j * (int64_t)(D1 * P.F1), P.F1, c1, gx1, active, "
      "P.rowptr != nullptr);")
    w("    if (NEED_2) fc_scatter_rows<T, D2>(P.g_in2 + e * (int64_t)(D2 * P.F2), P.F2, c2, gx2, active, false);")
    w("  }")
    w("}")
    w("")
    # ---------------- double backward body
    w("template <typename T>")
    w("FC_HD FC_INLINE void dbwd_body(const TpDbwdParams<T>& P, int64_t row, int c, bool active, "
      "T* dw_keep) {")
    w("  const int F = P.F; const int c1 = P.F1 == 1 ? 0 : c; const int c2 = P.F2 == 1 ? 0 : c;")
    w("  const bool NEED_DG = P.d_g != nullptr, NEED_DX1 = P.d_in1 != nullptr, "
      "NEED_DX2 = P.d_in2 != nullptr, NEED_DW = P.d_w != nullptr;")
    w("  const bool HAS_V1 = P.v1 != nullptr, HAS_V2 = P.v2 != nullptr, HAS_VW = P.vw != nullptr;")
    w("  const int cc = active ? c : 0, cc1 = active ? c1 : 0, cc2 = active ? c2 : 0;")
    w("  T g[NACC], dg[NACC];")
    w("  {")
    w("    const T* __restrict__ go = P.g_out + row * (int64_t)((P.reduce ? OUT_COMPS_RED : OUT_COMPS) * F) + cc;")
    w("    if (!active) { for (int k = 0; k < NACC; ++k) g[k] = T(0); }")
    w("    else if (!P.reduce) {")
    for k, (nr, r) in enumerate(stores):
        w(f"      g[{k}] = fc_ldg(go + {nr} * F);")
    w("    } else {")
    for k, (nr, r) in enumerate(stores):
        w(f"      g[{k}] = fc_ldg(go + {r} * F);")
    w("    }")
    w("    for (int k = 0; k < NACC; ++k) dg[k] = T(0);")
    w("  }")
    w("  int64_t e0, e1;")
    w("  if (P.rowptr) { e0 = P.rowptr[row]; e1 = P.rowptr[row + 1]; } else { e0 = row; e1 = row + 1; }")
    w("  for (int64_t e = e0; e < e1; ++e) {")
    w("    const int64_t j = P.rowptr ? P.idx_j[e] : row;")
    w("    if ((uint64_t)j >= (uint64_t)P.n_in1) { fc_flag(P.status, FC_DEV_BAD_INDEX); continue; }")
    w("    const int64_t r1 = j * (int64_t)(D1 * P.F1) + cc1, r2 = e * (int64_t)(D2 * P.F2) + cc2;")
    w("    const int64_t rw = (P.shared_w ? 0 : e * (int64_t)(NP * F)) + cc;")
    w("    T x1[D1], x2[D2], v1[D1], v2[D2], dx1[D1], dx2[D2], dw[NP];")
    w("    for (int q = 0; q < D1; ++q) { x1[q] = fc_ldg(P.in1 + r1 + q * P.F1); "
      "v1[q] = HAS_V1 ? fc_ldg(P.v1 + r1 + q * P.F1) : T(0); dx1[q] = T(0); }")
    w("    for (int q = 0; q < D2; ++q) { x2[q] = fc_ldg(P.in2 + r2 + q * P.F2); "
      "v2[q] = HAS_V2 ? fc_ldg(P.v2 + r2 + q * P.F2) : T(0); dx2[q] = T(0); }")
    w("    for (int q = 0; q < NP; ++q) dw[q] = T(0);")
    w("#define WLOAD(p) fc_ldg(P.w + rw + (p) * F)")
    w("#define VWLOAD(p) fc_ldg(P.vw + rw + (p) * F)")
    for p in range(sig.npaths):
        L.extend(dbwd_path_code(sig, p, "    "))
    w("#undef WLOAD")
    w("#undef VWLOAD")
    w("    if (NEED_DW) {")
    w("      if (P.shared_w) { for (int q = 0; q < NP; ++q) dw_keep[q] += dw[q]; }")
    w("      else if (active) { T* r = P.d_w + e * (int64_t)(NP * F) + c; "
      "for (int q = 0; q < NP; ++q) r[q * F] = dw[q]; }")
    w("    }")
    w("    if (NEED_DX1) fc_scatter_rows<T, D1>(P.d_in1 + j * (int64_t)(D1 * P.F1), P.F1, c1, dx1, active, "
      "P.rowptr != nullptr);")
    w("    if (NEED_DX2) fc_scatter_rows<T, D2>(P.d_in2 + e * (int64_t)(D2 * P.F2), P.F2, c2, dx2, active, false);")
    w("  }")
    w("  if (NEED_DG && active) {")
    w("    T* __restrict__ o = P.d_g + row * (int64_t)((P.reduce ? OUT_COMPS_RED : OUT_COMPS) * F) + c;")
    w("    if (!P.reduce) {")
    for k, (nr, r) in enumerate(stores):
        w(f"      o[{nr} * F] = dg[{k}];")
    w("    } else {")
    for r, ks in sorted(red.items()):
        # reduced layout: every path of the rank received the same g; its d_g is the sum
        w(f"      o[{r} * F] = {' + '.join(f'dg[{k}]' for k in ks)};")
    w("    }")
    w("  }")
    w("}")
    w("")
    w("#ifndef FC_HOST_EMU")
    L.append(emit_conv.emit(sig, stores))
    L.append(emit_pair.emit(sig, stores))
    L.append(emit_pair.emit_fwd4(sig, stores))
    L.append(emit_dense.emit(sig, stores))
    w("#endif")
    w("struct Ops {")
    w("  static constexpr int NP = sig_np, NACC = sig_nacc;".replace("sig_np", str(sig.npaths)).replace("sig_nacc", str(sig.nacc)))
    w("  template <typename T> FC_HD static FC_INLINE void fwd(const TpParams<T>& P, int64_t r, int c) "
      "{ fwd_body<T>(P, r, c); }")
    w("  template <typename T> FC_HD static FC_INLINE void bwd(const TpBwdParams<T>& P, int64_t r, int c, "
      "bool a, T* k) { bwd_body<T>(P, r, c, a, k); }")
    w("  template <typename T> FC_HD static FC_INLINE void dbwd(const TpDbwdParams<T>& P, int64_t r, int c, "
      "bool a, T* k) { dbwd_body<T>(P, r, c, a, k); }")
    w("#ifndef FC_HOST_EMU")
    w("  template <typename T> static int fwd2(const TpParams<T>& P, cudaStream_t s) { return launch_fwd2<T>(P, s); }")
    w("  template <typename T> static int bwd2(const TpBwdParams<T>& P, cudaStream_t s) "
      "{ return launch_bwd2<T>(P, s); }")
    w("  static int fwd3(const TpParams<float>& P, cudaStream_t s) { return launch_fwd3(P, s); }")
    w("  static int bwd3(const TpBwdParams<float>& P, cudaStream_t s) { return launch_bwd3(P, s); }")
    w("  static int dpfwd(const TpParams<float>& P, cudaStream_t s) { return launch_dpfwd(P, s); }")
    w("  static int dpbwd(const TpBwdParams<float>& P, cudaStream_t s) { return launch_dpbwd(P, s); }")
    w("  static constexpr int (*fwd4_fn)(const TpParams<float>&, cudaStream_t) = "
      + ("&launch_fwd4;" if emit_pair.has_fwd4(sig) else "nullptr;"))
    w("#endif")
    w("};")
    w(f"}}  // namespace sig_{n}")
    w("")
    w(f"FC_DEFINE_TP_SIGNATURE({n}, sig_{n})")
    w("}  // namespace fc")
    return "\n".join(L) + "\n"


def all_signatures(l_max: int = L_MAX) -> List[Sig]:
    sigs = []
    for l1 in range(l_max + 1):
        for l2 in range(l_max + 1):
            for lo in range(l_max + 1):
                s = Sig(l1, l2, lo, False)
                if s.npaths:
                    sigs.append(s)
                if l1 == l2:
                    s = Sig(l1, l2, lo, True)
                    if s.npaths:
                        sigs.append(s)
    return sigs


# ----------------------------------------------------------------------------------
# direction tensors (irreps) kernels
# ----------------------------------------------------------------------------------


def _poly_expr(poly: Dict[Tuple[int, int, int], Fraction]) -> str:
    terms = []
    for (px, py, pz), c in sorted(poly.items()):
        fac = ["x"] * px + ["y"] * py + ["z"] * pz
        v = "*".join(fac) if fac else "T(1)"
        terms.append((c, v))
    return lin(terms)


def emit_rms(l_max: int = L_MAX) -> str:
    """Invariant squared norms of stored rank blocks: rms_quad_l(x) = sum_ij K_l[i][j] x_i x_j
    with K_l the (l, l) -> 0 coupling of the tensor product (what the symmetric scalar
    product of the reference's RMS layer norm computes per channel), and its gradient
    (K_l + K_l^T) x."""
    L = []
    w = L.append
    w("// Generated by flashcart_b200/codegen/emit.py -- (l, l) -> 0 quadratic forms of stored STF")
    w(f"// components for l <= {l_max} (exact couplings of codegen/stf.py) and their gradients.")
    w('#include "../fc_base.cuh"')
    w("namespace fc {")
    for l in range(l_max + 1):
        K = stf.oriented_path_tensor(l, l, 0)
        n = 2 * l + 1
        terms = []
        for i in range(n):
            for j in range(i, n):
                c = K[0][i][j] if i == j else K[0][i][j] + K[0][j][i]
                if c != 0:
                    terms.append((c, f"x[{i}]*x[{j}]"))
        w("template <typename T>")
        w(f"FC_HD FC_INLINE T rms_quad_l{l}(const T* x) {{ return {lin(terms)}; }}")
        w("template <typename T>")
        w(f"FC_HD FC_INLINE void rms_quad_grad_l{l}(const T* x, T* g) {{")
        for m in range(n):
            gt = [(K[0][m][j] + K[0][j][m], f"x[{j}]") for j in range(n)]
            w(f"  g[{m}] = {lin(gt)};")
        w("}")
    w("}  // namespace fc")
    return "\n".join(L) + "\n"


def emit_irreps(l_max: int = L_MAX) -> str:
    L = []
    w = L.append
    w("// Generated by flashcart_b200/codegen/emit.py -- stored components of T^l(r) for l <= "
      f"{l_max} and their first and second derivatives (Eq. (1), Zaverkin et al. 2024).")
    w('#include "../irreps_common.cuh"')
    w("namespace fc {")
    # forward
    for lm in range(l_max + 1):
        w("template <typename T>")
        w(f"FC_HD FC_INLINE void irreps_fwd_l{lm}(T x, T y, T z, T* o) {{")
        k = 0
        for l in range(lm + 1):
            for poly in stf.irreps_polynomials(l):
                w(f"  o[{k}] = {_poly_expr(poly)};")
                k += 1
        w("}")
        # backward: g -> grad
        w("template <typename T>")
        w(f"FC_HD FC_INLINE void irreps_bwd_l{lm}(T x, T y, T z, const T* g, T* gx) {{")
        for ax, nm in enumerate("xyz"):
            pairs = []
            k = 0
            for l in range(lm + 1):
                for poly in stf.irreps_polynomials(l):
                    d = stf.poly_diff(poly, ax)
                    if d:
                        pairs.append((f"g[{k}]", _poly_expr(d)))
                    k += 1
            w(f"  gx[{ax}] = {prod_sum(pairs)};")
        w("}")
        # double backward: (g, v) -> d_g[a] = sum_k v_k dP_a/dx_k ; d_x[k] = sum_a g_a sum_j v_j d2P_a/dx_k dx_j
        w("template <typename T>")
        w(f"FC_HD FC_INLINE void irreps_dbwd_l{lm}(T x, T y, T z, const T* g, const T* v, T* dg, T* dx) {{")
        k = 0
        for l in range(lm + 1):
            for poly in stf.irreps_polynomials(l):
                pairs = []
                for ax, vn in enumerate(("v[0]", "v[1]", "v[2]")):
                    d = stf.poly_diff(poly, ax)
                    if d:
                        pairs.append((vn, _poly_expr(d)))
                w(f"  dg[{k}] = {prod_sum(pairs)};")
                k += 1
        for ax in range(3):
            pairs = []
            k = 0
            for l in range(lm + 1):
                for poly in stf.irreps_polynomials(l):
                    d1 = stf.poly_diff(poly, ax)
                    inner = []
                    for bx, vn in enumerate(("v[0]", "v[1]", "v[2]")):
                        d2 = stf.poly_diff(d1, bx)
                        if d2:
                            inner.append((vn, _poly_expr(d2)))
                    if inner:
                        pairs.append((f"g[{k}]", prod_sum(inner)))
                    k += 1
            w(f"  dx[{ax}] = {prod_sum(pairs)};")
        w("}")
    w(f"constexpr int IRREPS_L_MAX = {l_max};")
    w("}  // namespace fc")
    return "\n".join(L) + "\n"


def emit_dispatch(sigs: List[Sig]) -> str:
    L = ["// Generated by flashcart_b200/codegen/emit.py -- signature table.", "#pragma once",
         '#include "../tp_common.cuh"', "namespace fc {"]
    for s in sigs:
        L.append(f"FC_DECLARE_TP_SIGNATURE({s.name});")
    L.append("static const TpSigEntry kTpSignatures[] = {")
    for s in sigs:
        L.append(f"  {{{s.l1}, {s.l2}, {s.lo}, {1 if s.sym else 0}, {s.npaths}, &tp_table_{s.name}}},")
    L.append("};")
    L.append(f"static const int kNumTpSignatures = {len(sigs)};")
    L.append("}  // namespace fc")
    return "\n".join(L) + "\n"


def write_all(out_dir: str = GEN_DIR) -> List[str]:
    os.makedirs(out_dir, exist_ok=True)
    sigs = all_signatures()
    written = []
    for s in sigs:
        path = os.path.join(out_dir, f"tp_{s.name}.cu")
        _write_if_changed(path, emit_signature(s))
        written.append(path)
    _write_if_changed(os.path.join(out_dir, "tp_dispatch.inc"), emit_dispatch(sigs))
    _write_if_changed(os.path.join(out_dir, "irreps_poly.cuh"), emit_irreps())
    _write_if_changed(os.path.join(out_dir, "rms_quad.cuh"), emit_rms())
    return written


def _write_if_changed(path: str, text: str) -> None:
    if os.path.exists(path):
        with open(path) as f:
            if f.read() == text:
                return
    with open(path, "w") as f:
        f.write(text)


if __name__ == "__main__":
    files = write_all(sys.argv[1] if len(sys.argv) > 1 else GEN_DIR)
    print(f"wrote {len(files)} signature files")
