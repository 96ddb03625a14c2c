"""Convolution kernels for edge attributes shared by all channels.

Emitted into each signature file by :mod:`flashcart_b200.codegen.emit`; used for the
interaction-layer case of the receiver-CSR convolution: ``in2_features == 1`` and
``in1_features == F`` (= blockDim, a multiple of 32, at most 256), per-edge weights,
paths not reduced.

Structure of one CTA (one receiver ``blockIdx.x`` of one path group's launch):

* the signature's paths are split into *groups* whose accumulators fit a register
  budget; paths are taken in order of their in1 rank, so a group reads (and in the
  backward scatters) only a contiguous range of in1 components;
* every group is its own kernel launch (one code path per launch, so the instruction
  cache holds it, and its own register allocation); groups touch disjoint in1
  components, weights and outputs, so nothing is re-read across launches;
* a prefetch ring of ``RING`` slots streams, per edge, the group's in1 components of
  the sender row and the group's path weights of the edge into shared memory with
  1-D bulk async copies issued by thread 0 (completion on a per-slot mbarrier). After
  edge k thread 0 refills the slot of edge k-LAG+1, which the other warps have
  normally released already, so the gathers run RING-LAG+1 edges ahead of the
  arithmetic without a per-edge rendezvous of the warps;
* the receiver's edges are walked in chunks of ``EC``. Phase 1: the CTA computes for
  every edge of the chunk the channel-independent edge matrices
  ``M_p[a, i] = sum_j K_p[a, i, j] x2_j`` of the group's paths into shared memory.
  Phase 2: every thread (one channel) forms ``t_a = sum_i M_p[a, i] x1_i`` from
  broadcast shared-memory reads and accumulates ``w_p * t_a``.

Backward (same grouping, same M): ``h_i = sum_a g_a M_p[a, i]`` gives
``grad_w_p = sum_i x1_i h_i`` (stored per edge) and ``grad_x1_i += w_p h_i``
(scattered to the sender with ``red.global.add``); ``grad_x2_j = sum_c w_p sum_a g_a
sum_i K_p[a, i, j] x1_i`` is reduced over the warp by a transpose-reduce (each lane ends
with one component) and over warps with shared-memory atomics, then stored once per
edge per chunk (atomically when several groups contribute).
"""

from __future__ import annotations

from fractions import Fraction
from typing import Dict, List, Sequence, Tuple

from flashcart_b200.codegen import stf

EC = 16       # edges per chunk of phase 1 (32 measured 7% slower in the backward: one CTA less per SM)
NPART = 8     # phase-1 work split (EC x NPART = 128 threads)
RING = 4      # prefetch slots per CTA
BWD_RING_DEFAULT = True  # backward gathers through the prefetch ring (per-thread gathers measured 10% slower)

# Forward gathers: a signature kept as one path group streams its edges through the ring of
# bulk copies; a signature split into several groups loads sender rows and weights per
# thread (coalesced over channels), which measured faster there (C = 128, l <= 3).
BUDGET = 32   # accumulators (sum of 2lo+1) per path group when a signature is split
SINGLE_MAX = 40  # a signature with at most this many accumulators stays one group
LAG = 2       # a slot is refilled once the edge LAG-1 before the current one is released


def _const(fr: Fraction) -> str:
    return f"T({float(fr)!r})"


def _lin(terms: Sequence[Tuple[Fraction, str]]) -> str:
    parts = []
    for c, v in terms:
        if c == 0:
            continue
        if c == 1:
            parts.append(f"+{v}")
        elif c == -1:
            parts.append(f"-{v}")
        elif c > 0:
            parts.append(f"+{_const(c)}*{v}")
        else:
            parts.append(f"-{_const(-c)}*{v}")
    if not parts:
        return "T(0)"
    s = "".join(parts)
    return s[1:] if s[0] == "+" else s


def _q(r: int, i: int) -> int:
    return r * r + i


PURE_RANKS = True  # split a large signature at every change of in1 rank (measured fastest at C=128, l<=3)
MERGE_MAX = 40  # merge trailing groups up to this many accumulators (0: off): the in1-rank 1 and 0
# groups of (3,3)->3 as one, measured -8% backward / -3% forward; merging the leading two
# groups as well (59 accumulators) spilled, and 128 registers for every backward group lost
# more to occupancy than it gained


def make_groups(sig, budget: int) -> List[List[int]]:
    """Path groups (accumulator count, the sum of 2lo+1, within budget), filled in order of
    decreasing in1 rank so that each group touches a contiguous range of in1 components.
    Small signatures stay one group: their per-edge work is too small to pay for a launch
    and an edge walk per group."""
    if sum(2 * o + 1 for (_, _, o) in sig.paths) <= SINGLE_MAX:
        return [list(range(len(sig.paths)))]
    order = sorted(range(len(sig.paths)), key=lambda p: (-sig.paths[p][0], p))
    groups, cur, used = [], [], 0
    for p in order:
        n = 2 * sig.paths[p][2] + 1
        rank_change = PURE_RANKS and cur and sig.paths[cur[-1]][0] != sig.paths[p][0]
        if cur and (used + n > budget or rank_change):
            groups.append(sorted(cur))
            cur, used = [], 0
        cur.append(p)
        used += n
    if cur:
        groups.append(sorted(cur))
    # the lowest-rank groups are small: merge them while the union stays within MERGE_MAX
    # accumulators (each launch has a fixed per-edge cost: ring wait, reductions, indices)
    nacc = lambda g: sum(2 * sig.paths[p][2] + 1 for p in g)
    while MERGE_MAX and len(groups) > 1 and nacc(groups[-1]) + nacc(groups[-2]) <= MERGE_MAX:
        last = groups.pop()
        groups[-1] = sorted(groups[-1] + last)
    return groups


class GroupSlots:
    """M-matrix entries of a path group: slot s = (path, a, i) with a nonzero row K_p[a, i, :]."""

    def __init__(self, sig, paths: List[int]):
        self.sig = sig
        self.paths = paths
        self.slots: List[Tuple[int, int, int]] = []
        self.index: Dict[Tuple[int, int, int], int] = {}
        self.range: Dict[int, Tuple[int, int]] = {}
        for p in paths:
            r1, r2, o = sig.paths[p]
            K = stf.oriented_path_tensor(r1, r2, o)
            while len(self.slots) % 4:
                self.slots.append(None)  # each path's entries start 16-byte aligned
            start = len(self.slots)
            for a in range(2 * o + 1):
                for i in range(2 * r1 + 1):
                    if any(K[a][i][j] != 0 for j in range(2 * r2 + 1)):
                        self.index[(p, a, i)] = len(self.slots)
                        self.slots.append((p, a, i))
            self.range[p] = (start, len(self.slots))
        self.nm = len(self.slots)
        self.nmp = max(4, (self.nm + 3) // 4 * 4)  # padded row stride (16-byte multiple for float)
        self.nacc = sum(2 * sig.paths[p][2] + 1 for p in paths)
        ranks = [sig.paths[p][0] for p in paths]
        self.x_lo = min(ranks) ** 2                    # first in1 component read by the group
        self.x_n = (max(ranks) + 1) ** 2 - self.x_lo   # contiguous in1 components read
        self.w_pos = {p: k for k, p in enumerate(paths)}  # row of path p in the weight slice
        self.w_runs: List[Tuple[int, int, int]] = []   # (first path, count, first slice row)
        for k, p in enumerate(paths):
            if self.w_runs and self.w_runs[-1][0] + self.w_runs[-1][1] == p:
                f, n, r = self.w_runs[-1]
                self.w_runs[-1] = (f, n + 1, r)
            else:
                self.w_runs.append((p, 1, k))

    def m_expr(self, s: int, x2: str = "x2") -> str:
        if self.slots[s] is None:
            return "T(0)"
        p, a, i = self.slots[s]
        r1, r2, o = self.sig.paths[p]
        K = stf.oriented_path_tensor(r1, r2, o)
        return _lin([(K[a][i][j], f"{x2}[{_q(r2, j)}]") for j in range(2 * r2 + 1)])


def _phase1(gs: GroupSlots, ind: str) -> List[str]:
    """Edge-matrix entries split into NPART warp-uniform parts."""
    L = [f"{ind}switch (part) {{"]
    per = (gs.nm + NPART - 1) // NPART
    for part in range(NPART):
        L.append(f"{ind}  case {part}:")
        for s in range(part * per, min(gs.nm, (part + 1) * per)):
            if gs.slots[s] is not None:
                L.append(f"{ind}    m[{s}] = {gs.m_expr(s)};")
        L.append(f"{ind}    break;")
    L.append(f"{ind}}}")
    return L


def _mload(gs: GroupSlots, ind: str) -> List[str]:
    """Broadcast shared-memory loads of one edge's M row into registers mv[]."""
    n4 = (gs.nm + 3) // 4
    L = [f"{ind}T mv[{n4 * 4}];"]
    for k in range(n4):
        L.append(f"{ind}ld4(m + {4 * k}, mv + {4 * k});")
    return L


def _path_mload(gs: GroupSlots, p: int, ind: str) -> List[str]:
    """Broadcast shared-memory loads of one path's edge-matrix entries (16-byte vectors)."""
    s0, s1 = gs.range[p]
    n4 = (s1 - s0 + 3) // 4
    L = [f"{ind}T mv[{max(1, n4) * 4}];"]
    for k in range(n4):
        L.append(f"{ind}ld4(m + {s0 + 4 * k}, mv + {4 * k});")
    return L


def _fwd_group_body(gs: GroupSlots, ind: str, direct: bool = False) -> List[str]:
    sig = gs.sig
    L = []
    acc_base = 0
    for p in gs.paths:
        r1, r2, o = sig.paths[p]
        s0 = gs.range[p][0]
        L.append(f"{ind}{{ // path {p}: ({r1},{r2})->{o}")
        L.extend(_path_mload(gs, p, ind + "  "))
        wsrc = f"fc_ldg(wr + {p} * F)" if direct else f"sw[{gs.w_pos[p]} * F]"
        L.append(f"{ind}  const T wp = {wsrc};")
        for a in range(2 * o + 1):
            terms = [f"mv[{gs.index[(p, a, i)] - s0}]*x1[{_q(r1, i) - gs.x_lo}]" for i in range(2 * r1 + 1)
                     if (p, a, i) in gs.index]
            expr = " + ".join(terms) if terms else "T(0)"
            L.append(f"{ind}  acc[{acc_base + a}] += wp * ({expr});")
        L.append(f"{ind}}}")
        acc_base += 2 * o + 1
    return L


def _fwd_group_body_cpt(gs: GroupSlots, ind: str) -> List[str]:
    """Forward of one edge for CPT channels per thread (c + u*H, u < CPT): the edge matrix
    entries are loaded from shared memory once and used for every channel of the thread."""
    sig = gs.sig
    L = []
    acc_base = 0
    for p in gs.paths:
        r1, r2, o = sig.paths[p]
        s0 = gs.range[p][0]
        L.append(f"{ind}{{ // path {p}: ({r1},{r2})->{o}")
        L.extend(_path_mload(gs, p, ind + "  "))
        L.append(f"{ind}  T wp[CPT];")
        L.append(f"{ind}  for (int u = 0; u < CPT; ++u) wp[u] = fc_ldg(wr + {p} * F + u * H);")
        L.append(f"{ind}#pragma unroll")
        L.append(f"{ind}  for (int u = 0; u < CPT; ++u) {{")
        for a in range(2 * o + 1):
            terms = [f"mv[{gs.index[(p, a, i)] - s0}]*x1[u][{_q(r1, i) - gs.x_lo}]" for i in range(2 * r1 + 1)
                     if (p, a, i) in gs.index]
            expr = " + ".join(terms) if terms else "T(0)"
            L.append(f"{ind}    acc[u][{acc_base + a}] += wp[u] * ({expr});")
        L.append(f"{ind}  }}")
        L.append(f"{ind}}}")
        acc_base += 2 * o + 1
    return L


def _bwd_group_body(gs: GroupSlots, ind: str, d2p: int, direct: bool = False) -> List[str]:
    """Backward of one edge. The first contribution to a gradient register assigns it, so
    the registers need no zeroing per edge; components no path touches are zeroed last."""
    sig = gs.sig
    L = []
    base = 0
    set1, set2 = set(), set()

    def acc(name: str, k: int, expr: str, seen: set) -> str:
        op = "+=" if k in seen else "="
        seen.add(k)
        return f"{name}[{k}] {op} {expr};"
    for p in gs.paths:
        r1, r2, o = sig.paths[p]
        K = stf.oriented_path_tensor(r1, r2, o)
        s0 = gs.range[p][0]
        L.append(f"{ind}{{ // path {p}: ({r1},{r2})->{o}")
        L.extend(_path_mload(gs, p, ind + "  "))
        wsrc = f"fc_ldg(wr + {p} * F)" if direct else f"sw[{gs.w_pos[p]} * F]"
        L.append(f"{ind}  const T wp = {wsrc};")
        hs = []
        for i in range(2 * r1 + 1):
            terms = [f"g[{base + a}]*mv[{gs.index[(p, a, i)] - s0}]" for a in range(2 * o + 1)
                     if (p, a, i) in gs.index]
            if terms:
                L.append(f"{ind}  const T h{i} = {' + '.join(terms)};")
                hs.append(i)
        gw = " + ".join(f"x1[{_q(r1, i) - gs.x_lo}]*h{i}" for i in hs) or "T(0)"
        L.append(f"{ind}  if (NEED_W) gwr[{p} * F] = {gw};")
        if hs:
            L.append(f"{ind}  if (NEED_1) {{")
            for i in hs:
                L.append(f"{ind}    " + acc("gx1", _q(r1, i) - gs.x_lo, f"wp * h{i}", set1))
            L.append(f"{ind}  }}")
        body2 = []
        for j in range(2 * r2 + 1):
            pairs = []
            for a in range(2 * o + 1):
                n = _lin([(K[a][i][j], f"x1[{_q(r1, i) - gs.x_lo}]") for i in range(2 * r1 + 1)])
                if n != "T(0)":
                    pairs.append(f"g[{base + a}]*({n})")
            if pairs:
                body2.append(f"{ind}    " + acc("gx2", _q(r2, j), f"wp * ({' + '.join(pairs)})", set2))
        if body2:
            L.append(f"{ind}  if (NEED_2) {{")
            L.extend(body2)
            L.append(f"{ind}  }}")
        L.append(f"{ind}}}")
        base += 2 * o + 1
    for q in range(gs.x_n):
        if q not in set1:
            L.append(f"{ind}gx1[{q}] = T(0);")
    for q in range(d2p):
        if q not in set2:
            L.append(f"{ind}gx2[{q}] = T(0);")
    return L


def _ring_setup(gs: GroupSlots, extra_elems: str, ind: str) -> List[str]:
    """Shared-memory carve-up (M | ring slots | [extra] | mbarriers) and the first copies."""
    return [
        f"{ind}constexpr int XLO = {gs.x_lo}, XN = {gs.x_n}, NW = {len(gs.paths)}, NMP = {gs.nmp};",
        f"{ind}const int F = P.F, c = threadIdx.x, lane = c & 31;",
        f"{ind}T* sm = reinterpret_cast<T*>(smem);",
        f"{ind}T* ring = sm + NMP * {EC};",
        f"{ind}const int SLOT = (XN + NW) * F;",
        f"{ind}T* extra = ring + {RING} * SLOT;",
        f"{ind}uint64_t* full = reinterpret_cast<uint64_t*>(extra + {extra_elems});",
        f"{ind}uint64_t* empty = full + {RING};",
        f"{ind}volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + {RING});",
        f"{ind}const int64_t e0 = P.rowptr[row], ne_all = P.rowptr[row + 1] - e0;",
        f"{ind}if (c == 0) {{",
        f"{ind}  for (int s = 0; s < {RING}; ++s) {{ fc_mbar_init(&full[s], 1); fc_mbar_init(&empty[s], F >> 5); }}",
        f"{ind}  *abort_flag = 0;",
        f"{ind}  fc_mbar_init_fence();",
        f"{ind}}}",
        f"{ind}__syncthreads();",
    ]


def _issue_fn(gs: GroupSlots, ind: str) -> List[str]:
    """Thread 0: bulk copies of edge e0+kk (sender's in1 components, the group's weights)."""
    L = [f"{ind}int64_t issued = 0;",
         f"{ind}auto issue = [&](int64_t kk) {{",
         f"{ind}  issued = kk + 1;",
         f"{ind}  const int s = (int)(kk % {RING});",
         f"{ind}  const int64_t e = e0 + kk;",
         f"{ind}  const int64_t j = P.idx_j[e];",
         f"{ind}  const bool ok = (uint64_t)j < (uint64_t)P.n_in1;",
         f"{ind}  T* dst = ring + s * SLOT;",
         f"{ind}  fc_mbar_arrive_tx(&full[s], (uint32_t)(((ok ? XN : 0) + NW) * F * sizeof(T)));",
         f"{ind}  if (ok) fc_bulk_g2s(dst, P.in1 + j * (int64_t)(D1 * F) + XLO * F, (uint32_t)(XN * F * sizeof(T)), &full[s]);",
         f"{ind}  const T* wrow = P.w + e * (int64_t)(NP * F);"]
    for (p0, n, r) in gs.w_runs:
        L.append(f"{ind}  fc_bulk_g2s(dst + (XN + {r}) * F, wrow + {p0} * F, (uint32_t)({n} * F * sizeof(T)), &full[s]);")
    L.append(f"{ind}}};")
    L.append(f"{ind}if (c == 0) for (int64_t kk = 0; kk < ne_all && kk < {RING}; ++kk) issue(kk);")
    return L


def _ring_edge_begin(ind: str) -> List[str]:
    return [f"{ind}const int64_t kk = eb + k;",
            f"{ind}const int s = (int)(kk % {RING});",
            f"{ind}const bool landed = fc_mbar_wait(&full[s], (uint32_t)((kk / {RING}) & 1), abort_flag, P.status);",
            f"{ind}const int64_t e = e0 + kk;",
            f"{ind}const int64_t j = P.idx_j[e];",
            f"{ind}const bool valid = landed && (uint64_t)j < (uint64_t)P.n_in1;",
            f"{ind}if (landed && !valid && c == 0) fc_flag(P.status, FC_DEV_BAD_INDEX);"]


def _ring_edge_end(ind: str) -> List[str]:
    return [f"{ind}__syncwarp();",
            f"{ind}if (lane == 0) fc_mbar_arrive(&empty[s]);",
            f"{ind}if (c == 0) {{",
            f"{ind}  const int64_t r = kk - {LAG - 1};  // edge whose slot is refilled",
            f"{ind}  if (r >= 0 && r + {RING} < ne_all &&",
            f"{ind}      fc_mbar_wait(&empty[r % {RING}], (uint32_t)((r / {RING}) & 1), abort_flag, P.status))",
            f"{ind}    issue(r + {RING});",
            f"{ind}}}"]


def _ring_drain(ind: str) -> List[str]:
    """Thread 0: every issued copy has landed before the CTA exits (only an aborted
    CTA can have copies that no consumer waited for)."""
    return [f"{ind}if (c == 0 && *abort_flag) {{",
            f"{ind}  for (int64_t kk = issued > {RING} ? issued - {RING} : 0; kk < issued; ++kk)",
            f"{ind}    for (long long it = 0; it < FC_RING_WAIT_LIMIT; ++it)",
            f"{ind}      if (fc_mbar_test(&full[kk % {RING}], (uint32_t)((kk / {RING}) & 1))) break;",
            f"{ind}}}"]


def _phase1_loop(gs: GroupSlots, ind: str) -> List[str]:
    return [f"{ind}for (int t = c; t < {EC * NPART}; t += blockDim.x) {{",
            f"{ind}  const int le = t % {EC}, part = t / {EC};",
            f"{ind}  if (le < ne) {{",
            f"{ind}    T x2[D2];",
            f"{ind}    const T* __restrict__ a2 = P.in2 + (e0 + eb + le) * (int64_t)D2;",
            f"{ind}    for (int q = 0; q < D2; ++q) x2[q] = fc_ldg(a2 + q);",
            f"{ind}    T* m = sm + le * NMP;",
            *_phase1(gs, ind + "    "),
            f"{ind}  }}",
            f"{ind}}}",
            f"{ind}__syncthreads();"]


def emit(sig, store_offsets: List[Tuple[int, int]]) -> str:
    """Shared-attribute convolution kernels of one signature (appended inside its namespace)."""
    fwd_groups = [GroupSlots(sig, g) for g in make_groups(sig, BUDGET)]
    bwd_groups = [GroupSlots(sig, g) for g in make_groups(sig, BUDGET)]
    FWD_RING = len(fwd_groups) == 1
    BWD_RING = BWD_RING_DEFAULT

    def min_ctas(gs: GroupSlots) -> int:
        # __launch_bounds__(256, m): m = 3 caps a thread at 85 registers (5 CTAs of 128 threads
        # per SM), enough for up to 32 accumulators; larger groups keep 128 registers (m = 2)
        return 3 if gs.nacc <= BUDGET else 2
    d2p = 1
    while d2p < sig.d2:
        d2p *= 2
    L = []
    w = L.append
    w(f"// ---- shared-attribute convolution: {len(fwd_groups)} forward / {len(bwd_groups)} backward path groups")
    w(f"constexpr int BWD2_GROUPS = {len(bwd_groups)};")
    # shared memory per group (elements of T, F-dependent ring) + mbarriers / abort flag
    for kind, groups, extra in (("fwd", fwd_groups, 0), ("bwd", bwd_groups, EC * d2p)):
        w(f"inline size_t {kind}2_smem(int g, int F, size_t es) {{")
        w("  switch (g) {")
        for gi, gs in enumerate(groups):
            if (kind == "fwd" and not FWD_RING) or (kind == "bwd" and not BWD_RING):
                w(f"    case {gi}: return (size_t)({gs.nmp * EC} + {extra}) * es;")
                continue
            w(f"    case {gi}: return (size_t)({gs.nmp * EC} + {RING} * ({gs.x_n} + {len(gs.paths)}) * F + {extra}) * es"
              f" + {2 * RING * 8 + 16};")
        w("  }")
        w("  return 0;")
        w("}")
    acc_out = {}
    k = 0
    for p, (r1, r2, o) in enumerate(sig.paths):
        for a in range(2 * o + 1):
            acc_out[(p, a)] = store_offsets[k][0]
            k += 1
    # ---------------- forward
    for gi, gs in enumerate(fwd_groups):
        w("template <typename T, int CPT>")
        w(f"__device__ __forceinline__ void fwd2_g{gi}(const TpParams<T>& P, unsigned char* smem) {{")
        w("  const int64_t row = blockIdx.x;")
        if FWD_RING:
            w("  static_assert(CPT == 1, \"the prefetch ring maps one thread to one channel\");")
            L.extend(_ring_setup(gs, "0", "  "))
            L.extend(_issue_fn(gs, "  "))
            w(f"  T acc[{gs.nacc}];")
            w(f"  for (int q = 0; q < {gs.nacc}; ++q) acc[q] = T(0);")
        else:
            w(f"  constexpr int XLO = {gs.x_lo}, XN = {gs.x_n}, NMP = {gs.nmp};")
            w("  const int F = P.F, c = threadIdx.x, H = F / CPT;  // channels c + u*H, u < CPT")
            w("  T* sm = reinterpret_cast<T*>(smem);")
            w("  const int64_t e0 = P.rowptr[row], ne_all = P.rowptr[row + 1] - e0;")
            w(f"  T acc[CPT][{gs.nacc}];")
            w("  for (int u = 0; u < CPT; ++u)")
            w(f"    for (int q = 0; q < {gs.nacc}; ++q) acc[u][q] = T(0);")
        w(f"  for (int64_t eb = 0; eb < ne_all; eb += {EC}) {{")
        w(f"    const int ne = (int)min((int64_t){EC}, ne_all - eb);")
        L.extend(_phase1_loop(gs, "    "))
        w("    for (int k = 0; k < ne; ++k) {")
        if FWD_RING:
            L.extend(_ring_edge_begin("      "))
            w("      if (valid) {")
            w("        const T* sx = ring + s * SLOT + c;")
            w("        T x1[XN];")
            w("        for (int q = 0; q < XN; ++q) x1[q] = sx[q * F];")
            w("        const T* sw = sx + XN * F;")
            w("        const T* m = sm + k * NMP;")
            L.extend(_fwd_group_body(gs, "        "))
            w("      }")
            L.extend(_ring_edge_end("      "))
        else:
            w("      const int64_t e = e0 + eb + k;")
            w("      const int64_t j = P.idx_j[e];")
            w("      if ((uint64_t)j >= (uint64_t)P.n_in1) { if (c == 0) fc_flag(P.status, FC_DEV_BAD_INDEX); continue; }")
            w("      const T* __restrict__ a1 = P.in1 + j * (int64_t)(D1 * F) + XLO * F + c;")
            w("      T x1[CPT][XN];")
            w("      for (int u = 0; u < CPT; ++u)")
            w("        for (int q = 0; q < XN; ++q) x1[u][q] = fc_ldg(a1 + u * H + q * F);")
            w("      const T* __restrict__ wr = P.w + e * (int64_t)(NP * F) + c;")
            w("      const T* m = sm + k * NMP;")
            L.extend(_fwd_group_body_cpt(gs, "      "))
        w("    }")
        w("    __syncthreads();")
        w("  }")
        if FWD_RING:
            L.extend(_ring_drain("  "))
        w("  T* __restrict__ o = P.out + row * (int64_t)(OUT_COMPS * F) + c;")
        k = 0
        if not FWD_RING:
            w("  for (int u = 0; u < CPT; ++u) {")
        for p in gs.paths:
            o_ = sig.paths[p][2]
            for a in range(2 * o_ + 1):
                if FWD_RING:
                    w(f"  o[{acc_out[(p, a)]} * F] = acc[{k}];")
                else:
                    w(f"    o[{acc_out[(p, a)]} * F + u * H] = acc[u][{k}];")
                k += 1
        if not FWD_RING:
            w("  }")
        w("}")
    w("template <int G> struct Fwd2MinCtas;")
    for gi, gs in enumerate(fwd_groups):
        w(f"template <> struct Fwd2MinCtas<{gi}> {{ static constexpr int value = {min_ctas(gs)}; }};")
    # two channels per thread (64-thread CTAs at C = 128) when the signature is split into
    # groups: 128 registers (2 x the accumulators), the edge-matrix loads shared by both
    w(f"constexpr bool FWD2_CPT2 = {'false' if FWD_RING else 'true'};")
    w("template <typename T, int G, int CPT>")
    w("__global__ void __launch_bounds__(256, CPT == 1 ? Fwd2MinCtas<G>::value : 2) fwd2_kernel(TpParams<T> P) {")
    w("  extern __shared__ __align__(16) unsigned char fc_smem_raw[];")
    for gi in range(len(fwd_groups)):
        w(f"  if constexpr (G == {gi}) fwd2_g{gi}<T, CPT>(P, fc_smem_raw);")
    w("}")
    # ---------------- backward
    for gi, gs in enumerate(bwd_groups):
        w("template <typename T, int NM>")
        w(f"__device__ __forceinline__ void bwd2_g{gi}(const TpBwdParams<T>& P, unsigned char* smem, bool multi) {{")
        w("  // NM: requested gradients as a compile-time mask (1 in1, 2 in2, 4 weights), 0 = read the pointers")
        w("  const bool NEED_1 = NM ? (NM & 1) != 0 : P.g_in1 != nullptr;")
        w("  const bool NEED_2 = NM ? (NM & 2) != 0 : P.g_in2 != nullptr;")
        w("  const bool NEED_W = NM ? (NM & 4) != 0 : P.g_w != nullptr;")
        w("  const int64_t row = blockIdx.x;")
        if BWD_RING:
            L.extend(_ring_setup(gs, str(EC * d2p), "  "))
            w("  T* gsm = extra;  // [EC][D2P] grad_in2 partial sums")
            L.extend(_issue_fn(gs, "  "))
        else:
            w(f"  constexpr int XLO = {gs.x_lo}, XN = {gs.x_n}, NMP = {gs.nmp};")
            w("  const int F = P.F, c = threadIdx.x, lane = c & 31;")
            w("  T* sm = reinterpret_cast<T*>(smem);")
            w(f"  T* gsm = sm + NMP * {EC};  // [EC][D2P] grad_in2 partial sums")
            w("  const int64_t e0 = P.rowptr[row], ne_all = P.rowptr[row + 1] - e0;")
        w(f"  T g[{gs.nacc}];")
        w("  {")
        w("    const T* __restrict__ go = P.g_out + row * (int64_t)(OUT_COMPS * F) + c;")
        k = 0
        for p in gs.paths:
            o_ = sig.paths[p][2]
            for a in range(2 * o_ + 1):
                w(f"    g[{k}] = fc_ldg(go + {acc_out[(p, a)]} * F);")
                k += 1
        w("  }")
        w(f"  for (int64_t eb = 0; eb < ne_all; eb += {EC}) {{")
        w(f"    const int ne = (int)min((int64_t){EC}, ne_all - eb);")
        w(f"    for (int t = c; t < {EC * d2p}; t += blockDim.x) gsm[t] = T(0);")
        L.extend(_phase1_loop(gs, "    "))
        w("    for (int k = 0; k < ne; ++k) {")
        if BWD_RING:
            L.extend(_ring_edge_begin("      "))
            w("      if (valid) {")
            w("        const T* sx = ring + s * SLOT + c;")
            w("        T x1[XN], gx1[XN];")
            w(f"        T gx2[{d2p}];")
            w("        for (int q = 0; q < XN; ++q) x1[q] = sx[q * F];")
            w("        const T* sw = sx + XN * F;")
        else:
            w("      const int64_t kk = eb + k, e = e0 + kk;")
            w("      const int64_t j = P.idx_j[e];")
            w("      if ((uint64_t)j >= (uint64_t)P.n_in1) { if (c == 0) fc_flag(P.status, FC_DEV_BAD_INDEX); continue; }")
            w("      {")
            w("        const T* __restrict__ a1 = P.in1 + j * (int64_t)(D1 * F) + XLO * F + c;")
            w("        T x1[XN], gx1[XN];")
            w(f"        T gx2[{d2p}];")
            w("        for (int q = 0; q < XN; ++q) x1[q] = fc_ldg(a1 + q * F);")
            w("        const T* __restrict__ wr = P.w + e * (int64_t)(NP * F) + c;")
        w("        T* __restrict__ gwr = NEED_W ? P.g_w + e * (int64_t)(NP * F) + c : nullptr;")
        w("        const T* m = sm + k * NMP;")
        L.extend(_bwd_group_body(gs, "        ", d2p, direct=not BWD_RING))
        w("        if (NEED_1) {")
        w("          T* __restrict__ t1 = P.g_in1 + j * (int64_t)(D1 * F) + XLO * F + c;")
        w("          for (int q = 0; q < XN; ++q) fc_atomic_add(t1 + q * F, gx1[q]);")
        w("        }")
        w("        if (NEED_2) {")
        w(f"          const int comp = fc_warp_transpose_reduce<T, {d2p}>(gx2);")
        w(f"          if ((lane & {32 // d2p - 1}) == 0 && comp < D2) atomicAdd(gsm + k * {d2p} + comp, gx2[0]);")
        w("        }")
        w("      }")
        if BWD_RING:
            L.extend(_ring_edge_end("      "))
        w("    }")
        w("    __syncthreads();")
        w("    if (NEED_2) {")
        w(f"      for (int t = c; t < ne * D2; t += blockDim.x) {{")
        w("        const int k = t / D2, q = t % D2;")
        w(f"        T* dst = P.g_in2 + (e0 + eb + k) * (int64_t)D2 + q;")
        w(f"        const T v = gsm[k * {d2p} + q];")
        w("        if (multi) atomicAdd(dst, v); else *dst = v;")
        w("      }")
        w("    }")
        w("    __syncthreads();")
        w("  }")
        if BWD_RING:
            L.extend(_ring_drain("  "))
        w("}")
    w("template <int G> struct Bwd2MinCtas;")
    for gi, gs in enumerate(bwd_groups):
        w(f"template <> struct Bwd2MinCtas<{gi}> {{ static constexpr int value = {min_ctas(gs)}; }};")
    w("template <typename T, int G, int NM>")
    w("__global__ void __launch_bounds__(256, Bwd2MinCtas<G>::value) bwd2_kernel(TpBwdParams<T> P) {")
    w("  extern __shared__ __align__(16) unsigned char fc_smem_raw[];")
    for gi in range(len(bwd_groups)):
        w(f"  if constexpr (G == {gi}) bwd2_g{gi}<T, NM>(P, fc_smem_raw, BWD2_GROUPS > 1);")
    w("}")
    w("template <typename T, int G, int CPT>")
    w("int launch_fwd2_variant(const TpParams<T>& P, size_t smem, cudaStream_t s) {")
    w("  if (smem > 48 * 1024 && cudaFuncSetAttribute(fwd2_kernel<T, G, CPT>, "
      "cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return FC_ERR_LAUNCH;")
    w("  fwd2_kernel<T, G, CPT><<<(unsigned)P.n_rows, P.F / CPT, smem, s>>>(P);")
    w("  return fc_check_launch();")
    w("}")
    w("template <typename T, int G>")
    w("int launch_fwd2_group(const TpParams<T>& P, cudaStream_t s) {")
    w("  const size_t smem = fwd2_smem(G, P.F, sizeof(T));")
    w("  if (smem > 227 * 1024) return FC_ERR_UNSUPPORTED;")
    w("  if constexpr (FWD2_CPT2) {")
    w("    if (P.F % 64 == 0) return launch_fwd2_variant<T, G, 2>(P, smem, s);")
    w("  }")
    w("  return launch_fwd2_variant<T, G, 1>(P, smem, s);")
    w("}")
    w("template <typename T, int G, int NM>")
    w("int launch_bwd2_variant(const TpBwdParams<T>& P, size_t smem, cudaStream_t s) {")
    w("  if (smem > 48 * 1024 && cudaFuncSetAttribute(bwd2_kernel<T, G, NM>, "
      "cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return FC_ERR_LAUNCH;")
    w("  bwd2_kernel<T, G, NM><<<(unsigned)P.n_rows, P.F, smem, s>>>(P);")
    w("  return fc_check_launch();")
    w("}")
    w("template <typename T, int G>")
    w("int launch_bwd2_group(const TpBwdParams<T>& P, cudaStream_t s) {")
    w("  const size_t smem = bwd2_smem(G, P.F, sizeof(T));")
    w("  if (smem > 227 * 1024) return FC_ERR_UNSUPPORTED;")
    w("  // the gradient sets of the force / stress and training passes get their own code path")
    w("  const int nm = (P.g_in1 ? 1 : 0) | (P.g_in2 ? 2 : 0) | (P.g_w ? 4 : 0);")
    w("  if (nm == 7) return launch_bwd2_variant<T, G, 7>(P, smem, s);")
    w("  if (nm == 6) return launch_bwd2_variant<T, G, 6>(P, smem, s);")
    w("  return launch_bwd2_variant<T, G, 0>(P, smem, s);")
    w("}")
    for kind, params, groups in (("fwd", "TpParams", fwd_groups), ("bwd", "TpBwdParams", bwd_groups)):
        w("template <typename T>")
        w(f"int launch_{kind}2(const {params}<T>& P, cudaStream_t s) {{")
        w("  if (P.n_rows == 0) return 0;")
        w("  if (P.n_rows > 0x7fffffffLL) return FC_ERR_UNSUPPORTED;")
        for gi in range(len(groups)):
            w(f"  if (int rc = launch_{kind}2_group<T, {gi}>(P, s)) return rc;")
        w("  return 0;")
        w("}")
    return "\n".join(L) + "\n"
