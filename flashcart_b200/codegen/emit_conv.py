"""Second-generation convolution kernels for edge attributes shared by all channels.

Emitted into each signature file by :mod:`flashcart_b200.codegen.emit`; used for the
interaction-layer case of the receiver-CSR convolution: ``in2_features == 1`` and
``in1_features == F`` (= blockDim, a multiple of 32, at most 256), per-edge weights,
paths not reduced.

Structure of one CTA (receiver ``blockIdx.x / groups``, path group ``blockIdx.x % groups``, so
the groups of a receiver run side by side and share its senders' rows in L2):

* the signature's paths are split into consecutive *groups* whose accumulators fit a
  register budget, so a thread never holds all outputs of a large signature;
* the receiver's edges are walked in chunks of ``EC`` = 32. Phase 1: the CTA computes
  for every edge of the chunk the channel-independent edge matrices
  ``M_p[a, i] = sum_j K_p[a, i, j] x2_j`` of the group's paths into shared memory
  (lane = edge, warp = a quarter of the entries). Phase 2: every thread (one channel)
  gathers ``x1`` of the sender and forms ``t_a = sum_i M_p[a, i] x1_i`` from broadcast
  shared-memory reads, accumulating ``w_p * t_a``.

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

EC = 32       # edges per chunk (one per lane in phase 1)
NPART = 4     # phase-1 work split (one part per warp of a 128-thread CTA)


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


def make_groups(sig, budget: int) -> List[List[int]]:
    """Consecutive path groups whose accumulator count (sum of 2lo+1) stays within budget."""
    groups, cur, used = [], [], 0
    for p, (r1, r2, o) in enumerate(sig.paths):
        n = 2 * o + 1
        if cur and used + n > budget:
            groups.append(cur)
            cur, used = [], 0
        cur.append(p)
        used += n
    if cur:
        groups.append(cur)
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


def _fwd_group_body(gs: GroupSlots, ind: str) -> List[str]:
    sig = gs.sig
    L = []
    acc_base = 0
    for p in gs.paths:
        r1, r2, o = sig.paths[p]
        s0 = gs.range[p][0]
        L.append(f"{ind}{{ // path {p}: ({r1},{r2})->{o}")
        L.extend(_path_mload(gs, p, ind + "  "))
        L.append(f"{ind}  const T wp = fc_ldg(wr + {p} * F);")
        for a in range(2 * o + 1):
            terms = [f"mv[{gs.index[(p, a, i)] - s0}]*x1[{_q(r1, i)}]" for i in range(2 * r1 + 1)
                     if (p, a, i) in gs.index]
            expr = " + ".join(terms) if terms else "T(0)"
            L.append(f"{ind}  acc[{acc_base + a}] += wp * ({expr});")
        L.append(f"{ind}}}")
        acc_base += 2 * o + 1
    return L


def _bwd_group_body(gs: GroupSlots, ind: str) -> List[str]:
    sig = gs.sig
    L = []
    base = 0
    for p in gs.paths:
        r1, r2, o = sig.paths[p]
        K = stf.oriented_path_tensor(r1, r2, o)
        s0 = gs.range[p][0]
        L.append(f"{ind}{{ // path {p}: ({r1},{r2})->{o}")
        L.extend(_path_mload(gs, p, ind + "  "))
        L.append(f"{ind}  const T wp = fc_ldg(wr + {p} * F);")
        hs = []
        for i in range(2 * r1 + 1):
            terms = [f"g[{base + a}]*mv[{gs.index[(p, a, i)] - s0}]" for a in range(2 * o + 1)
                     if (p, a, i) in gs.index]
            if terms:
                L.append(f"{ind}  const T h{i} = {' + '.join(terms)};")
                hs.append(i)
        gw = " + ".join(f"x1[{_q(r1, i)}]*h{i}" for i in hs) or "T(0)"
        L.append(f"{ind}  if (NEED_W) gwr[{p} * F] = {gw};")
        if hs:
            L.append(f"{ind}  if (NEED_1) {{")
            for i in hs:
                L.append(f"{ind}    gx1[{_q(r1, i)}] += wp * h{i};")
            L.append(f"{ind}  }}")
        body2 = []
        for j in range(2 * r2 + 1):
            pairs = []
            for a in range(2 * o + 1):
                n = _lin([(K[a][i][j], f"x1[{_q(r1, i)}]") for i in range(2 * r1 + 1)])
                if n != "T(0)":
                    pairs.append(f"g[{base + a}]*({n})")
            if pairs:
                body2.append(f"{ind}    gx2[{_q(r2, j)}] += wp * ({' + '.join(pairs)});")
        if body2:
            L.append(f"{ind}  if (NEED_2) {{")
            L.extend(body2)
            L.append(f"{ind}  }}")
        L.append(f"{ind}}}")
        base += 2 * o + 1
    return L


def emit(sig, store_offsets: List[Tuple[int, int]]) -> str:
    """Conv-v2 kernels of one signature (appended inside its namespace)."""
    fwd_groups = [GroupSlots(sig, g) for g in make_groups(sig, 64)]
    bwd_groups = [GroupSlots(sig, g) for g in make_groups(sig, 40)]
    d2p = 1
    while d2p < sig.d2:
        d2p *= 2
    L = []
    w = L.append
    w(f"// ---- conv v2 (shared edge attributes): {len(fwd_groups)} forward / {len(bwd_groups)} backward path groups")
    w(f"constexpr int FWD2_GROUPS = {len(fwd_groups)}, BWD2_GROUPS = {len(bwd_groups)};")
    w(f"constexpr int FWD2_SMEM_ELEMS = {max(g.nmp for g in fwd_groups) * EC};")
    w(f"constexpr int BWD2_SMEM_ELEMS = {max(g.nmp for g in bwd_groups) * EC + EC * d2p};")
    # accumulator index -> output offset (non reduced), per path
    acc_out = {}
    k = 0
    for p, (r1, r2, o) in enumerate(sig.paths):
        for a in range(2 * o + 1):
            acc_out[(p, a)] = store_offsets[k][0]
            k += 1
    # ---------------- forward
    for gi, gs in enumerate(fwd_groups):
        w("template <typename T>")
        w(f"__device__ __forceinline__ void fwd2_g{gi}(const TpParams<T>& P, T* sm) {{")
        w("  const int F = P.F, tid = threadIdx.x, c = tid;")
        w("  const int64_t row = blockIdx.x / FWD2_GROUPS;")
        w(f"  T acc[{gs.nacc}];")
        w(f"  for (int k = 0; k < {gs.nacc}; ++k) acc[k] = T(0);")
        w("  const int64_t e0 = P.rowptr[row], e1 = P.rowptr[row + 1];")
        w(f"  for (int64_t eb = e0; eb < e1; eb += {EC}) {{")
        w(f"    const int ne = (int)min((int64_t){EC}, e1 - eb);")
        w(f"    for (int t = tid; t < {EC * NPART}; t += blockDim.x) {{")
        w(f"      const int le = t % {EC}, part = t / {EC};")
        w("      if (le < ne) {")
        w("        T x2[D2];")
        w("        const T* __restrict__ a2 = P.in2 + (eb + le) * (int64_t)D2;")
        w("        for (int q = 0; q < D2; ++q) x2[q] = fc_ldg(a2 + q);")
        w(f"        T* m = sm + le * {gs.nmp};")
        L.extend(_phase1(gs, "        "))
        w("      }")
        w("    }")
        w("    __syncthreads();")
        w("    for (int k = 0; k < ne; ++k) {")
        w("      const int64_t e = eb + k;")
        w("      const int64_t j = P.idx_j[e];")
        w("      if ((uint64_t)j >= (uint64_t)P.n_in1) { if (c == 0) fc_flag(P.status, FC_DEV_BAD_INDEX); continue; }")
        w("      const T* __restrict__ a1 = P.in1 + j * (int64_t)(D1 * F) + c;")
        w("      T x1[D1];")
        w("      for (int q = 0; q < D1; ++q) x1[q] = fc_ldg(a1 + q * F);")
        w("      const T* __restrict__ wr = P.w + e * (int64_t)(NP * F) + c;")
        w(f"      const T* m = sm + k * {gs.nmp};")
        L.extend(_fwd_group_body(gs, "      "))
        w("    }")
        w("    __syncthreads();")
        w("  }")
        w("  T* __restrict__ o = P.out + row * (int64_t)(OUT_COMPS * F) + c;")
        k = 0
        for p in gs.paths:
            o_ = sig.paths[p][2]
            for a in range(2 * o_ + 1):
                w(f"  o[{acc_out[(p, a)]} * F] = acc[{k}];")
                k += 1
        w("}")
    w("template <typename T>")
    w("__global__ void __launch_bounds__(256, 2) fwd2_kernel(TpParams<T> P) {")
    w("  extern __shared__ __align__(16) unsigned char fc_smem_raw[];")
    w("  T* sm = reinterpret_cast<T*>(fc_smem_raw);")
    w("  switch (blockIdx.x % FWD2_GROUPS) {  // the groups of one receiver run side by side (shared x1 in L2)")
    for gi in range(len(fwd_groups)):
        w(f"    case {gi}: fwd2_g{gi}<T>(P, sm); break;")
    w("  }")
    w("}")
    # ---------------- backward
    for gi, gs in enumerate(bwd_groups):
        w("template <typename T>")
        w(f"__device__ __forceinline__ void bwd2_g{gi}(const TpBwdParams<T>& P, T* sm, bool multi) {{")
        w("  const int F = P.F, tid = threadIdx.x, c = tid;")
        w("  const bool NEED_1 = P.g_in1 != nullptr, NEED_2 = P.g_in2 != nullptr, NEED_W = P.g_w != nullptr;")
        w("  const int64_t row = blockIdx.x / BWD2_GROUPS;")
        w(f"  T* gsm = sm + {gs.nmp * EC};  // [EC][D2P] grad_in2 partial sums")
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
        w("  const int64_t e0 = P.rowptr[row], e1 = P.rowptr[row + 1];")
        w(f"  for (int64_t eb = e0; eb < e1; eb += {EC}) {{")
        w(f"    const int ne = (int)min((int64_t){EC}, e1 - eb);")
        w(f"    for (int t = tid; t < {EC * d2p}; t += blockDim.x) gsm[t] = T(0);")
        w(f"    for (int t = tid; t < {EC * NPART}; t += blockDim.x) {{")
        w(f"      const int le = t % {EC}, part = t / {EC};")
        w("      if (le < ne) {")
        w("        T x2[D2];")
        w("        const T* __restrict__ a2 = P.in2 + (eb + le) * (int64_t)D2;")
        w("        for (int q = 0; q < D2; ++q) x2[q] = fc_ldg(a2 + q);")
        w(f"        T* m = sm + le * {gs.nmp};")
        L.extend(_phase1(gs, "        "))
        w("      }")
        w("    }")
        w("    __syncthreads();")
        w("    for (int k = 0; k < ne; ++k) {")
        w("      const int64_t e = eb + k;")
        w("      const int64_t j = P.idx_j[e];")
        w("      if ((uint64_t)j >= (uint64_t)P.n_in1) { if (c == 0) fc_flag(P.status, FC_DEV_BAD_INDEX); continue; }")
        w("      const T* __restrict__ a1 = P.in1 + j * (int64_t)(D1 * F) + c;")
        w("      T x1[D1], gx1[D1];")
        w(f"      T gx2[{d2p}];")
        w("      for (int q = 0; q < D1; ++q) { x1[q] = fc_ldg(a1 + q * F); gx1[q] = T(0); }")
        w(f"      for (int q = 0; q < {d2p}; ++q) gx2[q] = T(0);")
        w("      const T* __restrict__ wr = P.w + e * (int64_t)(NP * F) + c;")
        w("      T* __restrict__ gwr = NEED_W ? P.g_w + e * (int64_t)(NP * F) + c : nullptr;")
        w(f"      const T* m = sm + k * {gs.nmp};")
        L.extend(_bwd_group_body(gs, "      "))
        w("      if (NEED_1) {")
        w("        T* __restrict__ t1 = P.g_in1 + j * (int64_t)(D1 * F) + c;")
        w("        for (int q = 0; q < D1; ++q) fc_atomic_add(t1 + q * F, gx1[q]);")
        w("      }")
        w("      if (NEED_2) {")
        w(f"        const int comp = fc_warp_transpose_reduce<T, {d2p}>(gx2);")
        w(f"        if ((threadIdx.x & {32 // d2p - 1}) == 0 && comp < D2) atomicAdd(gsm + k * {d2p} + comp, gx2[0]);")
        w("      }")
        w("    }")
        w("    __syncthreads();")
        w("    if (NEED_2) {")
        w(f"      for (int t = tid; t < ne * D2; t += blockDim.x) {{")
        w("        const int k = t / D2, q = t % D2;")
        w(f"        T* dst = P.g_in2 + (eb + k) * (int64_t)D2 + q;")
        w(f"        const T v = gsm[k * {d2p} + q];")
        w("        if (multi) atomicAdd(dst, v); else *dst = v;")
        w("      }")
        w("    }")
        w("    __syncthreads();")
        w("  }")
        w("}")
    w("template <typename T>")
    w("__global__ void __launch_bounds__(256, 2) bwd2_kernel(TpBwdParams<T> P) {")
    w("  extern __shared__ __align__(16) unsigned char fc_smem_raw[];")
    w("  T* sm = reinterpret_cast<T*>(fc_smem_raw);")
    w("  const bool multi = BWD2_GROUPS > 1;")
    w("  switch (blockIdx.x % BWD2_GROUPS) {")
    for gi in range(len(bwd_groups)):
        w(f"    case {gi}: bwd2_g{gi}<T>(P, sm, multi); break;")
    w("  }")
    w("}")
    w("template <typename T>")
    w("int launch_fwd2(const TpParams<T>& P, cudaStream_t s) {")
    w("  if (P.n_rows == 0) return 0;")
    w("  const size_t smem = FWD2_SMEM_ELEMS * sizeof(T);")
    w("  if (smem > 48 * 1024 && cudaFuncSetAttribute(fwd2_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return FC_ERR_LAUNCH;")
    w("  if (P.n_rows * FWD2_GROUPS > 0x7fffffffLL) return FC_ERR_UNSUPPORTED;")
    w("  fwd2_kernel<T><<<(unsigned)(P.n_rows * FWD2_GROUPS), P.F, smem, s>>>(P);")
    w("  return cudaGetLastError() == cudaSuccess ? 0 : FC_ERR_LAUNCH;")
    w("}")
    w("template <typename T>")
    w("int launch_bwd2(const TpBwdParams<T>& P, cudaStream_t s) {")
    w("  if (P.n_rows == 0) return 0;")
    w("  const size_t smem = BWD2_SMEM_ELEMS * sizeof(T);")
    w("  if (smem > 48 * 1024 && cudaFuncSetAttribute(bwd2_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return FC_ERR_LAUNCH;")
    w("  if (P.n_rows * BWD2_GROUPS > 0x7fffffffLL) return FC_ERR_UNSUPPORTED;")
    w("  bwd2_kernel<T><<<(unsigned)(P.n_rows * BWD2_GROUPS), P.F, smem, s>>>(P);")
    w("  return cudaGetLastError() == cudaSuccess ? 0 : FC_ERR_LAUNCH;")
    w("}")
    return "\n".join(L) + "\n"
